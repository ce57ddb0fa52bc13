"""Build the reference's own depthwise kernels into oracle/_ref/ (TEST INFRASTRUCTURE ONLY).

    python oracle/build_ref.py [REFERENCE_ROOT]

The reference checkout is found from the argument, else the environment
variable ``DWB_REFERENCE_ROOT``, else the ``reference_path`` recorded in the
repository's BASELINE.json; without a checkout this is a no-op and the tests
that need these files skip.  Nothing from the reference is copied into this
repository: the sources are compiled where they lie, and only the built files
land in oracle/_ref/ (git-ignored; they travel to the GPU box with the tree).

Three products:

* ``libref_replknet.so`` -- the three RepLKNet kernel sources that depend on
  the CUDA runtime only (replknet/kernels/depthWise_ch_*_half_forward.cu),
  with the reference's own nvcc flags
  (replknet/kernels/depthwise_replknet_nhwc_ops.py:43) for sm_100a, plus
  oracle/ref_shim.cu (plain C entry points over their C interfaces);
* ``ext_convmixer/depthwise_convmixer.so`` -- the reference's ConvMixer
  extension (convmixer/kernels/depthwise_integration.cu), built exactly as its
  loader does (convmixer/kernels/depthwise_torch_ops.py:31-49:
  ``torch.utils.cpp_extension.load``, ``-O3 -std=c++17
  --expt-relaxed-constexpr -use_fast_math``) with TORCH_CUDA_ARCH_LIST=10.0a;
* ``ext_replknet/depthwise_replknet_nhwc_v2.so`` -- the reference's RepLKNet
  extension (replknet/kernels/depthwise_replknet_nhwc_ops.py:30-45: the
  integration file plus the three kernel files), built the same way.

Both extensions are PyTorch extension modules: they launch on PyTorch's
current stream, so they can be timed in CUDA graphs exactly like the engine.
``load_ext`` imports a built module by path without rebuilding (the GPU box
has no reference checkout).  ``depthwise_forward_32_1536_13`` of the ConvMixer
extension calls ``exit(1)`` (convmixer/kernels/depthwise_integration.cu:1013-1030)
and must never be called.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libref_replknet.so")
SOURCES = ["depthWise_ch_128_k_31_t_56_half_forward.cu", "depthWise_ch_256_k_29_t_28_half_forward.cu",
           "depthWise_ch_512_k_27_t_14_half_forward.cu"]
# the reference loaders' flags (depthwise_torch_ops.py:41-46, depthwise_replknet_nhwc_ops.py:43)
REF_CUDA_FLAGS = ["-O3", "-std=c++17", "--expt-relaxed-constexpr", "-use_fast_math"]
EXTENSIONS = {
    "depthwise_convmixer": ("ext_convmixer", ["convmixer/kernels/depthwise_integration.cu"], "convmixer/kernels"),
    "depthwise_replknet_nhwc_v2": ("ext_replknet", ["replknet/kernels/depthwise_replknet_nhwc_integration.cu"] +
                                   [f"replknet/kernels/{s}" for s in SOURCES], "replknet/kernels"),
}


def reference_root(explicit: str | None = None) -> str | None:
    """The reference checkout: argument, $DWB_REFERENCE_ROOT, or BASELINE.json's reference_path."""
    cands = [explicit, os.environ.get("DWB_REFERENCE_ROOT")]
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            cands.append(json.load(f).get("reference_path"))
    except (OSError, ValueError):
        pass
    for c in cands:
        if c and os.path.isdir(c):
            return c
    return None


def ext_path(name: str) -> str:
    sub, _, _ = EXTENSIONS[name]
    return os.path.join(OUT_DIR, sub, name + ".so")


def build_replknet_lib(ref_root: str, verbose: bool = False) -> str:
    kdir = os.path.join(ref_root, "replknet", "kernels")
    srcs = [os.path.join(kdir, s) for s in SOURCES] + [os.path.join(HERE, "ref_shim.cu")]
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(s) for s in srcs):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = os.environ.get("NVCC", "nvcc")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", *REF_CUDA_FLAGS, "-Xcompiler", "-fPIC", "-shared",
           "-I", kdir, *srcs, "-o", LIB]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference kernel build failed:\n{res.stdout}\n{res.stderr}")
    if verbose:
        print("built", LIB)
    return LIB


def build_ext(name: str, ref_root: str, verbose: bool = False) -> str:
    """Build one reference torch extension for sm_100a (a few minutes: PyTorch's headers)."""
    sub, rel_srcs, inc = EXTENSIONS[name]
    out = ext_path(name)
    srcs = [os.path.join(ref_root, s) for s in rel_srcs]
    if os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(s) for s in srcs):
        return out
    bdir = os.path.dirname(out)
    os.makedirs(bdir, exist_ok=True)
    # run the loader in a child process so the arch list and the import do not leak into this one
    code = (
        "import os, sys\n"
        "os.environ['TORCH_CUDA_ARCH_LIST'] = '10.0a'\n"
        "from torch.utils.cpp_extension import load\n"
        f"load(name={name!r}, sources={srcs!r}, extra_include_paths=[{os.path.join(ref_root, inc)!r}],\n"
        f"     extra_cuda_cflags={REF_CUDA_FLAGS!r}, build_directory={bdir!r}, verbose={verbose!r},\n"
        "     with_cuda=True)\n"
    )
    env = dict(os.environ, TORCH_CUDA_ARCH_LIST="10.0a", MAX_JOBS=str(os.cpu_count() or 4))
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env)
    if res.returncode != 0 or not os.path.exists(out):
        raise RuntimeError(f"reference extension {name} build failed:\n{res.stdout[-4000:]}\n{res.stderr[-4000:]}")
    if verbose:
        print("built", out)
    return out


def load_ext(name: str):
    """Import a built reference extension by path (no rebuild); None if it was not built."""
    path = ext_path(name)
    if not os.path.exists(path):
        return None
    import torch  # noqa: F401  (the extension links against the loaded libtorch)
    if name in sys.modules:
        return sys.modules[name]
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


def build(ref_root: str | None = None, verbose: bool = False, extensions: bool = True) -> str | None:
    """Build everything this machine's reference checkout allows; a no-op without one."""
    root = reference_root(ref_root)
    if root is None:
        return LIB if os.path.exists(LIB) else None
    build_replknet_lib(root, verbose)
    if extensions:
        for name in EXTENSIONS:
            build_ext(name, root, verbose)
    return LIB


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
