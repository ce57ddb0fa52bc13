"""Build the reference's RepLKNet depthwise kernels into oracle/_ref/ (test infrastructure).

    python oracle/build_ref.py [/path/to/luckychen-depthwise_conv]

Compiles, from where they lie in the reference checkout, the three kernel
sources that depend on the CUDA runtime only
(replknet/kernels/depthWise_ch_*_half_forward.cu), with the reference's own
nvcc flags (replknet/kernels/depthwise_replknet_nhwc_ops.py:43) for sm_100a,
plus oracle/ref_shim.cu, into oracle/_ref/libref_replknet.so.  Nothing is
copied into this repository.  The ConvMixer kernels
(convmixer/kernels/depthwise_integration.cu) include the PyTorch extension
headers and are not built (an external library).  Without the reference
checkout this is a no-op.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libref_replknet.so")
SOURCES = ["depthWise_ch_128_k_31_t_56_half_forward.cu", "depthWise_ch_256_k_29_t_28_half_forward.cu",
           "depthWise_ch_512_k_27_t_14_half_forward.cu"]


def build(ref_root: str = "/root/reference", verbose: bool = False) -> str | None:
    kdir = os.path.join(ref_root, "replknet", "kernels")
    if not os.path.isdir(kdir):
        return LIB if os.path.exists(LIB) else None
    srcs = [os.path.join(kdir, s) for s in SOURCES] + [os.path.join(HERE, "ref_shim.cu")]
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(s) for s in srcs):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
           "-use_fast_math", "-Xcompiler", "-fPIC", "-shared", "-I", kdir, *srcs, "-o", LIB]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference kernel build failed:\n{res.stdout}\n{res.stderr}")
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else "/root/reference", verbose=True))
