"""Build ``libdwconv_b200.so`` (the engine's C-ABI library) for sm_100a.

Compiles every ``*.cu`` in this directory with nvcc
(``-gencode arch=compute_100a,code=sm_100a``) and the planner with g++, in
parallel, into ``depthwise_conv_b200/_build/``, then links the shared library
into the package directory.  Objects are rebuilt only when a source or any
header is newer.  The library depends on the CUDA runtime only (no torch).

    python -m depthwise_conv_b200.csrc.build        # or: python build.py
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libdwconv_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the engine needs the CUDA toolkit to build")


def _headers_mtime() -> float:
    paths = [os.path.join(HERE, f) for f in os.listdir(HERE) if f.endswith((".cuh", ".h", ".inc"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths)


def _compile(src: str, obj: str, hdr_mtime: float) -> str:
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_mtime):
        return f"up to date: {os.path.basename(obj)}"
    if src.endswith(".cu"):
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
    else:
        cmd = ["g++", *CXX_FLAGS, "-I", INCLUDE, "-I", os.path.join(_cuda_home(), "include"), "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return f"compiled: {os.path.basename(obj)}"


def _cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(_nvcc())))


def build(verbose: bool = False, jobs: int | None = None) -> str:
    """Compile and link the library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(f for f in os.listdir(HERE) if f.endswith((".cu", ".cpp")))
    hdr = _headers_mtime()
    objs = [os.path.join(BUILD, os.path.splitext(s)[0] + ".o") for s in srcs]
    jobs = jobs or max(1, min(len(srcs), os.cpu_count() or 4))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for msg in ex.map(lambda so: _compile(os.path.join(HERE, so[0]), so[1], hdr), zip(srcs, objs)):
            if verbose:
                print(msg)
    newest_obj = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest_obj:
        cmd = [_nvcc(), *ARCH, "-shared", "--cudart", "static", "-o", LIB, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        if verbose:
            print(f"linked {LIB}")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
    sys.exit(0)
