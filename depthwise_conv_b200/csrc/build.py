"""Build ``libdwconv_b200.so`` (the engine's C-ABI library) for sm_100a.

Compiles every ``*.cu`` in this directory with nvcc
(``-gencode arch=compute_100a,code=sm_100a``) and the planner with g++, in
parallel, into ``depthwise_conv_b200/_build/``, then links the shared library
into the package directory.  Objects are rebuilt only when a source or any
header is newer.  The library depends on the CUDA runtime only (no torch).

    python -m depthwise_conv_b200.csrc.build        # or: python build.py
    python -m depthwise_conv_b200.csrc.build --regcaps   # regenerate dw_regcaps.inc first

Register caps.  How many warps an SM holds is set by the registers per
thread in steps (64, 72, 80, 96, 128, 168, 255 registers = 8 ... 2 warps per
sub-partition), and ptxas's own choice often lands above a step it could reach
with no or almost no spilling.  ``--regcaps`` compiles every kernel variant
uncapped and then at each step below its natural count (``__maxnreg__``),
reads the registers and spill bytes ptxas reports, and picks a cap per variant
(``choose_caps``: a near-step rule for all, a low-spill rule for K <= 13).
The result is ``dw_regcaps.inc``, committed with the sources; a plain build
uses it.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import re
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


REGCAPS = os.path.join(HERE, "dw_regcaps.inc")
_STEPS = (64, 72, 80, 96, 128, 168)
_SPILL_STORES_OK = 16  # bytes of spill a cap may cost (a few loop-invariant words)
_SPILL_LOADS_OK = 16
_ENTRY = re.compile(r"Compiling entry function '\S*dw_stream_kernel(?:_capped)?ILi(\d+)ELi(\d+)ELi(\d+)ELi(\d+)ELi(\d+)E")
_USED = re.compile(r"Used (\d+) registers")
_SPILL = re.compile(r"(\d+) bytes spill stores, (\d+) bytes spill loads")


def _ptxas_report(src: str, extra: list[str]) -> dict:
    """{(K, R, M, acc, pre): (registers, spill store bytes, spill load bytes)} of one source file."""
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-Xptxas", "-v", "-I", INCLUDE, "-c", src, "-o", os.devnull]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    out, key, spill = {}, None, (0, 0)
    for line in res.stderr.splitlines():
        m = _ENTRY.search(line)
        if m:
            key, spill = tuple(int(v) for v in m.groups()), (0, 0)
            continue
        m = _SPILL.search(line)
        if m and key:
            spill = (int(m.group(1)), int(m.group(2)))
        m = _USED.search(line)
        if m and key:
            out[key] = (int(m.group(1)), *spill)
            key = None
    return out


def choose_caps(reports: dict) -> dict:
    """reports: {cap (255 = uncapped): {variant: (regs, spill stores, spill loads)}} -> {variant: cap}.

    Near-step rule: a variant at most 10 registers above a step is capped at that step if it then
    spills at most 32 bytes of stores.  Low-spill rule (K <= 13 only): the lowest step below the
    uncapped count whose spills stay within 16 bytes of stores and 16 of loads.  A variant takes
    the lower cap of the rules that apply (255 = no cap).  Measured on B200: the low-spill rule
    gains the small kernels a warp per sub-partition (k9 R16: 128 -> 96 registers), while the
    large ones, already FMA-bound with 4 warps, lost 2-3% under it."""
    caps = {}
    for key, (natural, _, _) in reports[255].items():
        cap = 255
        step = max((b for b in _STEPS if b <= natural), default=None)
        if step is not None and step < natural <= step + 10 and step in reports and key in reports[step]:
            regs, st, _ = reports[step][key]
            if regs <= step and st <= 32:
                cap = step
        if key[0] <= 13:
            for low in _STEPS:
                if low >= natural or low not in reports or key not in reports[low]:
                    continue
                regs, st, ld = reports[low][key]
                if regs <= low and st <= _SPILL_STORES_OK and ld <= _SPILL_LOADS_OK:
                    cap = min(cap, low)
                    break
        caps[key] = cap
    return caps


def _reports(extra: list[str]) -> dict:
    srcs = sorted(os.path.join(HERE, f) for f in os.listdir(HERE) if f.startswith("dw_kernels_k") and f.endswith(".cu"))
    merged = {}
    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 4)) as ex:
        for rep in ex.map(lambda f: _ptxas_report(f, extra), srcs):
            merged.update(rep)
    return merged


def write_caps(caps: dict) -> None:
    lines = ["// dw_regcaps.inc -- per-variant register caps, generated by build.py --regcaps.",
             "// {K, R, M, ACC, PRE, max registers}"]
    lines += ["{%d, %d, %d, %d, %d, %d}," % (*k, c) for k, c in sorted(caps.items()) if c < 255]
    with open(REGCAPS, "w") as f:
        f.write("\n".join(lines) + "\n")


def regcaps(verbose: bool = False) -> dict:
    """Regenerate dw_regcaps.inc from ptxas's register and spill counts (see the module docstring)."""
    reports = {255: _reports(["-DDWB_NO_REGCAPS"])}
    for step in _STEPS:
        reports[step] = _reports([f"-DDWB_FORCE_CAP={step}"])
    caps = choose_caps(reports)
    write_caps(caps)
    if verbose:
        for key in sorted(caps):
            if caps[key] < 255:
                print(f"K={key[0]} R={key[1]} M={key[2]} acc={key[3]} pre={key[4]}: "
                      f"{reports[255][key][0]} -> {caps[key]} registers")
    return caps


if __name__ == "__main__":
    if "--regcaps" in sys.argv:
        regcaps(verbose=True)
    print(build(verbose=True))
    sys.exit(0)
