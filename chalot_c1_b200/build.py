"""Builds ``libchalot_b200.so`` in-tree for sm_100a.

CUDA sources are compiled with ``nvcc -gencode arch=compute_100a,code=sm_100a``
and ``--fmad=false`` (no float contraction on the parity-critical paths); host
sources with g++. The CUDA runtime is linked statically, so the library loads
on hosts without a GPU driver (symbol checks, file tools) and needs only
libcuda at run time.

    python -m chalot_c1_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "_lib")
# `python -m chalot_c1_b200.build --trace` builds a second library with the
# per-CTA phase trace compiled in (CHALOT_PHASE_TRACE; chalot_phase_trace()).
TRACE = os.environ.get("CHALOT_BUILD_TRACE") == "1"
BUILD = os.path.join(PKG, "_build_trace" if TRACE else "_build")
LIB = os.path.join(LIBDIR, "libchalot_b200_trace.so" if TRACE else "libchalot_b200.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(_nvcc())))


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + _headers())


def _compile(src: str, verbose: bool, ptxas_v: bool):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if src.endswith(".cu"):
        cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "--fmad=false", "-std=c++17",
               "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", CSRC, "-I", INCLUDE,
               "-c", src, "-o", obj] + (["-DCHALOT_PHASE_TRACE"] if TRACE else [])
        if ptxas_v:
            cmd[1:1] = ["-Xptxas", "-v"]
    else:
        cmd = ["g++", "-O2", "-fPIC", "-fvisibility=hidden", "-std=c++17", "-Wall",
               "-ffp-contract=off", "-I", CSRC, "-I", INCLUDE,
               "-I", os.path.join(_cuda_home(), "include"), "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{r.stdout}\n{r.stderr}")
    if ptxas_v and r.stderr:
        print(r.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    todo = [s for s in srcs if force or ptxas_v or _stale(os.path.join(BUILD, os.path.basename(s) + ".o"), s)]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(lambda s: _compile(s, verbose, ptxas_v), todo))
    objs = [os.path.join(BUILD, os.path.basename(s) + ".o") for s in srcs]
    if force or todo or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs,
               "-Xcompiler", "-fvisibility=hidden", "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem use per kernel")
    ap.add_argument("--trace", action="store_true", help="build the phase-trace library instead")
    a = ap.parse_args()
    if a.trace and not TRACE:
        os.environ["CHALOT_BUILD_TRACE"] = "1"
        os.execv(sys.executable, [sys.executable, "-m", "chalot_c1_b200.build"] +
                 [x for x in sys.argv[1:] if x != "--trace"])
    print(build(a.force, a.verbose, a.ptxas_v))
