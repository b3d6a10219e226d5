"""Build the sm_100a sampler library in-tree.

    python -m noel_b200.build          # generate the expf table, compile the .so

Steps:
1. ``csrc/gen_expf_table.cc`` (host C++, OpenMP) lists the inputs of (-15, 0]
   where the C library's expf differs from the correctly rounded exp, into
   ``csrc/_gen/expf_table.inc``.  It calls the C library's expf on this host,
   so the table matches the libm the reference sampler links against.
2. nvcc compiles ``csrc/sampler_cuda.cu`` for sm_100a into
   ``noel_b200/libnoel_sampler_cuda.so`` (C ABI of include/sampler.h and
   include/noel_sampler_cuda.h).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
GEN = os.path.join(CSRC, "_gen")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libnoel_sampler_cuda.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, **kw)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def gen_table(force: bool = False) -> str:
    os.makedirs(GEN, exist_ok=True)
    src = os.path.join(CSRC, "gen_expf_table.cc")
    exe = os.path.join(GEN, "gen_expf_table")
    inc = os.path.join(GEN, "expf_table.inc")
    deps = [src, os.path.join(CSRC, "ref_expf.h")]
    if force or _stale(exe, deps):
        _run(["g++", "-O2", "-std=c++17", "-fopenmp", "-ffp-contract=off", src, "-o", exe, "-lm"])
    if force or _stale(inc, [exe]):
        _run([exe, inc, os.path.join(GEN, "expf_table.bin")])
    return inc


def build(force: bool = False, verbose: bool = False) -> str:
    inc = gen_table(force)
    srcs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))]
    srcs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    if force or _stale(LIB, srcs + [inc]):
        cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC,
               os.path.join(CSRC, "sampler_cuda.cu"), "-o", LIB + ".tmp"]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = _run(cmd)
        os.replace(LIB + ".tmp", LIB)
        if verbose:
            print(r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
