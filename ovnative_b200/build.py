"""Build libovb200.so in place (sm_100a only).

    python -m ovnative_b200.build [--force]

Each CUDA source is compiled with nvcc for ``-gencode arch=compute_100a,
code=sm_100a`` and linked, with the C ABI translation unit, into
``ovnative_b200/libovb200.so`` next to this file (the CUDA runtime is linked
statically, so the library needs only the driver at run time).  No fast-math
and no multiply-add contraction (``-fmad=false``): the quantisers and the
GEMM epilogue must reproduce the reference's fp32 rounding exactly.
``-Xptxas -v`` output (registers, spills, shared memory) is kept in
``_build/ptxas.log``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libovb200.so")

CU_SOURCES = ["quant.cu", "weights.cu", "gemm_tc.cu", "gemm_f16.cu", "linear_static.cu", "sampler.cu",
              "attention.cu", "lm_ops.cu"]
CXX_SOURCES = ["capi.cpp", "ovw1.cpp", "lm.cpp"]
HEADERS = ["ovb_internal.h", "ovb_ptx.cuh", "ovb_quant.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC",
          "-I" + os.path.join(ROOT, "include")]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "ovb200.h")]
    objs = []
    log = []
    for src in CU_SOURCES + CXX_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if not force and not _stale(o, [s] + hdrs + [__file__]):
            continue
        cmd = [nvcc, *ARCH, *COMMON, "-c", s, "-o", o]
        if src.endswith(".cu"):
            cmd.insert(1, "-Xptxas=-v")
        else:
            cmd += ["-x", "cu"]  # compiled by nvcc so the CUDA headers resolve identically
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        log.append(f"== {src}\n{r.stdout}{r.stderr}")
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError(f"nvcc failed on {src}")
    if force or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    if log:
        with open(os.path.join(BUILD, "ptxas.log"), "a") as f:
            f.write("\n".join(log))
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
