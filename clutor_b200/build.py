"""Builds libclutor_b200.so in place (sm_100a only) with nvcc.

    python -m clutor_b200.build [--verbose] [--ptxas-v]

--fmad=false keeps every float operation separately rounded, as the reference's C build is (no FMA contraction); the kernels
spell out the few fused multiply-adds they want.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
SOURCES = ["api.cu", "decode.cu", "group.cu", "batched.cu", "backend.cu", "noalloc.cu", "grouped_tc.cu", "cache.cpp", "store.cu", "gguf.cpp",
           "fwd.cu", "model.cu", "route.cu", "prefill.cu", "epx.cu"]
LIB = os.path.join(HERE, "libclutor_b200.so")


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def flags(ptxas_v: bool = False) -> list[str]:
    f = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "--fmad=false", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-O2", f"-I{os.path.join(ROOT, 'include')}", "--expt-relaxed-constexpr"]
    if ptxas_v:
        f += ["-Xptxas", "-v"]
    return f


def build(verbose: bool = False, ptxas_v: bool = False, force: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))] + [os.path.join(ROOT, "include", "clb200.h")]
    if not force and os.path.exists(LIB) and all(os.path.getmtime(d) <= os.path.getmtime(LIB) for d in deps):
        return LIB
    bdir = os.path.join(HERE, "_build")
    os.makedirs(bdir, exist_ok=True)

    def compile_one(s: str) -> str:
        o = os.path.join(bdir, os.path.basename(s) + ".o")
        cmd = [nvcc(), *flags(ptxas_v), "-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s}:\n{r.stdout}\n{r.stderr}")
        if ptxas_v or verbose:
            sys.stdout.write(r.stdout + r.stderr)
        return o

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        objs = list(pool.map(compile_one, srcs))
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC", *objs, "-o", LIB, "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"linking failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_v, a.force or a.ptxas_v))
