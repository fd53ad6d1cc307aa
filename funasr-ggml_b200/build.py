"""Build libfunasr_dec.so (the C-ABI library) in-tree for sm_100a.

    python funasr-ggml_b200/build.py [--force] [--verbose]

Each CUDA translation unit is compiled with nvcc for exactly
`-gencode arch=compute_100a,code=sm_100a` (B200), objects go to
funasr-ggml_b200/_build/, the shared library to funasr-ggml_b200/libfunasr_dec.so.
The CUDA runtime is linked statically, so the library loads without PyTorch.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libfunasr_dec.so")
INCLUDE = os.path.join(ROOT, "include")

SOURCES = ["fa_api.cu", "k_append.cu", "k_attention.cu", "k_prefill_attn.cu", "k_gemm.cu", "k_gemm_tc.cu", "k_gemm_tc_skinny.cu", "k_gemv.cu", "k_row_step.cu", "k_small.cu",
           "gguf_file.cpp", "scheduler.cpp", "k_encoder.cu", "fa_encoder.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for cand in (os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"), shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (CUDA_HOME or PATH)")


def _deps(src: str):
    yield os.path.join(CSRC, src)
    for f in os.listdir(CSRC):
        if f.endswith((".cuh", ".hpp", ".h")):
            yield os.path.join(CSRC, f)
    yield os.path.join(INCLUDE, "funasr_dec.h")


def _stale(out: str, deps) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool, extra) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout, r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    objs = [os.path.join(BUILD, os.path.splitext(s)[0] + ".o") for s in SOURCES]
    todo = [s for s, o in zip(SOURCES, objs) if force or _stale(o, list(_deps(s)))]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            list(ex.map(lambda s: _compile(s, verbose, list(extra)), todo))
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-Xcompiler", "-fPIC"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem use per kernel")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra=extra))
    sys.exit(0)
