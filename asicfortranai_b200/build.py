"""Builds libq35.so in-tree with nvcc for sm_100a (B200).

    python -m asicfortranai_b200.build          # incremental
    python -m asicfortranai_b200.build --clean

Each csrc/*.cu compiles to an object under _build/ (parallel, skipped when up to
date), then the objects link into asicfortranai_b200/libq35.so against the CUDA runtime
and NCCL.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libq35.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "-Xcompiler", "-ffp-contract=off",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    # the flags live in this file: a change here rebuilds every object
    newest = max([os.path.getmtime(src), os.path.getmtime(os.path.abspath(__file__))] +
                 [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False, clean: bool = False) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        tmp = LIB + ".tmp"
        cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    build_cli()
    return LIB


CLI_SRC = os.path.join(PKG, "cli", "llama_generate.cpp")
CLI = os.path.join(PKG, "bin", "llama_generate")


def build_cli() -> str:
    """The llama_generate program (host C++ over libq35.so, found next to it at run time)."""
    newest = max(os.path.getmtime(CLI_SRC), os.path.getmtime(LIB), os.path.getmtime(os.path.abspath(__file__)))
    if os.path.exists(CLI) and os.path.getmtime(CLI) >= newest:
        return CLI
    os.makedirs(os.path.dirname(CLI), exist_ok=True)
    cxx = os.environ.get("CXX", "g++")
    cmd = [cxx, "-O2", "-std=c++17", "-Wall", "-I", os.path.join(ROOT, "include"), CLI_SRC, "-o", CLI + ".tmp",
           "-L", PKG, "-lq35", "-Wl,-rpath,$ORIGIN/.."]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building llama_generate failed:\n{r.stdout}\n{r.stderr}")
    os.replace(CLI + ".tmp", CLI)
    return CLI


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, clean="--clean" in sys.argv))
