"""Build ``libssd_b200.so`` in-tree with nvcc for sm_100a.

Usage: ``python -m selective_attention_b200._build`` (or ``build()`` from
``__graft_entry__``). Objects go to ``_build/`` at the repository root; the shared
library lands next to this file so it travels with the package.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD_DIR = os.path.join(ROOT, "_build")
LIB_NAME = "libssd_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

SOURCES = ["api.cu", "ssd_simt.cu", "ssd_tc.cu", "ssd_split.cu", "ssd_bwd.cu", "ssd_bwd_tc.cu", "ssu.cu", "ssm_conv.cu", "sattn.cu", "sattn_train.cu", "noalloc.cu"]
HEADERS = ["common.cuh", "sm100.cuh", "tmap.cuh", "sattn_tiles.cuh", "kernels.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
                "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; set NVCC or put CUDA's bin directory on PATH")
    return cand


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False, extra_flags=None) -> str:
    """Compile every source for sm_100a and link the shared library. Returns its path."""
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "ssd_b200.h")]
    flags = ARCH_FLAGS + COMMON_FLAGS + list(extra_flags or [])
    jobs = []
    objs = []
    for src in SOURCES:
        sp = os.path.join(CSRC, src)
        op = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
        objs.append(op)
        if force or _newer(op, [sp] + headers):
            jobs.append([nvcc, *flags, "-c", sp, "-o", op])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 1) or 1) as ex:
        list(ex.map(run, jobs))
    if force or jobs or _newer(LIB_PATH, objs):
        run([nvcc, *ARCH_FLAGS, "-shared", "-o", LIB_PATH, *objs])
    return LIB_PATH


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv,
          extra_flags=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None)
    print(LIB_PATH)
