"""Build recipe for libqwen_b200.so (sm_100a only).

    python rust-ts-tokio-inference-engine_b200/build.py

Compiles every csrc/*.cu with nvcc for compute_100a/sm_100a into one shared
library under _lib/, in-tree, so it travels with the repository snapshot.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "_lib"
LIB = OUT / "libqwen_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-I/usr/local/cuda/include",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall", "--expt-relaxed-constexpr"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "qwen_b200.h"]


def build(force: bool = False, verbose: bool = False) -> Path:
    OUT.mkdir(exist_ok=True)
    hdr_time = max(p.stat().st_mtime for p in headers())
    objs = []
    jobs = []
    for src in sources():
        obj = OUT / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time):
            jobs.append([NVCC, *FLAGS, "-c", str(src), "-o", str(obj)] + (["-Xptxas", "-v"] if verbose else []))
    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stderr
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for log in ex.map(run, jobs):
            if verbose and log:
                print(log, file=sys.stderr)
    if force or jobs or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        subprocess.run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs),
                        "-o", str(tmp), "-lcudart", "-lnccl"], check=True)
        tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
