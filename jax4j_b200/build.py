"""Builds libjax4j_cuda.so in-tree for sm_100a (B200) with nvcc.

    python -m jax4j_b200.build [--force] [-j N]

Every .cu file under jax4j_b200/csrc compiles to an object in
jax4j_b200/_build/ and links into jax4j_b200/libjax4j_cuda.so (NCCL from the
system, CUDA runtime static).  nvcc cross-compiles, so this runs without a GPU.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libjax4j_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                 "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"),
                 "-DJ4C_BUILDING_LIBRARY"]
LDFLAGS = ARCH + ["-shared", "-Xlinker", "--no-undefined", "-lnccl", "-lnvrtc", "-lcufft", "-lcusolver", "-ldl",
                  "-L/usr/local/cuda/lib64/stubs", "-Xlinker", "-rpath,/usr/local/cuda/lib64"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force, extra):
    obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
    if force or _stale(obj, [src] + _headers()):
        cmd = [NVCC] + CFLAGS + extra + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 8, verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, extra), srcs))
    if force or _stale(LIB, objs):
        cmd = [NVCC] + objs + LDFLAGS + ["-o", LIB]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    force = "--force" in sys.argv
    jobs = 8
    if "-j" in sys.argv:
        jobs = int(sys.argv[sys.argv.index("-j") + 1])
    print(build(force=force, jobs=jobs, verbose_ptxas="--ptxas-v" in sys.argv))
