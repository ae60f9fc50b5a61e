"""Build recipe of the CUDA library ``fable5_llm_b200/_lib/libf5b200.so``.

Every .cu under ``csrc/`` is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked into one shared
library with a plain C ABI (``include/f5b200.h``).  The library is built
in-tree so it travels with the repository snapshot; nothing is JIT-compiled
at import.

Usage: python -m fable5_llm_b200.build [--force] [--ptxas-v]
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIBDIR, "libf5b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE]


def nvcc():
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return (sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) +
            sorted(glob.glob(os.path.join(CSRC, "*.h"))) +
            [os.path.join(INCLUDE, "f5b200.h")])


def _compile(src, ptxas_v=False):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _sources() + _deps())


def build(force=False, ptxas_v=False, verbose=False):
    if not force and not ptxas_v and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        res = list(ex.map(lambda s: _compile(s, ptxas_v), srcs))
    if verbose or ptxas_v:
        for _, log in res:
            if log.strip():
                print(log, file=sys.stderr)
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *[o for o, _ in res],
           "-cudart", "shared", "-Xlinker", "-rpath,$ORIGIN"]
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, ptxas_v="--ptxas-v" in sys.argv, verbose=True)
    print(LIB)
