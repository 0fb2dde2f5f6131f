"""Builds libb200dp.so in-tree for sm_100a (cross-compiles without a GPU).

    python dpa4c-scale-aware-md_b200/build.py [--force] [--jobs N]

Every CUDA source is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked into one
shared library next to this file.  Host code gets ``-ffp-contract=off`` so the
box inverse used by the neighbour builder matches the CPU oracle bit for bit.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libb200dp.so")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler",
                "-fPIC,-ffp-contract=off,-O3", "-ccbin", shutil.which("g++", path="/usr/bin") or "g++"]
SOURCES = ["nlist.cu", "sea.cu", "embed_tc.cu", "embed_f64.cu", "fit_tc.cu", "c8l2.cu", "engine.cu", "selftest.cu", "noalloc.cu", "md.cu",
           "dd.cu"]
HEADERS = ["common.cuh", "nlist.cuh", "sea.cuh", "engine.hpp", "model.hpp", "umma.cuh", "embed_tc.cuh", "embed_f64.cuh", "fit_tc.cuh",
           "c8l2.cuh", "simt_gemm.cuh", "md_kernels.cuh"]


def nccl_paths():
    """Include and library directories of the NCCL that PyTorch ships (the nvidia-nccl package), so
    that this library and torch load the same libnccl.so.2 in one process whichever comes first;
    the system NCCL when the package is absent."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia.nccl")
    if spec and spec.submodule_search_locations:
        root = list(spec.submodule_search_locations)[0]
        inc, lib = os.path.join(root, "include"), os.path.join(root, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
            return ["-I" + inc], ["-L" + lib, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + lib]
    return [], ["-lnccl"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, jobs: int = 4, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(HERE, "..", "include", "b200dp.h")]
    objs, todo = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            todo.append((s, o))

    nccl_inc, nccl_link = nccl_paths()

    def compile_one(so):
        s, o = so
        cmd = [NVCC] + FLAGS + nccl_inc + ["-c", s, "-o", o]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {s}:\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for out in ex.map(compile_one, todo):
            if verbose and out:
                sys.stderr.write(out)
    if force or todo or _stale(LIB, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static"] + nccl_link + ["-lrt", "-lpthread",
                                                                                                 "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=4)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))
