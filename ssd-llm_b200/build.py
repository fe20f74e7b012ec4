"""Builds the sm_100a backend into ssd-llm_b200/libssdllm_cuda.so (in-tree).

nvcc cross-compiles for sm_100a without a GPU. Objects are cached in
ssd-llm_b200/_build/ and rebuilt when their sources or headers change.
NCCL comes from the nvidia-nccl wheel that torch uses, so one libnccl.so.2
serves both torch.distributed and this library in a process.

Usage: python ssd-llm_b200/build.py [-v]   (-v adds -Xptxas -v register reports)
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libssdllm_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs():
    import importlib.util
    spec = importlib.util.find_spec("nvidia")
    for base in (spec.submodule_search_locations if spec else []):
        inc, lib = os.path.join(base, "nccl", "include"), os.path.join(base, "nccl", "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    raise RuntimeError("nccl.h not found (nvidia-nccl wheel)")


def flags(verbose=False):
    inc, _ = nccl_dirs()
    f = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-I" + os.path.join(ROOT, "include"), "-I" + inc] + ARCH
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def _stale(src, obj, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in [src] + deps)


def build(verbose: bool = False, jobs: int = 8) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(ROOT, "include", "ssdllm_cuda.h")]
    fl = flags(verbose)

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if not verbose and not _stale(src, obj, deps):
            return obj, ""
        cmd = [NVCC] + fl + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        return obj, r.stderr

    with cf.ThreadPoolExecutor(jobs) as ex:
        results = list(ex.map(compile_one, srcs))
    if verbose:
        for _, err in results:
            sys.stderr.write(err)
    objs = [o for o, _ in results]
    _, nlib = nccl_dirs()
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + [
            "-L" + nlib, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + nlib]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
