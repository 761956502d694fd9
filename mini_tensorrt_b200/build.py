"""Builds libmtrtq.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m mini_tensorrt_b200.build        # or: python mini_tensorrt_b200/build.py

The library is compiled for sm_100a only (-gencode arch=compute_100a,code=sm_100a)
with the CUDA runtime linked statically, so it loads from any FFI without a
CUDA toolkit on the library path. Object files go to mini_tensorrt_b200/_build/.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmtrtq.so")
SOURCES = ["abi.cu", "prepack.cu", "gemv.cu", "gemv_cluster.cu", "gemv_stream.cu", "gemv_tc.cu", "decoder.cu",
           "gemm_tc.cu",
           "skinny_tc.cu", "shard.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "-I", os.path.join(HERE, "..", "include")]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _needs_rebuild() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(HERE, "..", "include", "mtrtq.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every source for sm_100a and link libmtrtq.so. Returns its path."""
    if not force and not _needs_rebuild():
        return LIB
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)

    def compile_one(src):
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        cmd = [nvcc, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        return obj, r.stderr

    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    objs = [o for o, _ in results]
    if verbose:
        for _, err in results:
            sys.stderr.write(err)
    tmp = LIB + ".tmp"
    r = subprocess.run([nvcc, *ARCH, "-shared", "-o", tmp, *objs], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
