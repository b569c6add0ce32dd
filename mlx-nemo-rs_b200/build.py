"""Builds libnemo_relpos.so in place: every CUDA source for sm_100a with
nvcc (-gencode arch=compute_100a,code=sm_100a -lineinfo), the C ABI host
code, statically linked against the CUDA runtime.

    python mlx-nemo-rs_b200/build.py [--force]
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
LIB = os.path.join(HERE, "libnemo_relpos.so")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr"]
SOURCES = ["gemm_sm100.cu", "gemm_tf32.cu", "attn_sm100.cu", "attn_simt.cu", "attn_stream.cu", "kernels_misc.cu",
           "noalloc.cu", "block_kernels.cu", "subsampling_kernels.cu", "api.cpp", "halo.cpp",
           "block.cpp", "subsampling.cpp"]


def _nccl_include():
    """Directory of nccl.h for halo.cpp (types and the config initializer
    only: the library is loaded with dlopen at run time).  The header of the
    NCCL that torch ships comes first, as that is the copy a torch process
    has loaded."""
    import sysconfig
    for base in (sysconfig.get_paths()["purelib"], sysconfig.get_paths()["platlib"]):
        d = os.path.join(base, "nvidia", "nccl", "include")
        if os.path.exists(os.path.join(d, "nccl.h")):
            return d
    for d in ("/usr/include", "/usr/local/cuda/include"):
        if os.path.exists(os.path.join(d, "nccl.h")):
            return d
    raise RuntimeError("nccl.h not found (needed to build halo.cpp)")


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force):
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD, src + ".o")
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    headers.append(os.path.join(os.path.dirname(HERE), "include", "nemo_relpos.h"))
    if not force and not _stale(obj, [path] + headers):
        return obj, ""
    cmd = [NVCC, *ARCH, *FLAGS, "-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, *FLAGS, "-x", "c++", "-c", path, "-o", obj]
        if src == "halo.cpp":
            cmd[1:1] = ["-I", _nccl_include()]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(lambda s: _compile(s, force), SOURCES))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log.strip():
                print(log)
    if force or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
