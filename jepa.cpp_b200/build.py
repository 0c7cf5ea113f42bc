"""Builds the engine's shared library, jepa.cpp_b200/lib/libjepa.so, for sm_100a.

Every .cu / .cpp under csrc/ is compiled by nvcc (-gencode arch=compute_100a,code=sm_100a, -fmad=false so
that no multiply-add is contracted where the reference rounds twice) and linked into one C-ABI
library with the CUDA runtime linked statically and NCCL from the Python environment's wheel.
Objects are rebuilt when their source or any header is newer. Run: python jepa.cpp_b200/build.py
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
OBJ = os.path.join(HERE, "lib", "obj")
LIB = os.path.join(HERE, "lib", "libjepa.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs() -> tuple[str, str]:
    """(include dir, lib dir) of the NCCL the Python environment ships (torch's own)."""
    try:
        import nvidia.nccl as n
        base = list(n.__path__)[0]
        return os.path.join(base, "include"), os.path.join(base, "lib")
    except Exception:
        return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def flags() -> list[str]:
    inc, _ = nccl_dirs()
    return ["-std=c++17", "-O3", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC,-fvisibility=hidden",
            "-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "-I" + inc] + ARCH


def compile_one(src: str) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    newest = max(os.path.getmtime(p) for p in [src] + headers)
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    cmd = [NVCC] + flags() + ["-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, "-x", "cu"] + flags() + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = True) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        _, nccl_lib = nccl_dirs()
        cmd = [NVCC, "-shared"] + ARCH + ["-o", LIB] + objs + [
            "-L" + nccl_lib, "-l:libnccl.so.2", "-Xlinker", "-rpath," + nccl_lib, "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    try:
        build()
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
