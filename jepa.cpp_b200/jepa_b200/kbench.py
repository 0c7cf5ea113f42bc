"""Kernel microbenchmark: the planner's tcgen05 GEMM at given shapes, through the C ABI.

    python -m jepa_b200.kbench M N K [reps]

Prints the mean device time per launch (CUDA events) and the algorithmic TFLOP/s (2 M N K per launch).
Used for isolated kernel timing and as a small, self-contained target for ncu captures.
"""
from __future__ import annotations

import ctypes as C
import sys

from . import lib as jlib


def gemm(M: int, N: int, K: int, reps: int = 20) -> float:
    ms = C.c_double()
    if jlib.load().jepa_b200_gemm_bench(M, N, K, reps, C.byref(ms)) != 0:
        raise RuntimeError(jlib.error_text())
    return ms.value


if __name__ == "__main__":
    M, N, K = (int(x) for x in sys.argv[1:4])
    reps = int(sys.argv[4]) if len(sys.argv) > 4 else 20
    t = gemm(M, N, K, reps)
    print(f"gemm M={M} N={N} K={K}: {t * 1e3:.2f} us/launch, {2.0 * M * N * K / (t * 1e-3) / 1e12:.2f} TFLOP/s")
