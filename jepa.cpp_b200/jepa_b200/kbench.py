"""Kernel microbenchmark: the planners' tcgen05 GEMMs at given shapes, through the C ABI.

    python -m jepa_b200.kbench M N K [reps] [--f16]
    python -m jepa_b200.kbench --attn n_cand n_frames rows heads hd [reps] [impl: 0 auto, 1 mma.sync, 2 tcgen05]

Prints the mean device time per launch (CUDA events) and the algorithmic TFLOP/s (2 M N K per launch).
Without --f16 it times the H-JEPA planner's 3xTF32 GEMM, with --f16 the V-JEPA 2-AC predictor's f16 GEMM.
--attn times the AC predictor's attention (the last frame's rows over all frames' keys).
Used for isolated kernel timing and as a small, self-contained target for ncu captures.
"""
from __future__ import annotations

import ctypes as C
import sys

from . import lib as jlib


def gemm(M: int, N: int, K: int, reps: int = 20, f16: bool = False) -> float:
    ms = C.c_double()
    L = jlib.load()
    fn = L.jepa_b200_gemm_f16_bench if f16 else L.jepa_b200_gemm_bench
    fn.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]
    if fn(M, N, K, reps, C.byref(ms)) != 0:
        raise RuntimeError(jlib.error_text())
    return ms.value


def attention(n_cand: int, n_frames: int, rows: int, heads: int, hd: int, reps: int = 20, impl: int = 0) -> float:
    ms = C.c_double()
    L = jlib.load()
    L.jepa_b200_attention_bench.argtypes = [C.c_int] * 7 + [C.POINTER(C.c_double)]
    if L.jepa_b200_attention_bench(n_cand, n_frames, rows, heads, hd, impl, reps, C.byref(ms)) != 0:
        raise RuntimeError(jlib.error_text())
    return ms.value


if __name__ == "__main__":
    if "--attn" in sys.argv:
        a = [int(x) for x in sys.argv[1:] if not x.startswith("--")]
        nc, nf, rows, heads, hd = a[:5]
        reps = a[5] if len(a) > 5 else 20
        impl = a[6] if len(a) > 6 else 0
        t = attention(nc, nf, rows, heads, hd, reps, impl)
        fl = 4.0 * nc * heads * hd * rows * (nf * rows)
        print(f"attention[{impl}] cand={nc} frames={nf} rows={rows} heads={heads} hd={hd}: {t * 1e3:.2f} us/launch, "
              f"{fl / (t * 1e-3) / 1e12:.2f} TFLOP/s")
        sys.exit(0)
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    f16 = "--f16" in sys.argv
    M, N, K = (int(x) for x in args[:3])
    reps = int(args[3]) if len(args) > 3 else 20
    t = gemm(M, N, K, reps, f16)
    kind = "f16" if f16 else "3xtf32"
    print(f"gemm[{kind}] M={M} N={N} K={K}: {t * 1e3:.2f} us/launch, {2.0 * M * N * K / (t * 1e-3) / 1e12:.2f} TFLOP/s")
