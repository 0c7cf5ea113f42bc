"""Kernel parity on the GPU through the C ABI: the tcgen05 3xTF32 GEMM against a float64 product, and
the device dequantisation against the host restatement of the block formats (bit-exact)."""
import ctypes as C

import numpy as np
import pytest

from jepa_b200 import capi, lib as jlib
from jepa_b200.gguf_write import quantize_q4_0, quantize_q8_0

pytestmark = pytest.mark.gpu


# split-K 64-wide tiles (N or K < 768), and the 128-wide unsplit tiles (N, K >= 768, or N >= 4096) with ragged
# M and N edges
@pytest.mark.parametrize("M,N,K", [(2048, 768, 3072), (256, 768, 3072), (1024, 768, 2048), (2048, 768, 8192), (1024, 768, 12000),
                                   (300, 1000, 9000), (2048, 768, 55296), (130, 900, 8196), (200, 1000, 2052),
                                   (300, 800, 20000), (130, 768, 16384)])
def test_gemm_ksplit_matches_f64_and_the_unsplit_kernel(M, N, K):
    """The planner's configuration of the persistent GEMM: K split in three parts, the partial tiles summed
    in a fixed order by the part that finishes last (ragged M, N and K edges included)."""
    L = jlib.load()
    L.jepa_b200_gemm_ksplit.argtypes = [capi.FP, capi.FP, C.c_int, C.c_int, C.c_int, capi.FP]
    rng = np.random.default_rng(M + 3 * N + K)
    A = rng.normal(size=(M, K)).astype(np.float32)
    B = rng.normal(size=(N, K)).astype(np.float32)
    Cs = np.zeros((M, N), np.float32)
    Cu = np.zeros((M, N), np.float32)
    assert L.jepa_b200_gemm_ksplit(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(Cs)) == 0, jlib.error_text()
    assert L.jepa_b200_gemm(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(Cu)) == 0, jlib.error_text()
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    scale = np.abs(ref).max()
    assert np.abs(Cs - ref).max() / scale < 1e-5 * max(1.0, K / 1536)
    assert np.abs(Cs - Cu).max() / scale < 2e-5 * max(1.0, K / 1536)
    # deterministic: the parts are summed in a fixed order whichever finishes last
    C2 = np.zeros((M, N), np.float32)
    assert L.jepa_b200_gemm_ksplit(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(C2)) == 0
    assert np.array_equal(Cs, C2)


@pytest.mark.parametrize("M,N,K", [(128, 64, 32), (256, 384, 384), (200, 130, 100), (1, 8, 4), (512, 2304, 384),
                                   (256, 384, 1536), (4096, 1152, 384), (300, 768, 768), (257, 800, 1000),
                                   (130, 4100, 64), (33, 3072, 768)])
def test_gemm_3xtf32_matches_f64(M, N, K):
    L = jlib.load()
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.normal(size=(M, K)).astype(np.float32)
    B = rng.normal(size=(N, K)).astype(np.float32)
    Cm = np.zeros((M, N), np.float32)
    assert L.jepa_b200_gemm(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(Cm)) == 0, jlib.error_text()
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    err = np.abs(Cm - ref).max() / np.abs(ref).max()
    # 3xTF32 keeps ~21 bits per operand; the tensor core's accumulator rounds toward zero per instruction,
    # so the error grows with K / 8 (measured ~1e-6 at K = 384)
    assert err < 1e-5 * max(1.0, K / 1536), err


def test_gemm_grouped_tile_order_matches_f64_and_changes_no_value():
    """A wide output whose B planes do not fit in L2 (N 8192, K 1536: 100 MB) walks groups of 16 row tiles
    rows-fastest; at 2100 rows the last group holds one ragged row tile. Every tile is computed (f64 check),
    and a row's bits are those of a 1024-row batch of the same rows (walked in another order)."""
    L = jlib.load()
    L.jepa_b200_gemm_plan.argtypes = [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)]
    M, N, K = 2100, 8192, 1536
    for m in (M, 1024):
        plan = (C.c_int * 3)()
        assert L.jepa_b200_gemm_plan(m, N, K, plan) == 0 and tuple(plan) == (1, 1, 1)
    rng = np.random.default_rng(77)
    A = rng.normal(size=(M, K)).astype(np.float32)
    B = rng.normal(size=(N, K)).astype(np.float32)
    Cm = np.zeros((M, N), np.float32)
    assert L.jepa_b200_gemm(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(Cm)) == 0, jlib.error_text()
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    assert np.abs(Cm - ref).max() / np.abs(ref).max() < 1e-5
    A2 = np.ascontiguousarray(A[1000:2024])
    C2 = np.zeros((1024, N), np.float32)
    assert L.jepa_b200_gemm(capi.fptr(A2), capi.fptr(B), 1024, N, K, capi.fptr(C2)) == 0, jlib.error_text()
    assert np.array_equal(C2.view(np.uint32), Cm[1000:2024].view(np.uint32))


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (16, 1024, 1408), (300, 192, 96), (1, 8, 8), (1000, 3072, 1024),
                                   (517, 1024, 4096), (2064, 1408, 1024), (40000, 512, 256)])
def test_gemm_f16_matches_f64_of_f16_operands(M, N, K):
    """The AC predictor's tcgen05 kind::f16 GEMM (persistent, two TMEM accumulators) against a float64
    product of the same f16-rounded operands: only the f32 accumulation differs."""
    L = jlib.load()
    L.jepa_b200_gemm_f16.argtypes = [capi.FP, capi.FP, C.c_int, C.c_int, C.c_int, capi.FP]
    rng = np.random.default_rng(M * 3 + N + K)
    A = rng.normal(size=(M, K)).astype(np.float32)
    B = rng.normal(size=(N, K)).astype(np.float32)
    Cm = np.zeros((M, N), np.float32)
    assert L.jepa_b200_gemm_f16(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(Cm)) == 0, jlib.error_text()
    ref = A.astype(np.float16).astype(np.float64) @ B.astype(np.float16).astype(np.float64).T
    err = np.abs(Cm - ref).max() / np.abs(ref).max()
    assert err < 2e-5 * max(1.0, K / 1024), err


def _attention_ref(q, kv, n_frames, rows, heads, hd):
    """float64 softmax attention of the last frame's rows over every frame's keys, on f16-rounded inputs."""
    D = heads * hd
    q = q.astype(np.float16).astype(np.float64)
    kv = kv.astype(np.float16).astype(np.float64)
    out = np.zeros_like(q)
    for c in range(q.shape[0]):
        for h in range(heads):
            Q = q[c, :, h * hd:(h + 1) * hd]
            K = kv[c, :, h * hd:(h + 1) * hd]
            V = kv[c, :, D + h * hd:D + (h + 1) * hd]
            s = Q @ K.T / np.sqrt(hd)
            p = np.exp(s - s.max(1, keepdims=True))
            out[c, :, h * hd:(h + 1) * hd] = (p / p.sum(1, keepdims=True)) @ V
    return out


@pytest.mark.parametrize("impl", [1, 2])
@pytest.mark.parametrize("n_cand,n_frames,rows,heads,hd", [(3, 3, 258, 2, 64), (2, 1, 258, 3, 64), (2, 2, 100, 2, 64),
                                                             (1, 4, 384, 1, 64), (2, 2, 64, 2, 64), (3, 2, 18, 4, 16)])
def test_attention_matches_f64(impl, n_cand, n_frames, rows, heads, hd):
    """Both attention kernels (the mma.sync one and the tcgen05 one) against float64 on the same f16 inputs:
    P is rounded to f16 before the P V product, so the bar is 3e-3 of the output scale."""
    if impl == 2 and (hd != 64 or rows > 288):
        pytest.skip("the tcgen05 kernel takes head width 64 and at most 288 rows")
    L = jlib.load()
    L.jepa_b200_attention.argtypes = [capi.FP, capi.FP] + [C.c_int] * 6 + [capi.FP]
    rng = np.random.default_rng(n_cand * 100 + rows + heads)
    D = heads * hd
    q = rng.normal(size=(n_cand, rows, D)).astype(np.float32)
    kv = rng.normal(size=(n_cand, n_frames * rows, 2 * D)).astype(np.float32)
    out = np.zeros((n_cand, rows, D), np.float32)
    assert L.jepa_b200_attention(capi.fptr(q), capi.fptr(kv), n_cand, n_frames, rows, heads, hd, impl, capi.fptr(out)) == 0, \
        jlib.error_text()
    ref = _attention_ref(q, kv, n_frames, rows, heads, hd)
    err = np.abs(out - ref).max() / np.abs(ref).max()
    assert err < 3e-3, err


def _host_dequant(t, raw, rows, ne0):
    import gguf
    qt = {0: gguf.GGMLQuantizationType.F32, 1: gguf.GGMLQuantizationType.F16,
          2: gguf.GGMLQuantizationType.Q4_0, 8: gguf.GGMLQuantizationType.Q8_0}[t]
    return np.asarray(gguf.quants.dequantize(np.frombuffer(raw, np.uint8).reshape(rows, -1), qt), np.float32).reshape(rows, ne0)


@pytest.mark.parametrize("t", [0, 1, 2, 8])
def test_dequant_bit_exact(t):
    L = jlib.load()
    rng = np.random.default_rng(t)
    rows, ne0 = 37, 96
    x = rng.normal(0, 0.05, (rows, ne0)).astype(np.float32)
    raw = {0: x.tobytes(), 1: x.astype(np.float16).tobytes(), 2: quantize_q4_0(x), 8: quantize_q8_0(x)}[t]
    out = np.zeros((rows, ne0), np.float32)
    buf = C.create_string_buffer(raw, len(raw))
    assert L.jepa_b200_dequant(t, buf, rows, ne0, capi.fptr(out)) == 0, jlib.error_text()
    ref = _host_dequant(t, raw, rows, ne0)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
