"""Kernel parity on the GPU through the C ABI: the tcgen05 3xTF32 GEMM against a float64 product, and
the device dequantisation against the host restatement of the block formats (bit-exact)."""
import ctypes as C

import numpy as np
import pytest

from jepa_b200 import capi, lib as jlib
from jepa_b200.gguf_write import quantize_q4_0, quantize_q8_0

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 64, 32), (256, 384, 384), (200, 130, 100), (1, 8, 4), (512, 2304, 384),
                                   (256, 384, 1536), (4096, 1152, 384)])
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
