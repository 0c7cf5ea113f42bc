"""jepa_b200_gemm_noalloc, the GEMM entry point for callers that cannot allocate device memory (a fixed
device-memory budget, a real-time loop where an allocation could stall the device, a plug-in inside
someone else's allocator): through the C ABI its product must equal jepa_b200_gemm's on the same host
buffers, call after call, although it keeps its device working set in one fixed array that every call
reuses. Collected last (file name), so a run that stops at the first failure has run everything else."""
import ctypes as C

import numpy as np
import pytest

from jepa_b200 import capi, lib as jlib

pytestmark = pytest.mark.gpu

MAX_FLOATS = 4 * 1024 * 1024   # JEPA_B200_NOALLOC_MAX_FLOATS


def _lib():
    L = jlib.load()
    L.jepa_b200_gemm_noalloc.restype = C.c_int
    L.jepa_b200_gemm_noalloc.argtypes = [capi.FP, capi.FP, C.c_int, C.c_int, C.c_int, capi.FP]
    return L


def _need(M, N, K):
    r = lambda n: (n + 63) // 64 * 64
    return 3 * (r(M * K) + r(N * K)) + r(M * N)


def _both(L, M, N, K, seed):
    rng = np.random.default_rng(seed)
    A = rng.normal(size=(M, K)).astype(np.float32)
    B = rng.normal(size=(N, K)).astype(np.float32)
    c_ref = np.zeros((M, N), np.float32)
    c_new = np.full((M, N), np.nan, np.float32)
    assert L.jepa_b200_gemm(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(c_ref)) == 0, jlib.error_text()
    assert L.jepa_b200_gemm_noalloc(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(c_new)) == 0, jlib.error_text()
    return c_new, c_ref


# split-K 64-wide tiles, ragged edges, the persistent 128 x 128 kernel (N, K >= 768), and a size that
# fills 98 % of the fixed array
SHAPES = [((256, 384, 384), 1), ((200, 130, 100), 2), ((512, 768, 768), 3), ((768, 768, 768), 4)]


def test_noalloc_matches_the_allocating_entry_point_call_after_call():
    L = _lib()
    assert _need(768, 768, 768) <= MAX_FLOATS < _need(832, 768, 768)
    # calls in a row: each finds the previous call's contents in the shared array; the same kernel on the
    # same shape gives the same bits as the allocating entry point
    for (M, N, K), seed in SHAPES + SHAPES[:2]:
        c_new, c_ref = _both(L, M, N, K, seed)
        assert np.array_equal(c_new, c_ref), (M, N, K, float(np.nanmax(np.abs(c_new - c_ref))))


def test_noalloc_allocates_no_device_memory():
    import torch
    L = _lib()
    M, N, K = 512, 768, 768
    rng = np.random.default_rng(9)
    A = rng.normal(size=(M, K)).astype(np.float32)
    B = rng.normal(size=(N, K)).astype(np.float32)
    Cm = np.zeros((M, N), np.float32)
    assert L.jepa_b200_gemm_noalloc(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(Cm)) == 0, jlib.error_text()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert L.jepa_b200_gemm_noalloc(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(Cm)) == 0, jlib.error_text()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def test_noalloc_refuses_sizes_beyond_its_array():
    L = _lib()
    M = N = K = 1024                               # 3 (M K + N K) + M N = 7 Mi floats > 4 Mi
    A = np.zeros((M, K), np.float32)
    B = np.zeros((N, K), np.float32)
    Cm = np.zeros((M, N), np.float32)
    L.jepa_error_reset()
    assert L.jepa_b200_gemm_noalloc(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(Cm)) == -1
    assert b"JEPA_B200_NOALLOC_MAX_FLOATS" in L.jepa_error_text()
