"""jepa_b200_gemm_noalloc, the GEMM entry point for callers that cannot allocate device memory (a fixed
device-memory budget, a real-time loop where an allocation could stall the device, a plug-in inside
someone else's allocator): through the C ABI its product must match jepa_b200_gemm's on the same host
buffers, call after call, although it keeps its device working set in one fixed array that every call
reuses. Collected last (file name), so a run that stops at the first failure has run everything else."""
import ctypes as C

import numpy as np
import pytest

from jepa_b200 import capi, lib as jlib

pytestmark = pytest.mark.gpu


def _lib():
    L = jlib.load()
    L.jepa_b200_gemm_noalloc.restype = C.c_int
    L.jepa_b200_gemm_noalloc.argtypes = [capi.FP, capi.FP, C.c_int, C.c_int, C.c_int, capi.FP]
    return L


def _both(L, M, N, K, seed):
    rng = np.random.default_rng(seed)
    A = rng.normal(size=(M, K)).astype(np.float32)
    B = rng.normal(size=(N, K)).astype(np.float32)
    c_ref = np.zeros((M, N), np.float32)
    c_new = np.full((M, N), np.nan, np.float32)
    assert L.jepa_b200_gemm(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(c_ref)) == 0, jlib.error_text()
    assert L.jepa_b200_gemm_noalloc(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(c_new)) == 0, jlib.error_text()
    return c_new, c_ref


def test_noalloc_matches_the_allocating_entry_point_twice():
    L = _lib()
    # two calls in a row: the second finds the first one's contents in the shared array
    for (M, N, K), seed in (((256, 384, 384), 1), ((200, 130, 100), 2)):
        c_new, c_ref = _both(L, M, N, K, seed)
        err = np.abs(c_new - c_ref).max() / np.abs(c_ref).max()
        assert err < 1e-5 * max(1.0, K / 1536), err   # the GEMM tests' bar


def test_noalloc_refuses_sizes_beyond_its_array():
    L = _lib()
    M = N = K = 1024                               # 3 (M K + N K) + M N = 7 Mi floats > 4 Mi
    A = np.zeros((M, K), np.float32)
    B = np.zeros((N, K), np.float32)
    Cm = np.zeros((M, N), np.float32)
    L.jepa_error_reset()
    assert L.jepa_b200_gemm_noalloc(capi.fptr(A), capi.fptr(B), M, N, K, capi.fptr(Cm)) == -1
    assert b"JEPA_B200_NOALLOC_MAX_FLOATS" in L.jepa_error_text()
