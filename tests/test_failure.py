"""Failure detection without a GPU fault.

Device side: every wait of the tensor-core kernels on an mbarrier is bounded; when the bound runs out the
kernel raises an error flag, frees its tensor memory and returns, the host reads the flag after the call
and the call returns -1. jepa_b200_check_wait_timeout runs that path on purpose (a wait on a barrier that
nothing arrives on, with a bound of about a millisecond), and the context has to stay usable after it.

Host side (no GPU): the reference's contract is 0 / -1 with the reason in jepa_error_text() for every
failure (reference: src/jepa.cpp:16-36); the NCCL set-up of the candidate sharding must return -1 instead
of hanging when a rank never joins."""
import ctypes as C

import numpy as np
import pytest

from jepa_b200 import capi, lib as jlib


@pytest.mark.gpu
def test_bounded_wait_runs_out_reports_and_leaves_the_context_usable():
    L = jlib.load()
    L.jepa_b200_check_wait_timeout.argtypes = [C.c_longlong, C.POINTER(C.c_int)]
    code = C.c_int(-5)
    assert L.jepa_b200_check_wait_timeout(2_000_000, C.byref(code)) == 0, jlib.error_text()
    assert code.value == 9
    # the flag was reset by its read: a GEMM right after runs and is correct
    rng = np.random.default_rng(1)
    A = rng.normal(size=(130, 96)).astype(np.float32)
    B = rng.normal(size=(70, 96)).astype(np.float32)
    Cm = np.zeros((130, 70), np.float32)
    assert L.jepa_b200_gemm(capi.fptr(A), capi.fptr(B), 130, 70, 96, capi.fptr(Cm)) == 0, jlib.error_text()
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    assert np.abs(Cm - ref).max() / np.abs(ref).max() < 1e-5
    # and the check itself repeats
    assert L.jepa_b200_check_wait_timeout(2_000_000, C.byref(code)) == 0 and code.value == 9


def test_timeout_check_refuses_bad_arguments():
    L = jlib.load()
    L.jepa_b200_check_wait_timeout.argtypes = [C.c_longlong, C.POINTER(C.c_int)]
    L.jepa_error_reset()
    assert L.jepa_b200_check_wait_timeout(0, C.byref(C.c_int())) == -1
    assert b"limit_cycles" in L.jepa_error_text()


_LONELY_RANK = r"""
import ctypes as C, os, sys, time
sys.path.insert(0, os.path.join(sys.argv[1], "jepa.cpp_b200"))
from jepa_b200 import lib as jlib
from jepa_b200.hjepa import Planner
P = Planner(sys.argv[2], device=0)
uid = C.create_string_buffer(128)
assert jlib.load().jepa_b200_nccl_unique_id(uid) == 0
t0 = time.time()
L = jlib.load()
L.jepa_b200_context_set_shard.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
rc = L.jepa_b200_context_set_shard(P.ctx, 0, 2, uid)
print("RC", rc, "S", round(time.time() - t0, 2), "MSG", jlib.error_text())
"""


@pytest.mark.gpu
def test_a_rank_that_never_joins_ends_in_an_error_not_a_hang(tmp_path):
    """Rank 0 of a 2-rank shard whose rank 1 never starts: the non-blocking NCCL set-up gives up after
    JEPA_B200_NCCL_TIMEOUT_MS, aborts the communicator and returns -1 with a reason (host-side failure; no
    kernel or collective is in flight). Run as a child process, itself bounded."""
    import os
    import subprocess
    import sys
    from jepa_b200 import synth
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    path = str(tmp_path / "tiny.gguf")
    synth.write_hjepa(path, synth.HJepaSpec(levels=[synth.Level(32, 1, 2, 64, 2)], ftype="f32"), seed=1)
    env = dict(os.environ, JEPA_B200_NCCL_TIMEOUT_MS="3000", NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", _LONELY_RANK, root, path], capture_output=True, text=True, timeout=120, env=env)
    line = [l for l in r.stdout.splitlines() if l.startswith("RC")]
    assert line, (r.stdout, r.stderr[-2000:])
    parts = line[0].split()
    assert parts[1] == "-1", line[0]
    assert float(parts[3]) < 60.0, line[0]
    assert "never joined" in line[0] or "did not complete" in line[0], line[0]
