"""The planner's host-side policies against the reference's own code, on the CPU.

The engine restates the reference planner's host steps in its own structure (jepa.cpp_b200/csrc/
plan_policy.cpp, hplan_api.cpp); the steps decide which numbers the GPU sees, so they must agree
exactly. Here the receding-horizon schedule (jepa_hjepa_horizons) is compared, over many random level
horizons, pre-decay horizons, strides, replanning intervals and budgets, with the reference's
src/hjepa-plan.cpp built unmodified (oracle/_ref). The host GGUF row decoder (gguf.h dequant_row, which
the oracle's shim also uses) is pinned bit for bit against gguf-py, an independent implementation.
The GEMM's dispatch (which kernel, how many K parts, which tile order a shape takes) is host arithmetic
too; its measured rules, and the row threshold that keeps a row's bits independent of its batch, are pinned
here.
"""
import ctypes as C
import os

import numpy as np
import pytest

import ref
from jepa_b200 import capi, synth
from jepa_b200 import lib as jlib

needs_ref = pytest.mark.skipif(not ref.available(), reason="oracle/_ref is not built (needs the reference tree)")


def _model(tmp, strides):
    levels = [synth.Level(32, 1, 2, 64, 2)]
    for s in strides:
        levels.append(synth.Level(32, 1, 2, 64, 4, stride=s, enc_kind="latent_mlp", act_enc_kind="mlp"))
    path = os.path.join(tmp, "sched-" + "-".join(map(str, strides)) + ".gguf")
    synth.write_hjepa(path, synth.HJepaSpec(levels=levels, ftype="f32"), seed=1)
    return path, len(levels)


@needs_ref
@pytest.mark.parametrize("strides", [(2,), (4,), (2, 3), (3, 2, 2)])
def test_horizon_schedule_matches_reference(tmp_path, strides):
    path, n = _model(str(tmp_path), strides)
    L = jlib.load()
    L.jepa_model_load.restype = C.c_void_p
    L.jepa_model_load.argtypes = [C.c_char_p, C.c_bool]
    L.jepa_model_free.argtypes = [C.c_void_p]
    capi.declare_planner(L)
    mine = L.jepa_model_load(path.encode(), False)
    assert mine, jlib.error_text()
    R = ref.RefPlanner(path)
    rng = np.random.default_rng(sum(strides))
    checked = 0
    for _ in range(60):
        rows = [capi.LevelPlan.of(horizon=int(rng.integers(1, 21)), pre_decay_horizon=int(rng.integers(0, 6)),
                                  n_samples=1, n_steps=1, lr=0.1, weight_decay=0.0, var_scale=1.0, action_noise=0.0,
                                  action_clip_sigma=0.0, min_its=0, early_stop_patience=0, early_stop_rel_delta=0.01,
                                  cost_last_n=1, intermediate_cost_weight=1.0, action_cost_weight=0.0, num_subgoals=1,
                                  horizon_one_goal_upper=0) for _ in range(n)]
        cfg = (capi.LevelPlan * n)(*rows)
        interval = int(rng.integers(1, 5))
        budget = int(rng.integers(1, 61))
        for step in range(0, budget + interval, interval):
            a, b = (C.c_int * n)(), (C.c_int * n)()
            ra = L.jepa_hjepa_horizons(mine, cfg, n, interval, budget, step, a)
            rb = R.lib.jepa_hjepa_horizons(R.model, cfg, n, interval, budget, step, b)
            assert ra == rb, (step, interval, budget)
            if ra == 0:
                assert list(a) == list(b), ([r.horizon for r in rows], [r.pre_decay_horizon for r in rows], interval, budget, step)
                checked += 1
    L.jepa_model_free(mine)
    R.close()
    assert checked > 100


def test_host_dequant_rows_match_gguf_py():
    """csrc/gguf.h dequant_row (the host decoder the weight loader and the oracle shim use), reached through
    the library's model loader: every f16 / q8_0 / q4_0 tensor of a written file decodes to gguf-py's values
    bit for bit."""
    gq = pytest.importorskip("gguf.quants")
    import gguf
    L = jlib.load()
    L.jepa_b200_host_dequant.argtypes = [C.c_uint32, C.c_void_p, C.c_int64, C.c_int64, capi.FP]
    L.jepa_b200_host_dequant.restype = C.c_int
    rng = np.random.default_rng(3)
    x = (rng.normal(size=(37, 96)) * rng.choice([1e-3, 1.0, 50.0], size=(37, 1))).astype(np.float32)
    x[0] = 0.0
    for qt, code in ((gguf.GGMLQuantizationType.Q8_0, 8), (gguf.GGMLQuantizationType.Q4_0, 2),
                     (gguf.GGMLQuantizationType.F16, 1)):
        blob = np.ascontiguousarray(gq.quantize(x, qt))
        want = gq.dequantize(blob, qt).astype(np.float32)
        got = np.zeros_like(x)
        assert L.jepa_b200_host_dequant(code, blob.ctypes.data, x.shape[0], x.shape[1], capi.fptr(got)) == 0
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), qt


def _gemm_plan(M, N, K):
    L = jlib.load()
    L.jepa_b200_gemm_plan.argtypes = [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)]
    L.jepa_b200_gemm_plan.restype = C.c_int
    out = (C.c_int * 3)()
    rc = L.jepa_b200_gemm_plan(M, N, K, out)
    return rc, tuple(out)


# (M, N, K) -> (persistent, K parts, grouped rows-fastest): the measured dispatch rules of the GEMM
@pytest.mark.parametrize("M,N,K,want", [
    (300, 768, 768, (1, 1, 0)),        # config 5's widths: persistent, whole tiles
    (256, 768, 768, (0, 0, 0)),        # at most two row tiles of a narrow output: split-K clusters
    (257, 768, 768, (1, 1, 0)),        # one row past the threshold
    (256, 55296, 768, (1, 1, 1)),      # adaLN modulation: wide output, 340 MB of B planes, two row tiles
    (128, 55296, 768, (1, 1, 0)),      # one row tile: nothing to group
    (2048, 4608, 768, (1, 1, 0)),      # one layer's modulation: 28 MB of B planes stays in L2
    (2048, 768, 55296, (1, 3, 0)),     # adaLN backward: narrow, long: K in three parts
    (1024, 768, 2048, (1, 3, 0)),      # the shortest split K
    (1024, 768, 2047, (1, 1, 0)),
    (1024, 1024, 3072, (1, 3, 0)),     # 8 column tiles
    (1024, 1025, 3072, (1, 1, 0)),     # 9 column tiles: enough to fill the device unsplit
    (1024, 3072, 3072, (1, 1, 0)),
    (1024, 512, 4096, (0, 0, 0)),      # narrow output, below 768
    (1024, 768, 512, (0, 0, 0)),       # short reduction
    (1024, 4096, 512, (1, 1, 0)),      # wide output, short reduction
])
def test_gemm_plan_rules(M, N, K, want):
    rc, got = _gemm_plan(M, N, K)
    assert rc == 0 and got == want, (M, N, K, got)


def test_gemm_plan_rejects_bad_shapes():
    assert _gemm_plan(0, 768, 768)[0] == -1
    assert _gemm_plan(16, -1, 768)[0] == -1


def test_gemm_plan_is_constant_on_each_side_of_the_row_threshold():
    """A row's arithmetic (kernel, K split) depends on the batch only through M <= 256: every batch on one side
    of it computes a row the same way, which is what makes a candidate's cost independent of how many other
    candidates share its batch (the tile order changes no value)."""
    rng = np.random.default_rng(5)
    shapes = [(768, 768), (768, 3072), (3072, 768), (768, 55296), (55296, 768), (384, 1536), (1536, 384)]
    shapes += [(int(rng.integers(1, 9000)), int(rng.integers(1, 9000))) for _ in range(40)]
    for N, K in shapes:
        small = {_gemm_plan(M, N, K)[1][:2] for M in (1, 17, 128, 129, 200, 256)}
        large = {_gemm_plan(M, N, K)[1][:2] for M in (257, 300, 1024, 4096, 65536, 131072)}
        assert len(small) == 1 and len(large) == 1, (N, K, small, large)
        if N >= 4096:
            assert small == large, (N, K)


def _tile_walk(M, N, K):
    L = jlib.load()
    L.jepa_b200_gemm_tile_walk.argtypes = [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int]
    L.jepa_b200_gemm_tile_walk.restype = C.c_int
    cap = ((M + 127) // 128) * ((N + 127) // 128)
    m0, n0 = (C.c_int * max(cap, 1))(), (C.c_int * max(cap, 1))()
    n = L.jepa_b200_gemm_tile_walk(M, N, K, m0, n0, cap)
    return n, np.array(m0[:max(n, 0)]), np.array(n0[:max(n, 0)])


@pytest.mark.parametrize("M,N,K", [
    (300, 768, 768), (2048, 3072, 768), (2048, 768, 55296),                 # n-fastest
    (256, 55296, 768), (2048, 55296, 768), (2100, 55296, 768),              # grouped: one group, whole, ragged
    (5000, 55296, 768), (131072, 55296, 768), (16 * 128 + 1, 8192, 8192),   # many groups, a one-tile last group
])
def test_gemm_tile_walk_visits_every_tile_once(M, N, K):
    """The persistent kernel's tile walk (its own origin function, run on the host) is a permutation of the
    output tiles: every tile is computed, none twice, whatever the group raggedness. In the grouped order the
    tiles that run side by side share a B column tile."""
    n, m0, n0 = _tile_walk(M, N, K)
    tm, tn = (M + 127) // 128, (N + 127) // 128
    assert n == tm * tn
    assert np.all(m0 % 128 == 0) and np.all(n0 % 128 == 0) and m0.max() < M and n0.max() < N
    keys = (m0 // 128) * tn + n0 // 128
    assert np.array_equal(np.sort(keys), np.arange(n))
    _, plan = _gemm_plan(M, N, K)
    if plan[2]:
        # within a group, consecutive tiles step down the rows of one column tile
        g = min(16, tm)
        assert np.all(n0[:g] == 0) and np.array_equal(m0[:g], np.arange(g) * 128)
    else:
        assert np.array_equal(keys, np.arange(n))


def test_gemm_tile_walk_refusals():
    n, _, _ = _tile_walk(256, 768, 768)          # split-K clusters: no persistent walk
    assert n == 0
    L = jlib.load()
    m0, n0 = (C.c_int * 4)(), (C.c_int * 4)()
    assert L.jepa_b200_gemm_tile_walk(1024, 1024, 1024, m0, n0, 4) == -1   # 64 tiles, room for 4
