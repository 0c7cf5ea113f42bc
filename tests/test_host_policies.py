"""The planner's host-side policies against the reference's own code, on the CPU.

The engine restates the reference planner's host steps in its own structure (jepa.cpp_b200/csrc/
plan_policy.cpp, hplan_api.cpp); the steps decide which numbers the GPU sees, so they must agree
exactly. Here the receding-horizon schedule (jepa_hjepa_horizons) is compared, over many random level
horizons, pre-decay horizons, strides, replanning intervals and budgets, with the reference's
src/hjepa-plan.cpp built unmodified (oracle/_ref). The host GGUF row decoder (gguf.h dequant_row, which
the oracle's shim also uses) is pinned bit for bit against gguf-py, an independent implementation.
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
