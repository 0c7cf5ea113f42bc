"""Parity pins against the reference's own planner.

tests/golden/hjepa_ref.npz holds outputs of the reference's src/hjepa-plan.cpp (built unmodified against
the ggml shim, oracle/_ref) on seeded forged models; tests/golden/make_golden.py wrote it. The cases include
the action cost (candidates pooled by the upper level's 'mlp' and 'seq' action encoders, action_cost_weight
!= 0) on its own and inside the hierarchy.

CPU (always): the oracle restatement reproduces every case; the engine's host-side horizon schedule
(jepa_hjepa_horizons) matches exactly; the models rebuild byte for byte (sha256).
GPU (-m gpu): the engine's GPU planner reproduces every case through the C ABI.
"""
import ctypes as C
import json
import os

import numpy as np
import pytest

import hjepa_oracle as O
from jepa_b200 import capi
from jepa_b200 import lib as jlib

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = np.load(os.path.join(HERE, "golden", "hjepa_ref.npz"))
META = json.loads(bytes(GOLDEN["meta"]))
CASES = META["cases"]


def _make_golden_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(HERE, "golden", "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    mg = _make_golden_module()
    d = str(tmp_path_factory.mktemp("golden"))
    out = {}
    for name, digest in META["models"].items():
        path, h = mg.build_model(name, d)
        assert h == digest, f"forged model {name} does not rebuild byte for byte"
        out[name] = path
    return out


def g(key, name):
    return GOLDEN[f"{key}.{name}"]


def rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(np.asarray(b)).max(), 1e-30))


# ---------------------------------------------------------------------------------------------
# oracle vs the reference (CPU)
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "cost"], ids=lambda c: c["key"])
def test_oracle_cost_matches_reference(models, case):
    m = O.Model(models[case["model"]])
    k = case["key"]
    cs = O.CostSpec(level=case["level"], horizon=case["horizon"], s0=g(k, "s0"), goal=g(k, "goal"), n_goal=case["n_goal"],
                    goal_level=case["goal_level"], dense=bool(case["dense"]), cost_last_n=case["plan"]["cost_last_n"],
                    intermediate_cost_weight=case["plan"]["intermediate_cost_weight"],
                    goal_action=g(k, "goal_action") if case.get("goal_action") else None,
                    action_cost_weight=case["plan"]["action_cost_weight"])
    costs, grad, _ = O.batch_cost(m, cs, g(k, "actions"))
    assert rel(costs, g(k, "costs")) < 1e-5
    assert rel(grad, g(k, "grad")) < 1e-4


@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "solve"], ids=lambda c: c["key"])
def test_oracle_solve_matches_reference(models, case):
    m = O.Model(models[case["model"]])
    k = case["key"]
    lp = case["plan"]
    cs = O.CostSpec(level=1, horizon=lp["horizon"], s0=g(k, "s0"), goal=g(k, "goal"))
    a, st, c, it = O.solve_level(m, cs, lp, O.replay(g(k, "draws")))
    assert it == int(g(k, "iters")[0])
    assert np.abs(a - g(k, "actions")).max() < 1e-4
    assert rel(st, g(k, "states")) < 1e-4
    assert abs(c - float(g(k, "cost")[0])) / abs(float(g(k, "cost")[0])) < 1e-5


@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "plan"], ids=lambda c: c["key"])
def test_oracle_plan_matches_reference(models, case):
    m = O.Model(models[case["model"]])
    k = case["key"]
    nz = O.replay(g(k, "draws"))
    a, info = O.plan(m, [g(k, "state1"), g(k, "state2")], [g(k, "goal1"), g(k, "goal2")], case["plans"], lambda lv: nz)
    assert np.abs(a - g(k, "actions")).max() < 1e-4
    assert info["iters"] == list(g(k, "iters"))
    assert rel(info["cost"], g(k, "cost")) < 1e-5


# ---------------------------------------------------------------------------------------------
# the engine's host logic (CPU): the horizon schedule needs a model, not a GPU
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "horizons"], ids=lambda c: c["key"])
def test_engine_horizons_match_reference(models, case):
    L = jlib.load()
    L.jepa_model_load.restype = C.c_void_p
    L.jepa_model_load.argtypes = [C.c_char_p, C.c_bool]
    L.jepa_model_free.argtypes = [C.c_void_p]
    model = L.jepa_model_load(models[case["model"]].encode(), False)
    assert model, jlib.error_text()
    mg = _make_golden_module()
    cfg = (capi.LevelPlan * 2)(*[capi.LevelPlan.of(**mg.plan_row(horizon=h)) for h in case["horizons"]])
    sched = []
    for c in range(len(g(case["key"], "schedule"))):
        h = (C.c_int * 2)()
        assert L.jepa_hjepa_horizons(model, cfg, 2, case["interval"], case["budget"], case["interval"] * c, h) == 0
        sched.append(list(h))
    L.jepa_model_free(model)
    assert np.array_equal(np.array(sched), g(case["key"], "schedule"))


# ---------------------------------------------------------------------------------------------
# the GPU planner vs the reference (-m gpu)
# ---------------------------------------------------------------------------------------------
@pytest.mark.gpu
@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "cost"], ids=lambda c: c["key"])
def test_gpu_cost_matches_reference(models, case):
    from jepa_b200.hjepa import Planner
    P = Planner(models[case["model"]])
    k = case["key"]
    costs, grad = P.plan_cost(case["level"], g(k, "s0"), g(k, "goal"), g(k, "actions"), goal_level=case["goal_level"],
                              dense=case["dense"], plan=case["plan"],
                              goal_actions=g(k, "goal_action") if case.get("goal_action") else None)
    assert rel(costs, g(k, "costs")) < 1e-3
    assert rel(grad, g(k, "grad")) < 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "solve"], ids=lambda c: c["key"])
def test_gpu_solve_matches_reference(models, case):
    from jepa_b200.hjepa import Planner
    P = Planner(models[case["model"]])
    k = case["key"]
    act, st, cost, iters, used = P.solve(1, g(k, "s0"), g(k, "goal"), case["plan"], noise=g(k, "draws"))
    assert used == len(g(k, "draws"))           # the reference's draws consumed exactly
    assert iters == int(g(k, "iters")[0])
    assert np.abs(act - g(k, "actions")).max() < 1e-3
    ref_st = g(k, "states")
    cosine = (st * ref_st).sum(1) / np.linalg.norm(st, axis=1) / np.linalg.norm(ref_st, axis=1)
    assert cosine.min() >= 0.9999
    assert abs(cost - float(g(k, "cost")[0])) / abs(float(g(k, "cost")[0])) < 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("case", [c for c in CASES if c["kind"] == "plan"], ids=lambda c: c["key"])
def test_gpu_plan_matches_reference(models, case):
    from jepa_b200.hjepa import Planner
    P = Planner(models[case["model"]])
    k = case["key"]
    out, info, used = P.plan([g(k, "state1"), g(k, "state2")], [g(k, "goal1"), g(k, "goal2")], case["plans"],
                             noise=g(k, "draws"))
    assert used == len(g(k, "draws"))
    assert np.abs(out - g(k, "actions")).max() < 1e-3
    assert list(info.iters)[:2] == list(g(k, "iters"))
    assert rel(list(info.cost)[:2], g(k, "cost")) < 1e-3
