"""Parity of the GPU H-JEPA planner (through the C ABI) with the oracle restatement of the reference
planner, on seeded forged models of every weight format.

Bars (the north star's): per-candidate costs and action gradients within 1e-3 relative (float32
accumulate), planned actions within 1e-3 max-abs, predicted states at cosine >= 0.9999.
"""
import os

import numpy as np
import pytest

import hjepa_oracle as O
from jepa_b200 import synth
from jepa_b200.hjepa import Planner

pytestmark = pytest.mark.gpu

REL = 1e-3


def forged(tmp, ftype="f32", seed=5, **kw):
    L1 = synth.Level(64, 2, 2, 128, 2, act_embed_hidden=16, act_embed_dim=8, out_proj=True, proj_hidden=32)
    L2 = synth.Level(64, 2, 2, 128, 4, stride=2, enc_kind="latent_mlp", enc_hidden=48, act_enc_kind="mlp", pred_dim=32)
    spec = synth.HJepaSpec(levels=[L1, L2], ftype=ftype, rand_all=True, cond_std=0.3, w_std=0.1, **kw)
    path = os.path.join(tmp, f"forged-{ftype}-{seed}.gguf")
    if not os.path.exists(path):
        synth.write_hjepa(path, spec, seed=seed)
    return path


@pytest.fixture(scope="module")
def tmpdir_mod(tmp_path_factory):
    return str(tmp_path_factory.mktemp("hjepa"))


def rel_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("ftype", ["f32", "f16", "q8_0", "q4_0"])
@pytest.mark.parametrize("level,goal_level,T,dense", [(1, 1, 5, 0), (2, 2, 3, 0), (1, 2, 6, 0), (1, 2, 3, 1)])
def test_plan_cost_matches_oracle(tmpdir_mod, ftype, level, goal_level, T, dense):
    path = forged(tmpdir_mod, ftype)
    m = O.Model(path)
    P = Planner(path)
    rng = np.random.default_rng(level * 10 + goal_level + T)
    D = m.levels[level - 1].hp["embed_dim"]
    A = m.levels[level - 1].hp["action_dim"]
    Dg = m.levels[goal_level - 1].hp["embed_dim"]
    S = 37
    cs = O.CostSpec(level=level, horizon=T, goal_level=goal_level, dense=bool(dense))
    n_scored = O.scored_states(m, cs)
    ng = min(2, n_scored) if goal_level > level else 1
    s0 = rng.normal(size=D).astype(np.float32)
    goal = rng.normal(size=(ng, Dg)).astype(np.float32)
    acts = rng.uniform(-1, 1, (S, T, A)).astype(np.float32)
    plan = dict(cost_last_n=ng, intermediate_cost_weight=0.5, action_cost_weight=0.0)
    costs, grad = P.plan_cost(level, s0, goal, acts, goal_level=goal_level, dense=dense, plan=plan)
    cs = O.CostSpec(level=level, horizon=T, s0=s0, goal=goal, n_goal=ng, goal_level=goal_level, dense=bool(dense),
                    cost_last_n=ng, intermediate_cost_weight=0.5)
    oc, og, _ = O.batch_cost(m, cs, acts)
    assert rel_err(costs, oc) < REL, rel_err(costs, oc)
    assert rel_err(grad, og) < REL, rel_err(grad, og)
    # costs only (no gradient) take the forward path alone and must agree with the gradient call
    c2, _ = P.plan_cost(level, s0, goal, acts, goal_level=goal_level, dense=dense, plan=plan, want_grad=False)
    assert np.array_equal(c2, costs)


def wide(tmp, ftype):
    """A predictor 768 wide (one block, MLP 768): with more than 256 rows its per-step products and its adaLN
    GEMM (6 x 768 outputs) take the persistent kernel's 128-wide tiles, every epilogue mode included."""
    spec = synth.HJepaSpec(levels=[synth.Level(768, 1, 12, 768, 2)], ftype=ftype, rand_all=True, cond_std=0.3, w_std=0.03)
    path = os.path.join(tmp, f"wide-{ftype}.gguf")
    if not os.path.exists(path):
        synth.write_hjepa(path, spec, seed=9)
    return path


@pytest.mark.parametrize("ftype", ["f32", "q8_0"])
def test_wide_predictor_matches_oracle(tmpdir_mod, ftype):
    path = wide(tmpdir_mod, ftype)
    m = O.Model(path)
    P = Planner(path)
    rng = np.random.default_rng(31)
    s0 = rng.normal(size=768).astype(np.float32)
    goal = rng.normal(size=(1, 768)).astype(np.float32)
    # 300 candidates: the persistent kernel's tiles (more than 256 rows), every fused epilogue of the block
    acts = rng.uniform(-1, 1, (300, 3, 2)).astype(np.float32)
    costs, grad = P.plan_cost(1, s0, goal, acts)
    oc, og, _ = O.batch_cost(m, O.CostSpec(level=1, horizon=3, s0=s0, goal=goal), acts)
    assert rel_err(costs, oc) < REL, rel_err(costs, oc)
    assert rel_err(grad, og) < REL, rel_err(grad, og)
    # a row's bits do not depend on the batch among batches of more than 256 rows either
    c_sub, g_sub = P.plan_cost(1, s0, goal, np.ascontiguousarray(acts[5:270]))
    assert np.array_equal(costs[5:270], c_sub)
    assert np.array_equal(grad[5:270], g_sub)
    # 256 rows and fewer take the split-K clusters: the same rows agree to rounding
    c_few, g_few = P.plan_cost(1, s0, goal, np.ascontiguousarray(acts[5:20]))
    assert rel_err(c_few, costs[5:20]) < REL and rel_err(g_few, grad[5:20]) < REL


def test_rows_do_not_depend_on_the_batch(tmpdir_mod):
    """A candidate's cost and gradient are the same bits whatever batch it is evaluated in (what makes the
    candidate sharding across GPUs exact)."""
    path = forged(tmpdir_mod, "q8_0")
    P = Planner(path)
    rng = np.random.default_rng(3)
    s0 = rng.normal(size=64).astype(np.float32)
    goal = rng.normal(size=(1, 64)).astype(np.float32)
    acts = rng.uniform(-1, 1, (300, 4, 2)).astype(np.float32)
    c_all, g_all = P.plan_cost(1, s0, goal, acts)
    c_sub, g_sub = P.plan_cost(1, s0, goal, np.ascontiguousarray(acts[130:170]))
    assert np.array_equal(c_all[130:170], c_sub)
    assert np.array_equal(g_all[130:170], g_sub)


def solve_plan(T=4, S=24, steps=12, **kw):
    p = dict(horizon=T, pre_decay_horizon=0, n_samples=S, n_steps=steps, lr=0.1, weight_decay=0.01, var_scale=1.0,
             action_noise=0.0, action_clip_sigma=0.0, min_its=5, early_stop_patience=3, early_stop_rel_delta=1e-2,
             cost_last_n=1, intermediate_cost_weight=1.0, action_cost_weight=0.0, num_subgoals=1, horizon_one_goal_upper=0)
    p.update(kw)
    return p


@pytest.mark.parametrize("ftype", ["f32", "q8_0"])
@pytest.mark.parametrize("opts", [{}, {"action_noise": 0.05, "early_stop_patience": 0}, {"action_clip_sigma": 1.5},
                                  {"early_stop_patience": 0, "weight_decay": 0.0}])
def test_solve_matches_oracle(tmpdir_mod, ftype, opts):
    path = forged(tmpdir_mod, ftype)
    m = O.Model(path)
    P = Planner(path)
    rng = np.random.default_rng(11)
    s0 = rng.normal(size=64).astype(np.float32)
    goal = rng.normal(size=(1, 64)).astype(np.float32)
    draws = rng.normal(size=200000).astype(np.float32)
    plan = solve_plan(**opts)
    act, st, cost, iters, used = P.solve(1, s0, goal, plan, noise=draws)
    cs = O.CostSpec(level=1, horizon=plan["horizon"], s0=s0, goal=goal)
    nz = O.replay(draws)
    oa, ost, oc, oit = O.solve_level(m, cs, plan, nz)
    assert iters == oit
    assert np.abs(act - oa).max() < 1e-3, np.abs(act - oa).max()
    cosine = (st * ost).sum(1) / np.linalg.norm(st, axis=1) / np.linalg.norm(ost, axis=1)
    assert cosine.min() >= 0.9999
    assert abs(cost - oc) / abs(oc) < REL


@pytest.mark.parametrize("opts", [{"early_stop_patience": 0}, {"early_stop_patience": 2, "action_noise": 0.05}])
def test_solve_does_not_depend_on_the_stream_count(tmpdir_mod, opts):
    # a level's candidates split into 1, 2, 3 or 5 chains side by side on the GPU: the same plan, bit for bit
    # (the reference's counterpart: results identical for any thread count)
    path = forged(tmpdir_mod, "f32")
    P = Planner(path)
    rng = np.random.default_rng(17)
    s0 = rng.normal(size=64).astype(np.float32)
    goal = rng.normal(size=(1, 64)).astype(np.float32)
    draws = rng.normal(size=400000).astype(np.float32)
    plan = solve_plan(S=301, steps=8, **opts)
    ref = None
    for n in (1, 2, 3, 5):
        P.set_streams(n)
        got = P.solve(1, s0, goal, plan, noise=draws)
        if ref is None:
            ref = got
            continue
        for a, b in zip(got[:4], ref[:4]):
            assert np.array_equal(np.asarray(a), np.asarray(b)), n
    P.set_streams(0)


def test_step_at_a_time_modulation_is_bit_identical(tmpdir_mod):
    # the memory-lean modes (modulation per step, recomputed in the backward; every step's modulation kept,
    # its gradient folded per step) against every step's at once: the same costs, gradients and plan, bit for bit
    path = forged(tmpdir_mod, "q8_0")
    P = Planner(path)
    rng = np.random.default_rng(23)
    s0 = rng.normal(size=64).astype(np.float32)
    goal = rng.normal(size=(2, 64)).astype(np.float32)
    acts = rng.uniform(-1, 1, (37, 6, 2)).astype(np.float32)
    draws = rng.normal(size=200000).astype(np.float32)
    plan = solve_plan(T=6, S=70, steps=6, early_stop_patience=0, cost_last_n=2)
    out = []
    for mode in (0, 1, 2):
        P.set_step_modulation(mode)
        c, g = P.plan_cost(1, s0, goal, acts, goal_level=2, plan=dict(plan, cost_last_n=2))
        out.append((c, g) + tuple(P.solve(1, s0, goal[:1], dict(plan, cost_last_n=1), noise=draws)[:4]))
    for other in out[1:]:
        for a, b in zip(out[0], other):
            assert np.array_equal(np.asarray(a), np.asarray(b))
    P.set_step_modulation(0)


def test_hierarchy_matches_oracle(tmpdir_mod):
    path = forged(tmpdir_mod, "f32")
    m = O.Model(path)
    P = Planner(path)
    rng = np.random.default_rng(21)
    states = [rng.normal(size=64).astype(np.float32), rng.normal(size=64).astype(np.float32)]
    goals = [rng.normal(size=64).astype(np.float32), rng.normal(size=64).astype(np.float32)]
    p1 = solve_plan(T=4, cost_last_n=2, num_subgoals=1, n_steps=10, early_stop_patience=0)
    p2 = solve_plan(T=3, cost_last_n=1, num_subgoals=2, n_steps=10, early_stop_patience=0)
    draws = rng.normal(size=100000).astype(np.float32)
    out, info, used = P.plan(states, goals, [p1, p2], noise=draws)
    nz = O.replay(draws)
    oa, oinfo = O.plan(m, states, goals, [p1, p2], lambda lv: nz)
    assert np.abs(out - oa).max() < 1e-3
    assert list(info.planned)[:2] == oinfo["planned"]
    assert list(info.iters)[:2] == oinfo["iters"]
    for k in range(2):
        assert abs(info.cost[k] - oinfo["cost"][k]) / abs(oinfo["cost"][k]) < REL


def test_errors_are_reported(tmpdir_mod):
    path = forged(tmpdir_mod, "f32")
    P = Planner(path)
    s0 = np.zeros(64, np.float32)
    goal = np.zeros((1, 64), np.float32)
    with pytest.raises(RuntimeError, match="no level 3 to plan"):
        P.plan_cost(3, s0, goal, np.zeros((2, 3, 2), np.float32))
    with pytest.raises(RuntimeError, match="shorter than one step of level 2"):
        P.plan_cost(1, s0, goal, np.zeros((2, 1, 2), np.float32), goal_level=2)
