"""Parity at the BASELINE configurations' own shapes (GPU, through the C ABI).

The golden and oracle tests elsewhere run forged models of width 48-96; these run the benchmark models
themselves (the synthetic GGUFs bench.py plans with: same generator, same seed) against

  * the reference's own planner, src/hjepa-plan.cpp compiled unmodified against the ggml shim
    (oracle/_ref, run live on the host cores here), for the H-JEPA configs 1, 2, 3 and 5;
  * the numpy restatement of the V-JEPA 2-AC predictor (oracle/ac_oracle.py, pinned to the reference's
    executable numpy specification) for config 4, at its full depth and width.

Bars (north star): per-candidate costs and action gradients within 1e-3 relative, planned actions within
1e-3 max-abs, equal iteration counts; predicted latents at cosine >= 0.9999 per step. Each test appends
the errors it measured, one JSON object per line, to $JEPA_PARITY_LOG when that is set.
"""
import json
import os

import numpy as np
import pytest

import ref
from jepa_b200 import capi, synth

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref.available(), reason="oracle/_ref is not built (needs the reference tree)")]

REL = 1e-3
THREADS = os.cpu_count() or 1


def record(**kw):
    path = os.environ.get("JEPA_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(kw) + "\n")


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("cfg")
    cache = {}

    def get(idx):
        if idx not in cache:
            spec, plans = synth.hjepa_config(idx)
            path = str(d / f"cfg{idx}.gguf")
            synth.write_hjepa(path, spec, seed=idx)
            cache[idx] = (path, spec, plans)
        return cache[idx]
    return get


def latents(spec, seed):
    rng = np.random.default_rng(seed)
    return ([rng.normal(size=l.embed_dim).astype(np.float32) for l in spec.levels],
            [rng.normal(size=l.embed_dim).astype(np.float32) for l in spec.levels])


def both_costs(path, spec, plans, level, S, seed):
    """Costs and gradients of S U[-1, 1] candidates of `level` from the GPU planner and the reference, the goal
    one level up (cost_last_n of its states) when there is a level above, else the top goal."""
    from jepa_b200.hjepa import Planner
    import ctypes as C
    p = plans[level - 1]
    lv = spec.levels[level - 1]
    rng = np.random.default_rng(seed)
    s0 = rng.normal(size=lv.embed_dim).astype(np.float32)
    acts = rng.uniform(-1, 1, (S, p["horizon"], lv.action_dim)).astype(np.float32)
    if level < len(spec.levels):
        n_goal, goal_level = p["cost_last_n"], level + 1
        goal = rng.normal(size=(n_goal, spec.levels[level].embed_dim)).astype(np.float32)
    else:
        n_goal, goal_level = 1, level
        goal = rng.normal(size=(1, lv.embed_dim)).astype(np.float32)
    P = Planner(path, device=0)
    costs, grad = P.plan_cost(level, s0, goal, acts, goal_level=goal_level, plan=p)
    P.close()
    R = ref.RefPlanner(path, n_threads=THREADS)
    g = capi.Goal(capi.fptr(goal), n_goal, goal_level, 0, capi.fptr(None))
    lp = capi.LevelPlan.of(**p)
    rc, rg = np.zeros(S, np.float32), np.zeros_like(acts)
    assert R.lib.jepa_hjepa_plan_cost(R.ctx, level, capi.fptr(s0), C.byref(g), C.byref(lp), capi.fptr(acts), S,
                                      p["horizon"], capi.fptr(rc), capi.fptr(rg)) == 0
    R.close()
    return costs, grad, rc, rg


def both_plans(path, spec, plans, S, n_steps, seed):
    """jepa_hjepa_plan of the GPU planner and of the reference on the same latents and the same recorded draws."""
    from jepa_b200.hjepa import Planner
    import ctypes as C
    states, goals = latents(spec, seed)
    p = [dict(q, n_samples=S, n_steps=n_steps) for q in plans]
    n_draw = sum((S - 1) * q["horizon"] * l.action_dim for l, q in zip(spec.levels, p))
    draws = np.random.default_rng(seed + 1).uniform(-1, 1, n_draw).astype(np.float32)
    P = Planner(path, device=0)
    out, info, used = P.plan(states, goals, p, noise=draws)
    P.close()
    assert used == n_draw
    n = len(p)
    R = ref.RefPlanner(path, n_threads=THREADS)
    SP = (capi.FP * n)(*[capi.fptr(s) for s in states])
    GP = (capi.FP * n)(*[capi.fptr(g) for g in goals])
    lps = (capi.LevelPlan * n)(*[capi.LevelPlan.of(**q) for q in p])
    ref_out = np.zeros_like(out)
    ref_info = capi.PlanInfo()
    rp = capi.Replay(draws)
    assert R.lib.jepa_hjepa_plan(R.ctx, SP, GP, lps, n, rp.fn, None, capi.fptr(ref_out), C.byref(ref_info)) == 0
    R.close()
    assert rp.exact()
    return out, info, ref_out, ref_info


def check_costs(cfg, level, S, costs, grad, rc, rg):
    ec, eg = rel(costs, rc), rel(grad, rg)
    record(test="plan_cost", config=cfg, level=level, candidates=S, cost_rel=ec, grad_rel=eg)
    assert ec < REL, ec
    assert eg < REL, eg


def check_plan(cfg, n, out, info, ref_out, ref_info):
    ea = float(np.abs(out - ref_out).max())
    ecost = rel(list(info.cost)[:n], list(ref_info.cost)[:n])
    record(test="plan", config=cfg, levels=n, actions_max_abs=ea, level_cost_rel=ecost,
           iters=list(info.iters)[:n], ref_iters=list(ref_info.iters)[:n])
    assert list(info.planned)[:n] == list(ref_info.planned)[:n]
    assert list(info.iters)[:n] == list(ref_info.iters)[:n]
    assert ea < REL, ea
    assert ecost < REL, ecost


# ---- config 1: 1 level f32, D256 L4 F1024, horizon 8, 64 candidates, 20 steps: the whole plan -----------
def test_config1_cost_and_full_plan(models):
    path, spec, plans = models(1)
    check_costs(1, 1, 64, *both_costs(path, spec, plans, 1, 64, seed=11))
    out, info, ref_out, ref_info = both_plans(path, spec, plans, S=64, n_steps=plans[0]["n_steps"], seed=12)
    check_plan(1, 1, out, info, ref_out, ref_info)


# ---- config 2: 2 levels q8_0, D384 L6 F1536, horizons 16 / 4 --------------------------------------------
@pytest.mark.parametrize("level", [1, 2])
def test_config2_costs(models, level):
    path, spec, plans = models(2)
    check_costs(2, level, 8, *both_costs(path, spec, plans, level, 8, seed=20 + level))


def test_config2_plan(models):
    path, spec, plans = models(2)
    out, info, ref_out, ref_info = both_plans(path, spec, plans, S=16, n_steps=3, seed=23)
    check_plan(2, 2, out, info, ref_out, ref_info)


# ---- config 3: 1 level f16, D192 L6 F768, horizon 5 ------------------------------------------------------
def test_config3_cost_and_plan(models):
    path, spec, plans = models(3)
    check_costs(3, 1, 32, *both_costs(path, spec, plans, 1, 32, seed=31))
    out, info, ref_out, ref_info = both_plans(path, spec, plans, S=32, n_steps=3, seed=32)
    check_plan(3, 1, out, info, ref_out, ref_info)


# ---- config 5: 4 levels q8_0, D768 L12 F3072, horizons 64 / 16 / 8 / 4 ------------------------------------
def test_config5_costs_and_plan(models):
    path, spec, plans = models(5)
    check_costs(5, 1, 4, *both_costs(path, spec, plans, 1, 4, seed=51))
    check_costs(5, 4, 4, *both_costs(path, spec, plans, 4, 4, seed=52))
    out, info, ref_out, ref_info = both_plans(path, spec, plans, S=4, n_steps=1, seed=53)
    check_plan(5, 4, out, info, ref_out, ref_info)


# ---- config 4: V-JEPA 2-AC predictor, 24 x 1024, 16 heads, MLP 4096, q8_0, 16 x 16 grid -------------------
def test_config4_rollout_matches_oracle_at_full_depth(tmp_path):
    import ac_oracle as O
    from jepa_b200.ac import ACWorldModel
    spec = synth.ACSpec(enc_dim=1408, pred_dim=1024, n_layer=24, n_head=16, ffn_dim=4096, grid=16, n_frames=4,
                        ftype="q8_0", name="bench-vjepa2-ac")
    path = str(tmp_path / "cfg4.gguf")
    synth.write_ac(path, spec, seed=4)
    rng = np.random.default_rng(41)
    HW, K, H, n_seed = spec.grid ** 2, 2, 2, 2
    lat = rng.normal(size=(n_seed * HW, spec.enc_dim)).astype(np.float32)
    sa = rng.normal(0, 0.05, size=(n_seed - 1, 7)).astype(np.float32)
    ss = rng.normal(0, 0.3, size=(n_seed, 7)).astype(np.float32)
    acts = rng.normal(0, 0.05, size=(K, H, 7)).astype(np.float32)
    wm = ACWorldModel(path, device=0)
    out = wm.rollout(lat, n_seed, ss, acts, seed_actions=sa)
    wm.close()

    def cosines(m):
        ref_roll = O.rollout(m, lat, n_seed, sa, ss, acts)
        cs = []
        for c in range(K):
            for s in range(H):
                a, b = out[c, s].astype(np.float64).ravel(), ref_roll[c, s].astype(np.float64).ravel()
                cs.append(float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b))))
        return cs

    m = O.ACModel(path)
    exact = cosines(m)
    # the same oracle with the engine's f16 copies of the linear weights: what remains is the f16
    # activations and attention of the GEMMs
    for name in list(m.T):
        if name.endswith(".weight") and any(k in name for k in ("attn_qkv", "attn_out", "ffn_up", "ffn_down",
                                                                 "pred.embed", "pred.proj")):
            m.T[name] = m.T[name].astype(np.float16).astype(np.float32)
    rounded = cosines(m)
    record(test="ac_rollout", config=4, layers=24, width=1024, candidates=K, steps=H,
           min_cosine_exact_weights=min(exact), min_cosine_f16_weights=min(rounded))
    assert min(exact) >= 0.9999, exact
    assert min(rounded) >= 0.9999, rounded
