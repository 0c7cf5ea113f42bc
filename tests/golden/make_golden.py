"""Writes tests/golden/hjepa_ref.npz: golden outputs of the REFERENCE planner (src/hjepa-plan.cpp, built
unmodified against the ggml shim by oracle/Makefile into oracle/_ref/libhjepa_ref.so) on seeded forged
models, for the parity tests of the oracle and of the GPU planner.

    make -C oracle && python tests/golden/make_golden.py

The models are not stored: tests rebuild them from MODELS (synth spec + seed) and check the GGUF's
sha256 against the one recorded here. Cases:
  cost.*   jepa_hjepa_plan_cost (costs + gradients) at every goal placement: own level, the level above
           (strided and dense), one and several goal states, intermediate weights
  solve.*  jepa_hjepa_solve on recorded normal draws, with early stopping / action noise / clamping
  plan.*   jepa_hjepa_plan over the 2-level hierarchy
  horizons jepa_hjepa_horizons over an episode
  acost*   jepa_hjepa_plan_cost with the action cost (the candidates' actions pooled by the upper level's
           action encoder, 'mlp' and 'seq', against the upper level's actions; action_cost_weight != 0)
  aplan    jepa_hjepa_plan over the hierarchy with the action cost on the lower level
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "jepa.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from jepa_b200 import capi, synth  # noqa: E402

OUT = os.path.join(HERE, "hjepa_ref.npz")


def model_specs():
    """name -> (spec, seed) of the forged models the fixtures are computed on."""
    L1 = synth.Level(64, 2, 2, 128, 2, act_embed_hidden=16, act_embed_dim=8, out_proj=True, proj_hidden=32, act_queue=40)
    L2 = synth.Level(64, 2, 2, 128, 4, stride=2, enc_kind="latent_mlp", enc_hidden=48, act_enc_kind="mlp", pred_dim=32)
    rich = synth.HJepaSpec(levels=[L1, L2], ftype="f32", rand_all=True, cond_std=0.3, w_std=0.1, name="golden-rich")
    P1 = synth.Level(96, 3, 3, 192, 2)
    P2 = synth.Level(96, 2, 3, 192, 6, stride=4, enc_kind="latent_mlp", enc_hidden=96, act_enc_kind="mlp")
    plain = synth.HJepaSpec(levels=[P1, P2], ftype="q8_0", rand_all=True, cond_std=0.3, w_std=0.1, name="golden-q8")
    S1 = synth.Level(48, 2, 2, 96, 2, act_embed_hidden=16, act_embed_dim=8)
    S2 = synth.Level(48, 2, 2, 96, 4, stride=3, enc_kind="latent_mlp", enc_hidden=32, act_enc_kind="seq", act_enc_dim=32,
                     act_enc_n_layer=2, act_enc_n_head=2)
    seq = synth.HJepaSpec(levels=[S1, S2], ftype="f32", rand_all=True, cond_std=0.3, w_std=0.1, name="golden-seq")
    return {"rich": (rich, 11), "q8": (plain, 12), "seq": (seq, 13)}


def build_model(name: str, workdir: str) -> tuple[str, str]:
    spec, seed = model_specs()[name]
    path = os.path.join(workdir, f"golden-{name}.gguf")
    synth.write_hjepa(path, spec, seed=seed)
    with open(path, "rb") as f:
        digest = hashlib.sha256(f.read()).hexdigest()
    return path, digest


def plan_row(**kw) -> dict:
    p = dict(horizon=4, pre_decay_horizon=0, n_samples=12, n_steps=10, lr=0.1, weight_decay=0.01, var_scale=1.0,
             action_noise=0.0, action_clip_sigma=0.0, min_its=4, early_stop_patience=3, early_stop_rel_delta=1e-2,
             cost_last_n=1, intermediate_cost_weight=1.0, action_cost_weight=0.0, num_subgoals=1, horizon_one_goal_upper=0)
    p.update(kw)
    return p


def main() -> None:
    import ref
    if not ref.available():
        sys.exit("build the reference planner first: make -C oracle")
    lib = ref.lib()
    out: dict[str, np.ndarray] = {}
    meta: dict = {"models": {}, "cases": []}
    rng = np.random.default_rng(2024)
    with tempfile.TemporaryDirectory() as tmp:
        for name in ("rich", "q8"):
            path, digest = build_model(name, tmp)
            meta["models"][name] = digest
            P = ref.RefPlanner(path, n_threads=4)
            spec, _ = model_specs()[name]
            D = [l.embed_dim for l in spec.levels]
            A = [l.action_dim for l in spec.levels]
            # ---- costs and gradients
            cost_cases = [(1, 1, 5, 0, 1), (2, 2, 3, 0, 1), (1, 2, 6, 0, 2), (1, 2, 3, 1, 2), (1, 2, 8, 0, 1)]
            for ci, (level, gl, T, dense, ng) in enumerate(cost_cases):
                if name == "q8" and gl > level and not dense and T < 4:
                    continue
                key = f"{name}.cost{ci}"
                S = 9
                s0 = rng.normal(size=D[level - 1]).astype(np.float32)
                goal = rng.normal(size=(ng, D[gl - 1])).astype(np.float32)
                acts = rng.uniform(-1.5, 1.5, (S, T, A[level - 1])).astype(np.float32)
                lp = plan_row(cost_last_n=ng, intermediate_cost_weight=0.5)
                g = capi.Goal(capi.fptr(goal), ng, gl, dense, capi.fptr(None))
                costs = np.zeros(S, np.float32)
                grad = np.zeros_like(acts)
                rc = lib.jepa_hjepa_plan_cost(P.ctx, level, capi.fptr(s0), C.byref(g), C.byref(capi.LevelPlan.of(**lp)),
                                              capi.fptr(acts), S, T, capi.fptr(costs), capi.fptr(grad))
                if rc != 0:
                    continue
                for k, v in (("s0", s0), ("goal", goal), ("actions", acts), ("costs", costs), ("grad", grad)):
                    out[f"{key}.{k}"] = v
                meta["cases"].append({"key": key, "kind": "cost", "model": name, "level": level, "goal_level": gl,
                                      "horizon": T, "dense": dense, "n_goal": ng, "plan": lp})
            # ---- single-level solves on recorded draws
            solve_cases = [dict(), dict(action_noise=0.05, early_stop_patience=0), dict(action_clip_sigma=1.5),
                           dict(early_stop_patience=0, weight_decay=0.0, n_steps=15)]
            for si, opts in enumerate(solve_cases):
                key = f"{name}.solve{si}"
                lp = plan_row(**opts)
                s0 = rng.normal(size=D[0]).astype(np.float32)
                goal = rng.normal(size=(1, D[0])).astype(np.float32)
                draws = rng.normal(size=20000).astype(np.float32)
                rp = capi.Replay(draws)
                g = capi.Goal(capi.fptr(goal), 1, 0, 0, capi.fptr(None))
                act = np.zeros((lp["horizon"], A[0]), np.float32)
                st = np.zeros((lp["horizon"] + 1, D[0]), np.float32)
                cost, it = C.c_float(), C.c_int()
                rc = lib.jepa_hjepa_solve(P.ctx, 1, capi.fptr(s0), C.byref(g), C.byref(capi.LevelPlan.of(**lp)), rp.fn, None,
                                          capi.fptr(act), capi.fptr(st), C.byref(cost), C.byref(it))
                assert rc == 0
                for k, v in (("s0", s0), ("goal", goal), ("draws", draws[:rp.pos]), ("actions", act), ("states", st),
                             ("cost", np.array([cost.value], np.float32)), ("iters", np.array([it.value], np.int64))):
                    out[f"{key}.{k}"] = v
                meta["cases"].append({"key": key, "kind": "solve", "model": name, "plan": lp})
            # ---- the hierarchy
            key = f"{name}.plan"
            T1 = 4 if name == "rich" else 8
            p1 = plan_row(horizon=T1, cost_last_n=2 if name == "rich" else 2, n_steps=8, early_stop_patience=0)
            p2 = plan_row(horizon=3 if name == "rich" else 2, num_subgoals=2, n_steps=8, early_stop_patience=0)
            states = [rng.normal(size=d).astype(np.float32) for d in D]
            goals = [rng.normal(size=d).astype(np.float32) for d in D]
            draws = rng.normal(size=20000).astype(np.float32)
            rp = capi.Replay(draws)
            SP = (capi.FP * 2)(capi.fptr(states[0]), capi.fptr(states[1]))
            GP = (capi.FP * 2)(capi.fptr(goals[0]), capi.fptr(goals[1]))
            lps = (capi.LevelPlan * 2)(capi.LevelPlan.of(**p1), capi.LevelPlan.of(**p2))
            act = np.zeros((T1, A[0]), np.float32)
            info = capi.PlanInfo()
            rc = lib.jepa_hjepa_plan(P.ctx, SP, GP, lps, 2, rp.fn, None, capi.fptr(act), C.byref(info))
            assert rc == 0, name
            for k, v in (("state1", states[0]), ("state2", states[1]), ("goal1", goals[0]), ("goal2", goals[1]),
                         ("draws", draws[:rp.pos]), ("actions", act), ("cost", np.array(list(info.cost)[:2], np.float32)),
                         ("iters", np.array(list(info.iters)[:2], np.int64)),
                         ("planned", np.array(list(info.planned)[:2], np.int64))):
                out[f"{key}.{k}"] = v
            meta["cases"].append({"key": key, "kind": "plan", "model": name, "plans": [p1, p2]})
            # ---- the horizon schedule of an episode
            key = f"{name}.horizons"
            cfg = (capi.LevelPlan * 2)(capi.LevelPlan.of(**plan_row(horizon=5)), capi.LevelPlan.of(**plan_row(horizon=3)))
            sched = []
            for c in range(12):
                h = (C.c_int * 2)()
                assert lib.jepa_hjepa_horizons(P.model, cfg, 2, 2, 24, 2 * c, h) == 0
                sched.append(list(h))
            out[f"{key}.schedule"] = np.array(sched, np.int64)
            meta["cases"].append({"key": key, "kind": "horizons", "model": name, "interval": 2, "budget": 24,
                                  "horizons": [5, 3]})
            P.close()
        # ---- the action cost: a separate stream of draws so the cases above stay as they were
        rng2 = np.random.default_rng(77)
        for name in ("rich", "seq"):
            path, digest = build_model(name, tmp)
            meta["models"][name] = digest
            P = ref.RefPlanner(path, n_threads=4)
            spec, _ = model_specs()[name]
            D = [l.embed_dim for l in spec.levels]
            A = [l.action_dim for l in spec.levels]
            stride = spec.levels[1].stride
            for ci, (T, ng, ncl) in enumerate([(2 * stride, 1, 1), (3 * stride + 1, 2, 2), (2 * stride + 1, 1, 2)]):
                key = f"{name}.acost{ci}"
                S = 7
                s0 = rng2.normal(size=D[0]).astype(np.float32)
                goal = rng2.normal(size=(ng, D[1])).astype(np.float32)
                goal_action = rng2.normal(0, 0.5, size=(ng, A[1])).astype(np.float32)
                acts = rng2.uniform(-1.5, 1.5, (S, T, A[0])).astype(np.float32)
                lp = plan_row(cost_last_n=ncl, action_cost_weight=0.7)
                g = capi.Goal(capi.fptr(goal), ng, 2, 0, capi.fptr(goal_action))
                costs = np.zeros(S, np.float32)
                grad = np.zeros_like(acts)
                rc = lib.jepa_hjepa_plan_cost(P.ctx, 1, capi.fptr(s0), C.byref(g), C.byref(capi.LevelPlan.of(**lp)),
                                              capi.fptr(acts), S, T, capi.fptr(costs), capi.fptr(grad))
                assert rc == 0, key
                for k, v in (("s0", s0), ("goal", goal), ("goal_action", goal_action), ("actions", acts), ("costs", costs),
                             ("grad", grad)):
                    out[f"{key}.{k}"] = v
                meta["cases"].append({"key": key, "kind": "cost", "model": name, "level": 1, "goal_level": 2,
                                      "horizon": T, "dense": 0, "n_goal": ng, "plan": lp, "goal_action": True})
            key = f"{name}.aplan"
            T1 = 2 * stride
            p1 = plan_row(horizon=T1, cost_last_n=2, n_steps=6, early_stop_patience=0, action_cost_weight=0.5)
            p2 = plan_row(horizon=3, num_subgoals=2, n_steps=6, early_stop_patience=0)
            states = [rng2.normal(size=d).astype(np.float32) for d in D]
            goals = [rng2.normal(size=d).astype(np.float32) for d in D]
            draws = rng2.normal(size=20000).astype(np.float32)
            rp = capi.Replay(draws)
            SP = (capi.FP * 2)(capi.fptr(states[0]), capi.fptr(states[1]))
            GP = (capi.FP * 2)(capi.fptr(goals[0]), capi.fptr(goals[1]))
            lps = (capi.LevelPlan * 2)(capi.LevelPlan.of(**p1), capi.LevelPlan.of(**p2))
            act = np.zeros((T1, A[0]), np.float32)
            info = capi.PlanInfo()
            rc = lib.jepa_hjepa_plan(P.ctx, SP, GP, lps, 2, rp.fn, None, capi.fptr(act), C.byref(info))
            assert rc == 0, key
            for k, v in (("state1", states[0]), ("state2", states[1]), ("goal1", goals[0]), ("goal2", goals[1]),
                         ("draws", draws[:rp.pos]), ("actions", act), ("cost", np.array(list(info.cost)[:2], np.float32)),
                         ("iters", np.array(list(info.iters)[:2], np.int64)),
                         ("planned", np.array(list(info.planned)[:2], np.int64))):
                out[f"{key}.{k}"] = v
            meta["cases"].append({"key": key, "kind": "plan", "model": name, "plans": [p1, p2]})
            P.close()
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(meta['cases'])} cases, {os.path.getsize(OUT) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
