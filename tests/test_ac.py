"""V-JEPA 2-AC parity: the numpy oracle against the reference's executable spec, and the GPU engine against
the oracle.

CPU (always):
  - the forged golden model rebuilds byte for byte; the oracle's predictor reproduces the predictions of
    the reference's numpy spec (tests/golden/ac_spec.npz, written by tests/golden/make_golden_ac.py from
    scripts/jepa_convert/selftest.py::ac_predictor_forward) for 1, 2 and 3 frames;
  - the oracle's 3-D RoPE reproduces the reference's hd64 "hf" golden vectors (tests/golden/rope3d_hf.npz);
  - the library's host-side pose update and L1 energy agree with the oracle;
  - the oracle's CEM keeps the rotation lanes at exactly 0 and rounds small gripper commands away.
GPU (-m gpu), through the C ABI:
  - predict_all matches the reference spec's predictions (cosine >= 0.9999 per frame) and the oracle on a
    model with the real head width (64) and frame size (2 + 256 rows);
  - predict == the last block of predict_all, bit for bit; block causality (a later frame's inputs do not
    move an earlier frame's predictions, bit for bit);
  - rollouts (with and without the seed actions, explicit poses or the pose update) match the oracle per
    step (cosine >= 0.9999); K candidates at once == one at a time, bit for bit; the cached context ==
    the explicit one, bit for bit, across update / trim;
  - jepa_ac_plan with explicit noise == the oracle's CEM refit driven by the GPU's own predictions
    (identical elite sets and energies, plan within 1e-6).
"""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

import ac_oracle as O
from jepa_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
SPEC = np.load(os.path.join(HERE, "golden", "ac_spec.npz"))
ROPE = np.load(os.path.join(HERE, "golden", "rope3d_hf.npz"))
COS_MIN = 0.9999


def _make_golden_ac():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden_ac", os.path.join(HERE, "golden", "make_golden_ac.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def golden_model(tmp_path_factory):
    mg = _make_golden_ac()
    path, digest = mg.build_model(str(tmp_path_factory.mktemp("ac_golden")))
    assert digest == json.loads(bytes(SPEC["meta"]))["model"], "the forged AC model does not rebuild byte for byte"
    return path


@pytest.fixture(scope="module")
def wide_model(tmp_path_factory):
    """The real head width (64) and frame size (2 + 16 x 16 rows), two layers, q8_0 weights."""
    path = str(tmp_path_factory.mktemp("ac_wide") / "wide.gguf")
    synth.write_ac(path, synth.ACSpec(enc_dim=128, pred_dim=256, n_layer=2, n_head=4, ffn_dim=512, grid=16, n_frames=4,
                                      ftype="q8_0", rand_all=True, w_std=0.05, name="ac-wide"), seed=5)
    return path


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


# ---------------------------------------------------------------------------------------------
# CPU: the oracle against the reference
# ---------------------------------------------------------------------------------------------
@pytest.mark.parametrize("T", [1, 2, 3])
def test_oracle_predict_matches_reference_spec(golden_model, T):
    m = O.ACModel(golden_model)
    pred = O.predict_all(m, SPEC[f"T{T}.context"], SPEC[f"T{T}.actions"], SPEC[f"T{T}.states"])
    ref = SPEC[f"T{T}.pred"]
    assert pred.shape == ref.shape
    np.testing.assert_allclose(pred, ref, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("case", ["hd64_g4x4x4", "hd64_g8x16x16_sub"])
def test_oracle_rope_matches_reference_vectors(case):
    x = ROPE[f"{case}.x"].astype(np.float32)
    ids = ROPE[f"{case}.ids"].astype(np.int64)
    grid = int(ROPE["grids"][0 if case.endswith("4x4x4") else 1][1])
    cos, sin = O.rope_tables(ids, grid, x.shape[-1], 10000.0, "tiled")
    out = O.rope_apply(x, cos, sin)
    np.testing.assert_allclose(out, ROPE[f"{case}.out"].astype(np.float32).reshape(out.shape), rtol=1e-5, atol=1e-5)


def _lib():
    from jepa_b200 import lib as jlib
    L = jlib.load()
    FP = C.POINTER(C.c_float)
    L.jepa_ac_next_state.argtypes = [C.c_void_p, FP, FP, FP]
    L.jepa_ac_next_state.restype = None
    L.jepa_ac_energy.argtypes = [FP, FP, C.c_int, C.c_int64, C.c_int64, FP]
    L.jepa_ac_energy.restype = None
    return L


def test_next_state_and_energy_match_oracle():
    L = _lib()
    rng = np.random.default_rng(3)
    FP = C.POINTER(C.c_float)
    for _ in range(50):
        s = rng.normal(0, 0.6, 7).astype(np.float32)
        a = rng.normal(0, 0.2, 7).astype(np.float32)
        out = np.zeros(7, np.float32)
        L.jepa_ac_next_state(None, s.ctypes.data_as(FP), a.ctypes.data_as(FP), out.ctypes.data_as(FP))
        np.testing.assert_allclose(out, O.next_state(s, a), rtol=0, atol=2e-7)
    pred = rng.normal(size=(5, 16, 24)).astype(np.float32)
    goal = rng.normal(size=(16, 24)).astype(np.float32)
    e = np.zeros(5, np.float32)
    L.jepa_ac_energy(pred.ctypes.data_as(FP), goal.ctypes.data_as(FP), 5, 16, 24, e.ctypes.data_as(FP))
    np.testing.assert_allclose(e, O.energy(pred, goal), rtol=1e-7)


def test_oracle_cem_invariants():
    """Rotation lanes stay exactly 0; |gripper| below round_gripper is rounded to 0 (reference:
    src/vjepa2_ac.cpp:936-945); every elite set has topk distinct candidates."""
    rng = np.random.default_rng(9)
    K, H, HW, E = 12, 2, 4, 8
    goal = rng.normal(size=(HW, E)).astype(np.float32)
    W = rng.normal(size=(7, HW * E)).astype(np.float32)

    def roll(acts):
        return np.tanh(acts @ W).reshape(K, H, HW, E).astype(np.float32)

    p = dict(samples=K, topk=4, cem_steps=3, horizon=H, maxnorm=0.05, gripper_clamp=0.75, momentum_mean=0.25,
             momentum_std=0.95, momentum_mean_gripper=0.15, momentum_std_gripper=0.15, round_gripper=0.25)
    noise = rng.normal(size=(3, H, K, 4)).astype(np.float32)
    out, best, elites = O.cem(None, None, 1, None, None, goal, p, noise, rollout_fn=roll, A=7)
    assert np.all(out[:, 3:6] == 0.0)
    assert np.all((out[:, 6] == 0.0) | (np.abs(out[:, 6]) >= 0.25))
    assert all(len(set(e.tolist())) == 4 for e in elites)
    assert best.shape == (3,)


# ---------------------------------------------------------------------------------------------
# GPU: the engine against the reference spec and the oracle
# ---------------------------------------------------------------------------------------------
def _wm(path):
    from jepa_b200.ac import ACWorldModel
    return ACWorldModel(path)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 2, 3])
def test_gpu_predict_all_matches_reference_spec(golden_model, T):
    wm = _wm(golden_model)
    ctx = SPEC[f"T{T}.context"][None]
    pred = wm.predict(ctx, SPEC[f"T{T}.actions"][None], SPEC[f"T{T}.states"][None], all_frames=True)[0]
    ref = SPEC[f"T{T}.pred"]
    HW = wm.HW
    for t in range(T):
        c = cosine(pred[t * HW:(t + 1) * HW], ref[t * HW:(t + 1) * HW])
        assert c >= COS_MIN, f"frame {t}: cosine {c}"


@pytest.mark.gpu
def test_gpu_predict_wide_model_matches_oracle(wide_model):
    wm = _wm(wide_model)
    m = O.ACModel(wide_model)
    rng = np.random.default_rng(11)
    T, B = 3, 2
    ctx = rng.normal(size=(B, T * wm.HW, m.enc_dim)).astype(np.float32)
    act = rng.normal(0, 0.5, size=(B, T, m.A)).astype(np.float32)
    st = rng.normal(0, 0.5, size=(B, T, m.S)).astype(np.float32)
    pred = wm.predict(ctx, act, st, all_frames=True)
    last = wm.predict(ctx, act, st, all_frames=False)
    assert np.array_equal(last[:, :, :], pred[:, -wm.HW:, :]), "predict != last block of predict_all"
    for b in range(B):
        ref = O.predict_all(m, ctx[b], act[b], st[b])
        for t in range(T):
            c = cosine(pred[b, t * wm.HW:(t + 1) * wm.HW], ref[t * wm.HW:(t + 1) * wm.HW])
            assert c >= COS_MIN, f"item {b} frame {t}: cosine {c}"


@pytest.mark.gpu
def test_gpu_block_causality(golden_model):
    wm = _wm(golden_model)
    rng = np.random.default_rng(12)
    T = 3
    ctx = rng.normal(size=(1, T * wm.HW, 96)).astype(np.float32)
    act = rng.normal(0, 0.5, size=(1, T, 7)).astype(np.float32)
    st = rng.normal(0, 0.5, size=(1, T, 7)).astype(np.float32)
    a = wm.predict(ctx, act, st, all_frames=True)
    ctx2, act2 = ctx.copy(), act.copy()
    ctx2[0, (T - 1) * wm.HW:] += 1.0
    act2[0, T - 1] += 0.3
    b = wm.predict(ctx2, act2, st, all_frames=True)
    n = (T - 1) * wm.HW
    assert np.array_equal(a[0, :n], b[0, :n]), "a later frame moved an earlier frame's prediction"
    assert not np.array_equal(a[0, n:], b[0, n:])


def _rollout_inputs(rng, HW, E, n_seed, K, H, A=7, S=7):
    latents = rng.normal(size=(n_seed * HW, E)).astype(np.float32)
    seed_actions = rng.normal(0, 0.05, size=(max(n_seed - 1, 1), A)).astype(np.float32)
    seed_states = rng.normal(0, 0.3, size=(n_seed, S)).astype(np.float32)
    actions = rng.normal(0, 0.05, size=(K, H, A)).astype(np.float32)
    return latents, seed_actions, seed_states, actions


@pytest.mark.gpu
@pytest.mark.parametrize("n_seed,H,with_seed_actions,with_states", [(1, 3, False, False), (2, 2, True, False),
                                                                     (2, 2, False, False), (2, 2, True, True)])
def test_gpu_rollout_matches_oracle(golden_model, n_seed, H, with_seed_actions, with_states):
    wm = _wm(golden_model)
    m = O.ACModel(golden_model)
    rng = np.random.default_rng(100 + n_seed * 10 + H)
    K = 3
    lat, sa, ss, acts = _rollout_inputs(rng, wm.HW, m.enc_dim, n_seed, K, H)
    states = rng.normal(0, 0.3, size=(K, H, 7)).astype(np.float32) if with_states else None
    sa = sa if with_seed_actions else None
    out = wm.rollout(lat, n_seed, ss, acts, states=states, seed_actions=sa)
    ref = O.rollout(m, lat, n_seed, sa, ss, acts, states)
    for c in range(K):
        for s in range(H):
            cs = cosine(out[c, s], ref[c, s])
            assert cs >= COS_MIN, f"candidate {c} step {s}: cosine {cs}"


@pytest.mark.gpu
def test_gpu_rollout_wide_model_matches_oracle(wide_model):
    wm = _wm(wide_model)
    m = O.ACModel(wide_model)
    rng = np.random.default_rng(21)
    K, H, n_seed = 2, 2, 2
    lat, sa, ss, acts = _rollout_inputs(rng, wm.HW, m.enc_dim, n_seed, K, H)
    out = wm.rollout(lat, n_seed, ss, acts, seed_actions=sa)
    ref = O.rollout(m, lat, n_seed, sa, ss, acts)
    for c in range(K):
        for s in range(H):
            cs = cosine(out[c, s], ref[c, s])
            assert cs >= COS_MIN, f"candidate {c} step {s}: cosine {cs}"


@pytest.mark.gpu
def test_gpu_rollout_batched_equals_sequential(golden_model):
    wm = _wm(golden_model)
    rng = np.random.default_rng(31)
    K, H, n_seed = 5, 3, 2
    lat, sa, ss, acts = _rollout_inputs(rng, wm.HW, 96, n_seed, K, H)
    batched = wm.rollout(lat, n_seed, ss, acts, seed_actions=sa)
    for c in range(K):
        one = wm.rollout(lat, n_seed, ss, acts[c:c + 1], seed_actions=sa)
        assert np.array_equal(one[0], batched[c]), f"candidate {c} differs between K={K} and K=1"


@pytest.mark.gpu
def test_gpu_cached_context_equals_explicit(golden_model):
    wm = _wm(golden_model)
    rng = np.random.default_rng(41)
    K, H = 4, 2
    HW, E = wm.HW, 96
    lat, sa, ss, acts = _rollout_inputs(rng, HW, E, 2, K, H)
    h = wm.context_new(lat, 2, sa, ss)
    cached = wm.rollout_cached(h, acts, E=E)
    explicit = wm.rollout(lat, 2, ss, acts, seed_actions=sa)
    assert np.array_equal(cached, explicit)
    assert np.array_equal(wm.rollout_cached(h, acts, E=E), cached), "a second cached call differs"
    # receding horizon: add an observation, then drop the oldest frame
    new_lat = rng.normal(size=(HW, E)).astype(np.float32)
    new_act = rng.normal(0, 0.05, size=7).astype(np.float32)
    new_st = rng.normal(0, 0.3, size=7).astype(np.float32)
    wm.context_update(h, new_lat, new_act, new_st)
    lat3 = np.concatenate([lat, new_lat])
    sa3 = np.concatenate([sa[:1], new_act[None]])
    ss3 = np.concatenate([ss, new_st[None]])
    assert np.array_equal(wm.rollout_cached(h, acts, E=E), wm.rollout(lat3, 3, ss3, acts, seed_actions=sa3))
    wm.context_trim(h, 2)
    assert np.array_equal(wm.rollout_cached(h, acts, E=E), wm.rollout(lat3[HW:], 2, ss3[1:], acts, seed_actions=sa3[1:]))


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [0, 7])
def test_gpu_cem_default_draws_match_the_reference_generator(golden_model, seed):
    """jepa_ac_plan without noise draws from the reference's seeded generator (src/vjepa2_ac.cpp:804-826,
    restated in oracle/ac_oracle.py cem_draws): the plan equals the oracle's CEM refit fed with those draws
    and the GPU's own predictions."""
    wm = _wm(golden_model)
    m = O.ACModel(golden_model)
    rng = np.random.default_rng(61)
    HW, E = wm.HW, 96
    lat, sa, ss, _ = _rollout_inputs(rng, HW, E, 2, 1, 1)
    goal = rng.normal(size=(HW, E)).astype(np.float32)
    h = wm.context_new(lat, 2, sa, ss)
    p = dict(samples=20, topk=5, cem_steps=3, horizon=2, maxnorm=0.05, gripper_clamp=0.75, momentum_mean=0.25,
             momentum_std=0.95, momentum_mean_gripper=0.15, momentum_std_gripper=0.15, round_gripper=0.25)
    plan, best = wm.plan(h, goal, wm.cem_params(seed=seed, **p), noise=None)
    draws = O.cem_draws(seed, p["cem_steps"] * p["horizon"] * p["samples"] * 4).reshape(
        p["cem_steps"], p["horizon"], p["samples"], 4)
    ref, ref_best, _ = O.cem(m, None, 2, None, None, goal, p, draws, rollout_fn=lambda a: wm.rollout_cached(h, a, E=E))
    np.testing.assert_allclose(plan, ref, rtol=0, atol=1e-6)
    np.testing.assert_allclose(best, ref_best, rtol=1e-6)
    # explicit noise equal to those draws gives the same plan bit for bit
    plan2, best2 = wm.plan(h, goal, wm.cem_params(seed=seed + 1, **p), noise=draws)
    assert np.array_equal(plan, plan2) and np.array_equal(best, best2)


def test_oracle_cem_draws_are_normal_and_seeded():
    a = O.cem_draws(0, 4000)
    assert np.array_equal(a[:50], O.cem_draws(0, 50))
    assert not np.array_equal(a[:50], O.cem_draws(1, 50))
    assert abs(float(a.mean())) < 0.06 and abs(float(a.std()) - 1.0) < 0.05


@pytest.mark.gpu
def test_gpu_cem_matches_oracle_refit(golden_model):
    wm = _wm(golden_model)
    m = O.ACModel(golden_model)
    rng = np.random.default_rng(51)
    HW, E = wm.HW, 96
    lat, sa, ss, _ = _rollout_inputs(rng, HW, E, 2, 1, 1)
    goal = rng.normal(size=(HW, E)).astype(np.float32)
    h = wm.context_new(lat, 2, sa, ss)
    p = dict(samples=24, topk=6, cem_steps=4, horizon=2, maxnorm=0.05, gripper_clamp=0.75, momentum_mean=0.25,
             momentum_std=0.95, momentum_mean_gripper=0.15, momentum_std_gripper=0.15, round_gripper=0.25)
    noise = rng.normal(size=(p["cem_steps"], p["horizon"], p["samples"], 4)).astype(np.float32)
    plan, best = wm.plan(h, goal, wm.cem_params(**p), noise=noise)
    ref, ref_best, _ = O.cem(m, None, 2, None, None, goal, p, noise, rollout_fn=lambda a: wm.rollout_cached(h, a, E=E))
    np.testing.assert_allclose(plan, ref, rtol=0, atol=1e-6)
    np.testing.assert_allclose(best, ref_best, rtol=1e-6)
    assert np.all(plan[:, 3:6] == 0.0)
    # the numpy world model itself: the plan agrees to the f16 tolerance of the predictions
    ref_np, _, _ = O.cem(m, lat, 2, sa, ss, goal, p, noise)
    assert np.abs(plan - ref_np).max() < 0.02
