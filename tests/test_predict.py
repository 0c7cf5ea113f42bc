"""The H-JEPA multi-frame predictor (jepa_hjepa_predict / jepa_hjepa_rollout) and the state / action encoders
(jepa_hjepa_embed / _lift / _action_embed / _action_encode) against the reference.

tests/golden/hjepa_predict_ref.npz holds outputs of the reference's executable numpy specification of these
entry points (scripts/jepa_convert/hjepa_numpy_ref.py, which mirrors src/hjepa.cpp:566-667) on seeded
forged models; tests/golden/make_golden_predict.py wrote it.

CPU (always): the models rebuild byte for byte; the oracle restatement reproduces every case.
GPU (-m gpu): the engine reproduces every case through the C ABI (float32 SIMT products and the causal
attention kernel: within 1e-4 of the largest output, 1e-3 for rollouts, whose steps feed back), causality
holds exactly (a changed last action leaves the earlier rows' bits alone), and out-of-range arguments are
refused with the reference's messages.
"""
import importlib.util
import json
import os

import numpy as np
import pytest

import hjepa_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = np.load(os.path.join(HERE, "golden", "hjepa_predict_ref.npz"))
META = json.loads(bytes(GOLDEN["meta"]))
CASES = META["cases"]


def _generator():
    spec = importlib.util.spec_from_file_location("make_golden_predict", os.path.join(HERE, "golden", "make_golden_predict.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    mg = _generator()
    d = str(tmp_path_factory.mktemp("golden_predict"))
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


@pytest.fixture(scope="module")
def oracles(models):
    return {k: O.Model(p) for k, p in models.items()}


PRED = [c for c in CASES if c["kind"] in ("predict", "rollout")]


@pytest.mark.parametrize("case", PRED, ids=lambda c: c["key"])
def test_oracle_matches_reference(oracles, case):
    m, k = oracles[case["model"]], case["key"]
    if case["kind"] == "predict":
        y = O.predict(m, case["level"], g(k, "states"), g(k, "actions"))
    else:
        y = O.rollout(m, case["level"], g(k, "seeds"), g(k, "actions"), case["n_steps"], case["history"])
    assert rel(y, g(k, "out")) < 1e-5


@pytest.fixture(scope="module")
def planners(models):
    from jepa_b200.hjepa import Planner
    return {k: Planner(p) for k, p in models.items()}


@pytest.mark.gpu
@pytest.mark.parametrize("case", PRED, ids=lambda c: c["key"])
def test_gpu_matches_reference(planners, case):
    P, k = planners[case["model"]], case["key"]
    if case["kind"] == "predict":
        y = P.predict(case["level"], g(k, "states"), g(k, "actions"))
        assert rel(y, g(k, "out")) < 1e-4
    else:
        y = P.rollout(case["level"], g(k, "seeds"), g(k, "actions"), case["n_steps"], case["history"])
        assert rel(y, g(k, "out")) < 1e-3


@pytest.mark.gpu
def test_gpu_predict_is_causal(planners):
    # row t depends on frames 0..t only: a different last action leaves rows 0..T-2 unchanged, bit for bit
    P = planners["pb"]
    rng = np.random.default_rng(5)
    s = rng.normal(size=(5, 96)).astype(np.float32)
    a = rng.uniform(-1, 1, (5, 3)).astype(np.float32)
    y = P.predict(1, s, a)
    a2 = a.copy()
    a2[-1] += 0.5
    y2 = P.predict(1, s, a2)
    assert np.array_equal(y[:-1], y2[:-1])
    assert not np.array_equal(y[-1], y2[-1])


@pytest.mark.gpu
def test_gpu_predict_refuses_out_of_range(planners):
    P = planners["pa"]
    s = np.zeros((5, 64), np.float32)
    a = np.zeros((5, 2), np.float32)
    with pytest.raises(RuntimeError, match="position slots"):
        P.predict(1, s, a)                      # 5 frames, 4 slots
    with pytest.raises(RuntimeError, match="history 5 is outside 1..4"):
        P.rollout(1, s[:1], a[:4], 4, 5)
    with pytest.raises(RuntimeError, match="out of range"):
        P.predict(3, s[:1], a[:1])              # the model has 2 levels


# ---------------------------------------------------------------------------------------------
# the state and action encoders (jepa_hjepa_embed / _lift / _action_embed / _action_encode)
# ---------------------------------------------------------------------------------------------
ENC = [c for c in CASES if c["kind"] in ("embed", "lift", "action_embed", "action_encode")]


def _oracle_encode(m, case):
    k = case["key"]
    if case["kind"] == "embed":
        return O.embed(m, g(k, "cls"), g(k, "proprio") if case["proprio"] else None)
    fn = {"lift": O.lift, "action_embed": O.action_embed, "action_encode": O.action_encode}[case["kind"]]
    return fn(m, case["level"], g(k, "in"))


@pytest.mark.parametrize("case", ENC, ids=lambda c: c["key"])
def test_oracle_encoders_match_reference(oracles, case):
    assert rel(_oracle_encode(oracles[case["model"]], case), g(case["key"], "out")) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("case", ENC, ids=lambda c: c["key"])
def test_gpu_encoders_match_reference(planners, case):
    P, k = planners[case["model"]], case["key"]
    if case["kind"] == "embed":
        y = P.encode_states(g(k, "cls"), g(k, "proprio") if case["proprio"] else None)
    else:
        y = P.encoder(case["kind"], case["level"], g(k, "in"))
    assert y.shape == g(k, "out").shape
    assert rel(y, g(k, "out")) < 1e-4
