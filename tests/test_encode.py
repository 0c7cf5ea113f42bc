"""The image encoder (jepa_encode for the image families) and the pooling helpers against the reference.

tests/golden/encode_ref.npz holds outputs of the reference's executable numpy specification of the
encoder graph (scripts/jepa_convert/selftest.py `encoder_forward`, the graph of src/jepa.cpp:586-632) on
seeded forged models and seeded 224 x 224 images; tests/golden/make_golden_encode.py wrote it.

CPU (always): the models rebuild byte for byte; the oracle restatement (oracle/encoder_oracle.py) reproduces
the fixture. GPU (-m gpu): jepa_encode reproduces it through the C ABI (3xTF32 tensor-core products and a
float32 attention: within 1e-4 of the largest output), two images of one call equal two single-image calls
bit for bit, jepa_pool_cls / jepa_pool_mean match their definitions, and inputs that do not fit the model are
refused with the reference's messages.
"""
import importlib.util
import json
import os

import numpy as np
import pytest

import encoder_oracle as EO

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = np.load(os.path.join(HERE, "golden", "encode_ref.npz"))
META = json.loads(bytes(GOLDEN["meta"]))


def _generator():
    spec = importlib.util.spec_from_file_location("make_golden_encode", os.path.join(HERE, "golden", "make_golden_encode.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MG = _generator()


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("golden_encode"))
    out = {}
    for name, digest in META["models"].items():
        path, h = MG.build_model(name, d)
        assert h == digest, f"forged model {name} does not rebuild byte for byte"
        out[name] = path
    return out


def rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(np.asarray(b)).max(), 1e-30))


@pytest.mark.parametrize("name", sorted(META["models"]))
def test_oracle_matches_reference(models, name):
    assert rel(EO.encode(models[name], MG.images(name)), GOLDEN[name]) < 1e-5


@pytest.fixture(scope="module")
def planners(models):
    from jepa_b200.hjepa import Planner
    return {k: Planner(p) for k, p in models.items()}


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(META["models"]))
def test_gpu_encode_matches_reference(planners, name):
    y = planners[name].encode(MG.images(name))
    assert y.shape == GOLDEN[name].shape
    assert rel(y, GOLDEN[name]) < 1e-4


@pytest.mark.gpu
def test_gpu_encode_items_are_independent(planners):
    P = planners["ea"]
    imgs = MG.images("ea")
    both = P.encode(imgs)
    one = np.concatenate([P.encode(imgs[i:i + 1]) for i in range(len(imgs))], 0)
    assert np.array_equal(both, one)


@pytest.mark.gpu
def test_gpu_pooling(planners):
    P = planners["ea"]
    enc = P.encode(MG.images("ea")[:1])
    assert np.array_equal(P.pool("cls", enc), enc[0])
    ref = enc[1:].astype(np.float64).mean(0).astype(np.float32)
    assert np.allclose(P.pool("mean", enc), ref, rtol=0, atol=1e-6)


@pytest.mark.gpu
def test_gpu_encode_refuses_what_does_not_fit(planners):
    P = planners["ea"]
    with pytest.raises(RuntimeError, match="does not match enc.pos_embed"):
        P.encode(np.zeros((1, 3, 112, 112), np.float32))
    with pytest.raises(RuntimeError, match="channels"):
        P.encode(np.zeros((1, 1, 224, 224), np.float32))
    with pytest.raises(RuntimeError, match="multiple of the patch size"):
        P.encode(np.zeros((1, 3, 225, 224), np.float32))


def _split_qkv_model(tmp_path):
    """Model 'ea' with every block's q / k / v rows written as attn_q, attn_k, attn_v (qkv_fused = false)."""
    import dataclasses as dc
    from jepa_b200 import synth
    spec, seed, _ = MG.model_specs()["ea"]
    path = str(tmp_path / "ea-split.gguf")
    synth.write_hjepa(path, dc.replace(spec, enc_qkv_fused=False), seed=seed)
    return path


def test_split_qkv_model_holds_the_fused_rows(models, tmp_path):
    """The forged split model carries exactly the fused model's q / k / v rows (the generator's draws)."""
    Tf, _ = EO.load_tensors(models["ea"])
    Ts, meta = EO.load_tensors(_split_qkv_model(tmp_path))
    assert meta["jepa.enc.qkv_fused"] is False or meta["jepa.enc.qkv_fused"] == 0
    for i in range(2):
        b = f"enc.blk.{i}."
        for part in ("weight", "bias"):
            cat = np.concatenate([Ts[b + f"attn_{x}.{part}"] for x in "qkv"], 0)
            assert np.array_equal(cat, Tf[b + f"attn_qkv.{part}"])


@pytest.mark.gpu
def test_gpu_encode_with_separate_q_k_v(tmp_path):
    """A file with q, k and v as three linears (src/jepa.cpp:409-412) encodes as its fused twin: the golden 'ea'."""
    from jepa_b200.hjepa import Planner
    P = Planner(_split_qkv_model(tmp_path))
    y = P.encode(MG.images("ea"))
    P.close()
    assert rel(y, GOLDEN["ea"]) < 1e-4
