"""The video encoders (jepa_encode for vjepa2, vjepa2_1 and levjepa) against the reference.

tests/golden/encode_video_ref.npz holds outputs of the reference's executable numpy specifications of the
video encoder graph (scripts/jepa_convert/vjepa2_numpy_ref.py `encoder_forward`, selftest.py
`levjepa_encoder_forward`; the graph of src/jepa.cpp:750-1000) on seeded forged models and clips;
tests/golden/make_golden_video.py wrote it. The cases cover V-JEPA 2 (tiled 3-D RoPE, tubelet 2, a 2 x 3
patch grid), V-JEPA 2.1 (interleaved RoPE, modality vectors, q8_0 weights, its one-frame image tokenizer),
LeVJEPA (CLS token with identity RoPE rows, block-causal attention across temporal slots, tubelet 1) and RoPE
position interpolation to a reference grid (3 heads of 64: lanes outside the rotated 3 d stay put).

CPU: the models rebuild byte for byte; the oracle restatement (oracle/encoder_oracle.py encode_video)
reproduces the fixture. GPU (-m gpu): jepa_encode reproduces it through the C ABI (3xTF32 tensor-core
products, float32 attention: within 1e-4 of the largest output); two clips in one call equal two single-clip
calls bit for bit; with block-causal attention a later slot's frames do not move an earlier slot's rows; a
clip that does not fill whole tubelets is refused.
"""
import importlib.util
import json
import os

import numpy as np
import pytest

import encoder_oracle as EO

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = np.load(os.path.join(HERE, "golden", "encode_video_ref.npz"))
META = json.loads(bytes(GOLDEN["meta"]))


def _generator():
    spec = importlib.util.spec_from_file_location("make_golden_video", os.path.join(HERE, "golden", "make_golden_video.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MG = _generator()


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("golden_video"))
    out = {}
    for name, digest in META["models"].items():
        path, h = MG.build_model(name, d)
        assert h == digest, f"forged model {name} does not rebuild byte for byte"
        out[name] = path
    return out


def rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(np.asarray(b)).max(), 1e-30))


CASES = [(n, i) for n in sorted(META["models"]) for i in range(len(MG.clips(n)))]


@pytest.mark.parametrize("name,i", CASES)
def test_oracle_matches_reference(models, name, i):
    clip = MG.clips(name)[i]
    assert rel(EO.encode_video(models[name], clip[None]), GOLDEN[f"{name}.{i}"]) < 1e-5


@pytest.fixture(scope="module")
def encoders(models):
    from jepa_b200.hjepa import Planner
    return {k: Planner(p, device=0) for k, p in models.items()}


@pytest.mark.gpu
@pytest.mark.parametrize("name,i", CASES)
def test_gpu_video_encoder_matches_reference(encoders, name, i):
    clip = MG.clips(name)[i]
    y = encoders[name].encode(clip[None])
    ref = GOLDEN[f"{name}.{i}"]
    assert y.shape == ref.shape
    assert rel(y, ref) < 1e-4, rel(y, ref)


@pytest.mark.gpu
def test_gpu_clips_of_one_call_equal_single_calls(encoders):
    a, b = MG.clips("va")
    both = encoders["va"].encode(np.stack([a, b]))
    one = np.concatenate([encoders["va"].encode(a[None]), encoders["va"].encode(b[None])])
    assert np.array_equal(both, one)


@pytest.mark.gpu
def test_gpu_block_causal_slots_do_not_see_the_future(encoders):
    clip = MG.clips("vc")[0]
    y = encoders["vc"].encode(clip[None])
    later = clip.copy()
    later[:, 2] += 1.0                       # the last temporal slot (tubelet 1: frame 2)
    y2 = encoders["vc"].encode(later[None])
    tpf = 4                                  # 2 x 2 patches per slot, after the CLS row
    assert np.array_equal(y[1:1 + 2 * tpf], y2[1:1 + 2 * tpf])
    assert not np.array_equal(y[1 + 2 * tpf:], y2[1 + 2 * tpf:])
    assert not np.array_equal(y[0], y2[0])   # the CLS row reads the whole clip


@pytest.mark.gpu
def test_gpu_video_refusals(encoders):
    with pytest.raises(RuntimeError, match="whole tubelets"):
        encoders["va"].encode(np.zeros((1, 3, 3, 32, 48), np.float32))
    with pytest.raises(RuntimeError, match="multiple of the patch size"):
        encoders["va"].encode(np.zeros((1, 3, 4, 30, 48), np.float32))
