"""The GGUF reader and the jepa.* schema on the CPU, for every model family the reference's loader knows
(src/jepa-gguf.cpp:254-560; the key schema of its docs/gguf-schema.md).

A model loads without a GPU (metadata, host tensors, introspection); the planners then need one. Files are
written by this repository's own GGUF writer (jepa_b200/gguf_write.py). Refusals -- a wrong architecture, an
unknown family, a missing required key, an integer out of its range, a per-level array without one entry
per level, a truncated file -- return NULL with the reason in jepa_error_text(), never a half-loaded model.
"""
import ctypes as C
import os

import numpy as np
import pytest

from jepa_b200 import lib as jlib
from jepa_b200 import synth
from jepa_b200.gguf_write import GGUFWriter

FAMILIES = ["ijepa", "vjepa", "vjepa2", "vjepa2_1", "levjepa", "hfvit", "lewm"]


@pytest.fixture(scope="module")
def L():
    L = jlib.load()
    L.jepa_model_load.restype = C.c_void_p
    L.jepa_model_load.argtypes = [C.c_char_p, C.c_bool]
    L.jepa_model_free.argtypes = [C.c_void_p]
    for name in ("jepa_model_family", "jepa_model_name"):
        getattr(L, name).restype = C.c_char_p
        getattr(L, name).argtypes = [C.c_void_p]
    for name in ("jepa_model_embed_dim", "jepa_model_patch_size", "jepa_model_tubelet_size", "jepa_model_n_frames",
                 "jepa_model_n_layer", "jepa_model_n_head", "jepa_model_n_registers", "jepa_hjepa_n_levels",
                 "jepa_ac_action_dim", "jepa_ac_state_dim", "jepa_ac_tokens_per_frame", "jepa_ac_max_frames"):
        getattr(L, name).restype = C.c_int
        getattr(L, name).argtypes = [C.c_void_p]
    L.jepa_model_has_cls.restype = C.c_bool
    L.jepa_model_has_cls.argtypes = [C.c_void_p]
    L.jepa_hjepa_embed_dim.restype = C.c_int
    L.jepa_hjepa_embed_dim.argtypes = [C.c_void_p, C.c_int]
    return L


def encoder_file(path, family, drop=None, **over):
    kv = {"jepa.enc.embed_dim": 64, "jepa.enc.n_layer": 2, "jepa.enc.n_head": 4, "jepa.enc.ffn_dim": 256,
          "jepa.enc.patch_size": 16, "jepa.enc.img_size": 224, "jepa.enc.in_chans": 3}
    if family in ("vjepa", "vjepa2", "vjepa2_1"):
        kv.update({"jepa.enc.tubelet_size": 2, "jepa.enc.n_frames": 16})
    if family in ("ijepa", "hfvit", "lewm"):
        kv.update({"jepa.enc.cls_token": True})
    if family == "levjepa":
        kv.update({"jepa.enc.n_registers": 4})
    kv.update(over)
    w = GGUFWriter()
    w.add_kv("general.architecture", "jepa")
    w.add_kv("general.name", f"tiny-{family}")
    w.add_kv("jepa.family", family)
    for k, v in kv.items():
        if k != drop:
            w.add_kv(k, v)
    w.add_tensor("enc.norm.weight", np.ones(64, np.float32))
    w.write(path)
    return kv


@pytest.mark.parametrize("family", FAMILIES)
def test_every_family_loads_and_reports_its_shape(L, tmp_path, family):
    path = str(tmp_path / f"{family}.gguf")
    kv = encoder_file(path, family)
    L.jepa_error_reset()
    m = L.jepa_model_load(path.encode(), False)
    assert m, jlib.error_text()
    assert L.jepa_model_family(m).decode() == family
    assert L.jepa_model_name(m).decode() == f"tiny-{family}"
    assert L.jepa_model_embed_dim(m) == 64 and L.jepa_model_n_layer(m) == 2 and L.jepa_model_n_head(m) == 4
    assert L.jepa_model_patch_size(m) == 16
    assert L.jepa_model_tubelet_size(m) == kv.get("jepa.enc.tubelet_size", 1)
    assert L.jepa_model_n_frames(m) == kv.get("jepa.enc.n_frames", 1)
    assert L.jepa_model_has_cls(m) == bool(kv.get("jepa.enc.cls_token", False))
    assert L.jepa_model_n_registers(m) == kv.get("jepa.enc.n_registers", 0)
    assert L.jepa_hjepa_n_levels(m) == 0
    L.jepa_model_free(m)


def test_hjepa_and_ac_bundles_load(L, tmp_path):
    spec, _ = synth.hjepa_config(2)
    p = str(tmp_path / "h.gguf")
    synth.write_hjepa(p, spec, seed=1)
    m = L.jepa_model_load(p.encode(), False)
    assert m, jlib.error_text()
    assert L.jepa_model_family(m) == b"hjepa" and L.jepa_hjepa_n_levels(m) == 2
    L.jepa_model_free(m)
    a = str(tmp_path / "ac.gguf")
    synth.write_ac(a, synth.ACSpec(enc_dim=64, pred_dim=64, n_layer=1, n_head=2, ffn_dim=128, grid=4, n_frames=3,
                                   ftype="f32", name="tiny-ac"), seed=2)
    m = L.jepa_model_load(a.encode(), False)
    assert m, jlib.error_text()
    assert (L.jepa_ac_action_dim(m), L.jepa_ac_state_dim(m), L.jepa_ac_tokens_per_frame(m), L.jepa_ac_max_frames(m)) == \
        (7, 7, 16, 3)
    L.jepa_model_free(m)


def _refused(L, path, needle):
    L.jepa_error_reset()
    m = L.jepa_model_load(path.encode(), False)
    assert not m
    text = jlib.error_text()
    assert needle in text, text


def test_refusals_name_the_problem(L, tmp_path):
    p = str(tmp_path / "bad.gguf")
    encoder_file(p, "ijepa", drop="jepa.enc.ffn_dim")
    _refused(L, p, "jepa.enc.ffn_dim")
    encoder_file(p, "ijepa", **{"jepa.enc.n_layer": 0})
    _refused(L, p, "jepa.enc.n_layer")
    encoder_file(p, "nojepa")
    _refused(L, p, "nojepa")
    w = GGUFWriter()
    w.add_kv("general.architecture", "llama")
    w.write(p)
    _refused(L, p, "llama")
    good = str(tmp_path / "h.gguf")
    synth.write_hjepa(good, synth.HJepaSpec(levels=[synth.Level(32, 1, 2, 64, 2),
                                                    synth.Level(32, 1, 2, 64, 2, stride=2, enc_kind="latent_mlp")]), seed=3)
    raw = open(good, "rb").read()
    # truncated: the tensor data cut short
    with open(p, "wb") as f:
        f.write(raw[: len(raw) - 100])
    L.jepa_error_reset()
    assert not L.jepa_model_load(p.encode(), False)
    assert jlib.error_text()


def test_per_level_arrays_need_one_entry_per_level(L, tmp_path):
    """A 2-level H-JEPA file whose jepa.hjepa.stride array holds one value is refused with the key named."""
    p = str(tmp_path / "levels.gguf")
    w = GGUFWriter()
    w.add_kv("general.architecture", "jepa")
    w.add_kv("jepa.family", "hjepa")
    for k, v in (("embed_dim", 32), ("n_layer", 1), ("n_head", 2), ("ffn_dim", 64), ("patch_size", 16)):
        w.add_kv("jepa.enc." + k, v)
    w.add_kv("jepa.hjepa.n_levels", 2)
    w.add_kv("jepa.hjepa.embed_dim", [32, 32])
    w.add_kv("jepa.hjepa.stride", [1])
    w.add_tensor("enc.norm.weight", np.ones(32, np.float32))
    w.write(p)
    _refused(L, p, "jepa.hjepa.stride")
    # and a level count out of range
    w = GGUFWriter()
    w.add_kv("general.architecture", "jepa")
    w.add_kv("jepa.family", "hjepa")
    for k, v in (("embed_dim", 32), ("n_layer", 1), ("n_head", 2), ("ffn_dim", 64), ("patch_size", 16)):
        w.add_kv("jepa.enc." + k, v)
    w.add_kv("jepa.hjepa.n_levels", 0)
    w.add_tensor("enc.norm.weight", np.ones(32, np.float32))
    w.write(p)
    _refused(L, p, "jepa.hjepa.n_levels")
