"""Writes the V-JEPA 2-AC golden fixtures from the REFERENCE's own executable spec:

  tests/golden/ac_spec.npz     predictions of scripts/jepa_convert/selftest.py::ac_predictor_forward (the
                               reference's numpy spec of jepa.pred.kind == "ac") on a seeded forged model,
                               for 1, 2 and 3 context frames
  tests/golden/rope3d_hf.npz   the reference's RoPE golden vectors for the tiled layout the AC predictor
                               uses (tests/vectors/rope3d/hd64_*_hf_*), copied so the GPU box has them

    JEPA_REF=/path/to/jepa.cpp python tests/golden/make_golden_ac.py     (needs the reference checkout)

The model is not stored: tests rebuild it from MODEL (synth spec + seed) and check its sha256.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("JEPA_REF", "")
sys.path.insert(0, os.path.join(ROOT, "jepa.cpp_b200"))

from jepa_b200 import synth  # noqa: E402


def model_spec():
    return synth.ACSpec(enc_dim=96, pred_dim=64, n_layer=2, n_head=4, ffn_dim=128, grid=4, n_frames=4, ftype="f32",
                        rand_all=True, w_std=0.1, name="golden-ac"), 21


def build_model(workdir: str) -> tuple[str, str]:
    spec, seed = model_spec()
    path = os.path.join(workdir, "golden-ac.gguf")
    synth.write_ac(path, spec, seed=seed)
    with open(path, "rb") as f:
        return path, hashlib.sha256(f.read()).hexdigest()


def main() -> None:
    if not REF:
        sys.exit("set JEPA_REF to the reference checkout (its scripts/jepa_convert is imported)")
    sys.path.insert(0, os.path.join(REF, "scripts", "jepa_convert"))
    import selftest   # the reference's numpy spec (read-only import from the reference tree)
    out = {}
    rng = np.random.default_rng(77)
    with tempfile.TemporaryDirectory() as tmp:
        path, digest = build_model(tmp)
        m = selftest.Model(path)
        spec, _ = model_spec()
        HW = spec.grid * spec.grid
        for T in (1, 2, 3):
            ctx = rng.normal(size=(T * HW, spec.enc_dim)).astype(np.float32)
            act = rng.normal(0, 0.5, size=(T, spec.action_dim)).astype(np.float32)
            st = rng.normal(0, 0.5, size=(T, spec.state_dim)).astype(np.float32)
            pred = selftest.ac_predictor_forward(m, ctx, act, st).astype(np.float32)
            out[f"T{T}.context"], out[f"T{T}.actions"], out[f"T{T}.states"], out[f"T{T}.pred"] = ctx, act, st, pred
    out["meta"] = np.frombuffer(json.dumps({"model": digest}).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, "ac_spec.npz"), **out)
    vec = os.path.join(REF, "tests", "vectors", "rope3d")
    rope = {}
    for case in ("hd64_g4x4x4", "hd64_g8x16x16_sub"):
        rope[f"{case}.x"] = np.load(os.path.join(vec, f"{case}_x.npy"))
        rope[f"{case}.out"] = np.load(os.path.join(vec, f"{case}_hf_out.npy"))
        ids_path = os.path.join(vec, f"{case}_ids.npy")
        rope[f"{case}.ids"] = np.load(ids_path) if os.path.exists(ids_path) else np.arange(rope[f"{case}.x"].shape[0])
    rope["grids"] = np.array([[4, 4, 4], [8, 16, 16]], np.int64)
    np.savez_compressed(os.path.join(HERE, "rope3d_hf.npz"), **rope)
    print("wrote ac_spec.npz and rope3d_hf.npz")


if __name__ == "__main__":
    main()
