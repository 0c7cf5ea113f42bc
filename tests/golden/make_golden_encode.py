"""Writes tests/golden/encode_ref.npz: outputs of the reference's executable numpy specification of the image
encoder (scripts/jepa_convert/selftest.py `encoder_forward`, the graph jepa_encode builds for the image
families, src/jepa.cpp:586-632) on seeded forged models and seeded images.

The specification is imported from the reference tree, which only this generator reads; the tests read the
committed fixture and regenerate the same models and images from their seeds. Run (from the repository root,
with the reference checked out at $JEPA_REF):

    JEPA_REF=/path/to/jepa.cpp python tests/golden/make_golden_encode.py

Models: 'ea' (f32, 96 wide, 3 heads of 32, 2 blocks), 'eb' (q8_0 blocks, 128 wide, 2 heads of 64, 1 block) and
'ec' (f16, 64 wide, 2 heads of 32, 1 block, the tanh form of GELU that HF ViT checkpoints use); all encode
224 x 224 images in 14 x 14 patches (256 patches + CLS). Images are N(0, 1) per pixel (seed).
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
sys.path.insert(0, os.path.join(ROOT, "jepa.cpp_b200"))

from jepa_b200 import synth  # noqa: E402

OUT = os.path.join(HERE, "encode_ref.npz")


def model_specs():
    """name -> (spec, seed, n_images) of the forged models (an H-JEPA file carries its image encoder)."""
    L = synth.Level(64, 1, 2, 128, 2)
    ea = synth.HJepaSpec(levels=[L], ftype="f32", rand_all=True, w_std=0.1, name="golden-ea", enc_dim=96, enc_layers=2,
                         enc_heads=3, enc_ffn=192)
    eb = synth.HJepaSpec(levels=[L], ftype="q8_0", rand_all=True, w_std=0.1, name="golden-eb", enc_dim=128, enc_layers=1,
                         enc_heads=2, enc_ffn=256)
    ec = synth.HJepaSpec(levels=[L], ftype="f16", rand_all=True, w_std=0.1, name="golden-ec", enc_dim=64, enc_layers=1,
                         enc_heads=2, enc_ffn=192, enc_act="gelu_tanh")
    return {"ea": (ea, 41, 2), "eb": (eb, 42, 1), "ec": (ec, 43, 1)}


def build_model(name: str, workdir: str) -> tuple[str, str]:
    spec, seed, _ = model_specs()[name]
    path = os.path.join(workdir, f"golden-{name}.gguf")
    synth.write_hjepa(path, spec, seed=seed)
    with open(path, "rb") as f:
        digest = hashlib.sha256(f.read()).hexdigest()
    return path, digest


def images(name: str) -> np.ndarray:
    """The seeded NCHW batch of a model's case."""
    _, seed, n = model_specs()[name]
    return np.random.default_rng(1000 + seed).normal(size=(n, 3, 224, 224)).astype(np.float32)


def main() -> None:
    ref = os.environ.get("JEPA_REF")
    if not ref:
        sys.exit("set JEPA_REF to the reference checkout (its scripts/jepa_convert is imported)")
    sys.path.insert(0, os.path.join(ref, "scripts"))
    from jepa_convert import selftest as ST

    out: dict[str, np.ndarray] = {}
    meta: dict = {"models": {}}
    with tempfile.TemporaryDirectory() as tmp:
        for name in model_specs():
            path, digest = build_model(name, tmp)
            meta["models"][name] = digest
            m = ST.Model(path)
            out[name] = np.concatenate([ST.encoder_forward(m, img).astype(np.float32) for img in images(name)], 0)
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {', '.join(f'{k} {v.shape}' for k, v in out.items() if k != 'meta')}")


if __name__ == "__main__":
    main()
