"""Writes tests/golden/encode_video_ref.npz: outputs of the reference's executable numpy specifications of the
video encoders on seeded forged models and seeded clips --
  * V-JEPA 2 / 2.1: scripts/jepa_convert/vjepa2_numpy_ref.py `encoder_forward` (tubelet patches, 3-D RoPE in the
    tiled or interleaved layout, modality vectors, the 2.1 one-frame image tokenizer, position interpolation);
  * LeVJEPA: scripts/jepa_convert/selftest.py `levjepa_encoder_forward` (CLS token, block-causal attention).
The graph they specify is jepa_encode_video / jepa_build_encoder_video (src/jepa.cpp:750-1000).

The specifications are imported from the reference tree, which only this generator reads; the tests read the
committed fixture and regenerate the same models and clips from their seeds. Run (from the repository root,
with the reference checked out at $JEPA_REF):

    JEPA_REF=/path/to/jepa.cpp python tests/golden/make_golden_video.py
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

OUT = os.path.join(HERE, "encode_video_ref.npz")


def cases():
    """name -> (spec, seed, clip shapes [C, T, H, W] encoded one clip at a time)."""
    va = synth.VideoEncSpec(family="vjepa2", dim=128, n_layer=2, n_head=2, ffn_dim=256, tubelet=2, ftype="f32",
                            rope_layout="tiled", name="golden-va")
    vb = synth.VideoEncSpec(family="vjepa2_1", dim=96, n_layer=2, n_head=2, ffn_dim=192, tubelet=2, ftype="q8_0",
                            rope_layout="interleaved", modality_embed=True, image_patch_embed=True, name="golden-vb")
    vc = synth.VideoEncSpec(family="levjepa", dim=128, n_layer=2, n_head=2, ffn_dim=256, tubelet=1, ftype="f32",
                            rope_layout="tiled", cls_token=True, block_causal=True, name="golden-vc")
    vd = synth.VideoEncSpec(family="vjepa2", dim=192, n_layer=1, n_head=3, ffn_dim=256, tubelet=2, ftype="f32",
                            rope_layout="tiled", rope_interpolate=True, rope_ref_grid=4, rope_theta=5000.0, name="golden-vd")
    return {"va": (va, 51, [(3, 4, 32, 48), (3, 4, 32, 48)]),
            "vb": (vb, 52, [(3, 4, 32, 32), (3, 1, 32, 32)]),
            "vc": (vc, 53, [(3, 3, 32, 32)]),
            "vd": (vd, 54, [(3, 2, 32, 48)])}


def build_model(name: str, workdir: str) -> tuple[str, str]:
    spec, seed, _ = cases()[name]
    path = os.path.join(workdir, f"golden-{name}.gguf")
    synth.write_video_encoder(path, spec, seed=seed)
    with open(path, "rb") as f:
        digest = hashlib.sha256(f.read()).hexdigest()
    return path, digest


def clips(name: str) -> list:
    """The seeded clips of a case, N(0, 1) per pixel."""
    _, seed, shapes = cases()[name]
    rng = np.random.default_rng(2000 + seed)
    return [rng.normal(size=s).astype(np.float32) for s in shapes]


def main() -> None:
    ref = os.environ.get("JEPA_REF")
    if not ref:
        sys.exit("set JEPA_REF to the reference checkout (its scripts/jepa_convert is imported)")
    sys.path.insert(0, os.path.join(ref, "scripts"))
    sys.path.insert(0, os.path.join(ref, "scripts", "jepa_convert"))
    from jepa_convert import selftest as ST
    import vjepa2_numpy_ref as VR

    out: dict[str, np.ndarray] = {}
    meta: dict = {"models": {}}
    with tempfile.TemporaryDirectory() as tmp:
        for name, (spec, _, _) in cases().items():
            path, digest = build_model(name, tmp)
            meta["models"][name] = digest
            for i, clip in enumerate(clips(name)):
                if spec.family == "levjepa":
                    y = ST.levjepa_encoder_forward(ST.Model(path), clip)
                else:
                    kv, W = VR.load_gguf(path)
                    mode = "image" if clip.shape[1] == 1 and spec.image_patch_embed else "video"
                    y, _ = VR.encoder_forward(kv, W, clip, mode=mode)
                out[f"{name}.{i}"] = np.asarray(y, np.float32)
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {', '.join(f'{k} {v.shape}' for k, v in out.items() if k != 'meta')}")


if __name__ == "__main__":
    main()
