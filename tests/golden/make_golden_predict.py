"""Writes tests/golden/hjepa_predict_ref.npz: outputs of the reference's executable numpy specification of the
H-JEPA multi-frame predictor (scripts/jepa_convert/hjepa_numpy_ref.py: predict / rollout, which mirror
jepa_hjepa_predict / jepa_hjepa_rollout of src/hjepa.cpp) on seeded forged models.

The specification is imported from the reference tree, which only this generator reads; the tests read the
committed fixture. Run (from the repository root, with the reference checked out at $JEPA_REF):

    JEPA_REF=/path/to/jepa.cpp python tests/golden/make_golden_predict.py

Cases: every frame count 1..n_frames of every level (predict), and rollouts from one and two seed frames at
every history 1..n_frames, on 'pa' (2 levels, f32; level 1 with an action-embedding MLP, an output projection
and a projection MLP; level 2 with a 32-wide predictor inside 64-wide states, so in_proj / out_proj) and 'pb'
(1 level, q8_0, the 'adaln_bare' predictor: its own action embedder, no inner norms); 'pc' (2 levels, an mlp
projector and a proprio stream into the level-1 state, a 2-layer 'seq' action encoder at stride 3) and 'pd'
(a layernorm projector) add the state and action encoders: embed, lift, action_embed and action_encode at
whole and ragged chunk counts (jepa_hjepa_embed / _lift / _action_embed / _action_encode).
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

OUT = os.path.join(HERE, "hjepa_predict_ref.npz")


def model_specs():
    """name -> (spec, seed) of the forged models."""
    A1 = synth.Level(64, 2, 2, 128, 2, act_embed_hidden=16, act_embed_dim=8, out_proj=True, proj_hidden=32, n_frames=4)
    A2 = synth.Level(64, 2, 2, 128, 4, stride=2, enc_kind="latent_mlp", enc_hidden=48, act_enc_kind="mlp", pred_dim=32,
                     n_frames=3)
    pa = synth.HJepaSpec(levels=[A1, A2], ftype="f32", rand_all=True, cond_std=0.3, w_std=0.1, name="golden-pa")
    B1 = synth.Level(96, 2, 3, 192, 3, n_frames=5, pred_kind="adaln_bare")
    pb = synth.HJepaSpec(levels=[B1], ftype="q8_0", rand_all=True, cond_std=0.3, w_std=0.1, name="golden-pb")
    C1 = synth.Level(48, 2, 2, 96, 2, act_embed_hidden=16, act_embed_dim=8, enc_kind="vit_proprio", n_frames=3)
    C2 = synth.Level(48, 2, 2, 96, 4, stride=3, enc_kind="latent_mlp", enc_hidden=32, act_enc_kind="seq", act_enc_dim=32,
                     act_enc_n_layer=2, act_enc_n_head=2, n_frames=3)
    pc = synth.HJepaSpec(levels=[C1, C2], ftype="f32", rand_all=True, cond_std=0.3, w_std=0.1, name="golden-pc",
                         enc_dim=40, proj_kind="mlp", proj_hidden=24, proprio_dim=7, proprio_hidden=12, proprio_out=16)
    D1 = synth.Level(64, 1, 2, 128, 2, n_frames=2)
    pd = synth.HJepaSpec(levels=[D1], ftype="f32", rand_all=True, cond_std=0.3, w_std=0.1, name="golden-pd",
                         proj_kind="layernorm")
    return {"pa": (pa, 31), "pb": (pb, 32), "pc": (pc, 33), "pd": (pd, 34)}


def build_model(name: str, workdir: str) -> tuple[str, str]:
    spec, seed = model_specs()[name]
    path = os.path.join(workdir, f"golden-{name}.gguf")
    synth.write_hjepa(path, spec, seed=seed)
    with open(path, "rb") as f:
        digest = hashlib.sha256(f.read()).hexdigest()
    return path, digest


def main() -> None:
    ref = os.environ.get("JEPA_REF")
    if not ref:
        sys.exit("set JEPA_REF to the reference checkout (its scripts/jepa_convert is imported)")
    sys.path.insert(0, os.path.join(ref, "scripts"))
    from jepa_convert import hjepa_numpy_ref as HJ
    from jepa_convert import selftest as ST

    out: dict[str, np.ndarray] = {}
    meta: dict = {"models": {}, "cases": []}
    rng = np.random.default_rng(909)
    with tempfile.TemporaryDirectory() as tmp:
        for name, (spec, _) in model_specs().items():
            path, digest = build_model(name, tmp)
            meta["models"][name] = digest
            m = ST.Model(path)
            for k, lv in enumerate(spec.levels, start=1):
                D, A, nf = lv.embed_dim, lv.action_dim, lv.n_frames
                for T in range(1, nf + 1):
                    key = f"{name}.l{k}.predict{T}"
                    s = rng.normal(size=(T, D)).astype(np.float32)
                    a = rng.uniform(-1.0, 1.0, (T, A)).astype(np.float32)
                    y = HJ.predict(m, k, s, a).astype(np.float32)
                    out[f"{key}.states"], out[f"{key}.actions"], out[f"{key}.out"] = s, a, y
                    meta["cases"].append({"key": key, "kind": "predict", "model": name, "level": k, "T": T})
                for n_seed in (1, 2):
                    n_steps = 5
                    seeds = rng.normal(size=(n_seed, D)).astype(np.float32)
                    acts = rng.uniform(-1.0, 1.0, (n_seed + n_steps - 1, A)).astype(np.float32)
                    for hist in range(1, nf + 1):
                        key = f"{name}.l{k}.rollout_s{n_seed}_h{hist}"
                        y = HJ.rollout(m, k, seeds, acts, hist).astype(np.float32)
                        assert y.shape == (n_steps, D)
                        out[f"{key}.seeds"], out[f"{key}.actions"], out[f"{key}.out"] = seeds, acts, y
                        meta["cases"].append({"key": key, "kind": "rollout", "model": name, "level": k,
                                              "n_seed": n_seed, "n_steps": n_steps, "history": hist})
        # the state and action encoders (their own draws, so the cases above keep their inputs)
        rng2 = np.random.default_rng(910)
        for name, (spec, _) in model_specs().items():
            path, _ = build_model(name, tmp)
            m = ST.Model(path)
            L = spec.levels
            Dv = spec.enc_dim or (L[0].embed_dim - (spec.proprio_out if spec.proprio_dim else 0))
            key = f"{name}.embed"
            cls = rng2.normal(size=(5, Dv)).astype(np.float32)
            pro = rng2.normal(size=(5, spec.proprio_dim)).astype(np.float32) if spec.proprio_dim else None
            out[f"{key}.cls"], out[f"{key}.out"] = cls, HJ.embed(m, cls, pro).astype(np.float32)
            if pro is not None:
                out[f"{key}.proprio"] = pro
            meta["cases"].append({"key": key, "kind": "embed", "model": name, "level": 1, "proprio": pro is not None})
            for k, lv in enumerate(L, start=1):
                key = f"{name}.l{k}.action_embed"
                a = rng2.uniform(-1.0, 1.0, (7, lv.action_dim)).astype(np.float32)
                out[f"{key}.in"], out[f"{key}.out"] = a, HJ.act_embed(m, k, a).astype(np.float32)
                meta["cases"].append({"key": key, "kind": "action_embed", "model": name, "level": k})
                if k == 1:
                    continue
                for n_rows in (lv.stride * 3, lv.stride * 2 + 1):
                    key = f"{name}.l{k}.lift{n_rows}"
                    below = rng2.normal(size=(n_rows, L[k - 2].embed_dim)).astype(np.float32)
                    out[f"{key}.in"], out[f"{key}.out"] = below, HJ.lift(m, k, below).astype(np.float32)
                    meta["cases"].append({"key": key, "kind": "lift", "model": name, "level": k})
                    key = f"{name}.l{k}.action_encode{n_rows}"
                    emb = rng2.normal(size=(n_rows, L[k - 2].E())).astype(np.float32)
                    chunks, n_valid = HJ.act_chunks(emb, lv.stride)
                    out[f"{key}.in"], out[f"{key}.out"] = emb, HJ.act_encode(m, k, chunks, n_valid).astype(np.float32)
                    meta["cases"].append({"key": key, "kind": "action_encode", "model": name, "level": k})
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(meta['cases'])} cases")


if __name__ == "__main__":
    main()
