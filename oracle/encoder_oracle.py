"""ORACLE ONLY -- test infrastructure, never the product path.

A numpy restatement of the reference's image encoder (jepa_encode for the image families:
jepa_encode_image / jepa_build_encoder_image, src/jepa.cpp:586-720; the block jepa_build_block,
src/jepa.cpp:444-471). Only tests/ may import it, and only as the checker.

Parity pin: checked against outputs of the reference's executable numpy specification of the same graph
(scripts/jepa_convert/selftest.py `encoder_forward`), committed as tests/golden/encode_ref.npz by
tests/golden/make_golden_encode.py.
"""
from __future__ import annotations

import math

import numpy as np

from hjepa_oracle import load_tensors

f32 = np.float32


def _ln(x, w, b, eps):
    mu = x.mean(-1, keepdims=True, dtype=np.float64)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    y = ((x - mu) / np.sqrt(var + eps)).astype(f32)
    return (y * w + b).astype(f32)


def _gelu(x):
    from scipy.special import erf
    return (0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))).astype(f32)


def patch_rows(img, P):
    """img [C][H][W] -> [n_patches][C P P]: patches h-major, C, then P x P inside a row (jepa_patchify)."""
    C, H, W = img.shape
    gh, gw = H // P, W // P
    x = img[:, :gh * P, :gw * P].reshape(C, gh, P, gw, P).transpose(1, 3, 0, 2, 4)
    return np.ascontiguousarray(x.reshape(gh * gw, C * P * P))


def encode(path: str, images) -> np.ndarray:
    """images [B][C][H][W] -> [B N][D], every image its own sequence, rows concatenated in batch order."""
    T, meta = load_tensors(path)
    g = lambda k, d=None: meta.get("jepa.enc." + k, d)
    D, P, H = int(g("embed_dim")), int(g("patch_size")), int(g("n_head"))
    eps = float(g("ln_eps", 1e-6))
    n_reg = int(g("n_registers", 0) or 0)
    out = []
    for img in np.asarray(images, f32):
        x = patch_rows(img, P) @ T["enc.patch_embed.weight"].T + T["enc.patch_embed.bias"]
        pre = []
        if g("cls_token", False):
            pre.append(T["enc.cls_token"].reshape(1, D))
        if n_reg:
            pre.append(T["enc.reg_tokens"].reshape(n_reg, D))
        x = (np.concatenate(pre + [x], 0) + T["enc.pos_embed"]).astype(f32)
        hd = D // H
        for i in range(int(g("n_layer"))):
            b = f"enc.blk.{i}."
            h = _ln(x, T[b + "ln1.weight"], T[b + "ln1.bias"], eps)
            qkv = (h @ T[b + "attn_qkv.weight"].T + T.get(b + "attn_qkv.bias", 0)).astype(f32)
            q, k, v = (qkv[:, j * D:(j + 1) * D].reshape(-1, H, hd).transpose(1, 0, 2) for j in range(3))
            s = (q @ k.transpose(0, 2, 1)) / math.sqrt(hd)
            p = np.exp(s - s.max(-1, keepdims=True))
            a = ((p / p.sum(-1, keepdims=True)) @ v).transpose(1, 0, 2).reshape(-1, D).astype(f32)
            a = a @ T[b + "attn_out.weight"].T + T.get(b + "attn_out.bias", 0)
            if b + "ls1" in T:
                a = a * T[b + "ls1"]
            x = (x + a).astype(f32)
            h = _ln(x, T[b + "ln2.weight"], T[b + "ln2.bias"], eps)
            f = _gelu(h @ T[b + "ffn_up.weight"].T + T.get(b + "ffn_up.bias", 0))
            f = f @ T[b + "ffn_down.weight"].T + T.get(b + "ffn_down.bias", 0)
            if b + "ls2" in T:
                f = f * T[b + "ls2"]
            x = (x + f).astype(f32)
        out.append(_ln(x, T["enc.norm.weight"], T["enc.norm.bias"], eps))
    return np.concatenate(out, 0)
