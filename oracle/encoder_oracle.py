"""ORACLE ONLY -- test infrastructure, never the product path.

A numpy restatement of the reference's encoders: the image families (jepa_encode_image /
jepa_build_encoder_image, src/jepa.cpp:586-720) and the video families (jepa_encode_video /
jepa_build_encoder_video, src/jepa.cpp:750-1000: tubelet patches, 3-D RoPE, modality vectors, LeVJEPA's CLS
and block-causal attention); the block is jepa_build_block, src/jepa.cpp:444-471. Only tests/ may import it,
and only as the checker.

Parity pin: checked against outputs of the reference's executable numpy specifications of the same graphs
(scripts/jepa_convert/selftest.py `encoder_forward` and `levjepa_encoder_forward`,
scripts/jepa_convert/vjepa2_numpy_ref.py `encoder_forward`), committed as tests/golden/encode_ref.npz and
tests/golden/encode_video_ref.npz by tests/golden/make_golden_encode.py and make_golden_video.py.
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


def _act(name):
    """The encoder MLP's activation by its jepa.enc.act name (scripts/jepa_convert/selftest.py:104-111 `act_fn`;
    relu as the loader accepts it, src/jepa-gguf.cpp:26-35)."""
    if name == "gelu_tanh":
        return lambda x: (0.5 * x * (1 + np.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))).astype(f32)
    if name == "silu":
        return lambda x: (x / (1.0 + np.exp(-x))).astype(f32)
    if name == "relu":
        return lambda x: np.maximum(x, 0).astype(f32)
    return _gelu


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
    act = _act(str(g("act", "gelu_erf")))
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
            f = act(h @ T[b + "ffn_up.weight"].T + T.get(b + "ffn_up.bias", 0))
            f = f @ T[b + "ffn_down.weight"].T + T.get(b + "ffn_down.bias", 0)
            if b + "ls2" in T:
                f = f * T[b + "ls2"]
            x = (x + f).astype(f32)
        out.append(_ln(x, T["enc.norm.weight"], T["enc.norm.bias"], eps))
    return np.concatenate(out, 0)


# ---------------------------------------------------------------------------------------------
# video encoders (V-JEPA 2 / 2.1, LeVJEPA): src/jepa.cpp:750-1000, the shape rules of
# jepa_video_shape_for (:761-803) and the 3-D RoPE tables of src/rope3d.cpp
# ---------------------------------------------------------------------------------------------
def tubelet_rows(clip, tub, P):
    """clip [C][T][H][W] -> [gt gh gw][C tub P P]: tokens t-major, then h, then w; C, frame, row, column inside a
    row (the Conv3d weight flattened row-major; jepa_patchify)."""
    C, T, H, W = clip.shape
    gt, gh, gw = T // tub, H // P, W // P
    x = clip[:, :gt * tub, :gh * P, :gw * P].reshape(C, gt, tub, gh, P, gw, P).transpose(1, 3, 5, 0, 2, 4, 6)
    return np.ascontiguousarray(x.reshape(gt * gh * gw, C * tub * P * P))


def rope3d(gt, gh, gw, hd, theta, layout, n_prefix=0, ref_grid=0):
    """cos / sin [n_prefix + gt gh gw][hd]: lanes [0, d) by the temporal position, [d, 2d) the row, [2d, 3d) the
    column, d = 2 ((hd // 3) // 2), the rest identity; frequency k = theta^(-k / (d / 2)); 'tiled' repeats the
    d/2 frequencies as two halves, 'interleaved' doubles each; ref_grid > 0 rescales rows and columns to a
    ref_grid x ref_grid grid; identity rows for the prefix tokens (they are not on the grid)."""
    n = gt * gh * gw
    i = np.arange(n)
    pos = [(i // (gh * gw)).astype(np.float64), ((i % (gh * gw)) // gw).astype(np.float64),
           ((i % (gh * gw)) % gw).astype(np.float64)]
    if ref_grid:
        if gh > 1:
            pos[1] = pos[1] * (ref_grid - 1) / (gh - 1)
        if gw > 1:
            pos[2] = pos[2] * (ref_grid - 1) / (gw - 1)
    d = 2 * ((hd // 3) // 2)
    omega = 1.0 / float(theta) ** (np.arange(d // 2, dtype=np.float64) / (d / 2.0))
    cos = np.ones((n_prefix + n, hd), f32)
    sin = np.zeros((n_prefix + n, hd), f32)
    for ax in range(3):
        f = pos[ax][:, None] * omega[None, :]
        c, s = np.cos(f), np.sin(f)
        if layout == "interleaved":
            c, s = np.repeat(c, 2, -1), np.repeat(s, 2, -1)
        else:
            c, s = np.concatenate([c, c], -1), np.concatenate([s, s], -1)
        cos[n_prefix:, ax * d:(ax + 1) * d] = c
        sin[n_prefix:, ax * d:(ax + 1) * d] = s
    return cos, sin


def _rope(x, cos, sin):
    """x [H][N][hd]: pairs (2k, 2k + 1) -> x cos + (-x[2k+1], x[2k]) sin."""
    r = np.empty_like(x)
    r[..., 0::2] = -x[..., 1::2]
    r[..., 1::2] = x[..., 0::2]
    return (x * cos[None] + r * sin[None]).astype(f32)


def encode_video(path: str, clips) -> np.ndarray:
    """clips [B][C][T][H][W] -> [B N][D]: every clip its own sequence (N = prefix + gt gh gw)."""
    T_, meta = load_tensors(path)
    g = lambda k, d=None: meta.get("jepa.enc." + k, d)
    D, P, H = int(g("embed_dim")), int(g("patch_size")), int(g("n_head"))
    eps = float(g("ln_eps", 1e-6))
    act = _act(str(g("act", "gelu_erf")))
    hd = D // H
    out = []
    for clip in np.asarray(clips, f32):
        C, T, Hh, Ww = clip.shape
        image_path = T == 1 and bool(g("image_patch_embed", False)) and "enc.patch_embed_img.weight" in T_
        tub = 1 if image_path else int(g("tubelet_size", 1))
        gt, gh, gw = T // tub, Hh // P, Ww // P
        pw = "enc.patch_embed_img" if image_path else "enc.patch_embed"
        x = tubelet_rows(clip, tub, P) @ T_[pw + ".weight"].T + T_[pw + ".bias"]
        if g("modality_embed", False):
            x = x + T_["enc.mod_embed_img" if image_path else "enc.mod_embed_video"]
        n_prefix = 1 if g("cls_token", False) else 0
        if n_prefix:
            x = np.concatenate([T_["enc.cls_token"].reshape(1, D), x], 0)
        x = x.astype(f32)
        cos, sin = rope3d(gt, gh, gw, hd, float(g("rope_theta", 10000.0)), str(g("rope_freq_layout", "tiled")), n_prefix,
                          int(g("rope_ref_grid", 0)) if g("rope_interpolate", False) else 0)
        N = x.shape[0]
        allow = np.ones((N, N), bool)
        if str(g("attn_mode", "full")) == "block_causal":
            slot = np.arange(N - n_prefix) // (gh * gw)
            allow[n_prefix:, :] = False
            allow[n_prefix:, n_prefix:] = slot[:, None] >= slot[None, :]
        for i in range(int(g("n_layer"))):
            b = f"enc.blk.{i}."
            h = _ln(x, T_[b + "ln1.weight"], T_[b + "ln1.bias"], eps)
            qkv = (h @ T_[b + "attn_qkv.weight"].T + T_.get(b + "attn_qkv.bias", 0)).astype(f32)
            q, k, v = (qkv[:, j * D:(j + 1) * D].reshape(-1, H, hd).transpose(1, 0, 2) for j in range(3))
            q, k = _rope(q, cos, sin), _rope(k, cos, sin)
            s = np.where(allow[None], (q @ k.transpose(0, 2, 1)) / math.sqrt(hd), -np.inf)
            p = np.exp(s - s.max(-1, keepdims=True))
            a = ((p / p.sum(-1, keepdims=True)) @ v).transpose(1, 0, 2).reshape(-1, D).astype(f32)
            x = (x + a @ T_[b + "attn_out.weight"].T + T_.get(b + "attn_out.bias", 0)).astype(f32)
            h = _ln(x, T_[b + "ln2.weight"], T_[b + "ln2.bias"], eps)
            f = act(h @ T_[b + "ffn_up.weight"].T + T_.get(b + "ffn_up.bias", 0))
            x = (x + f @ T_[b + "ffn_down.weight"].T + T_.get(b + "ffn_down.bias", 0)).astype(f32)
        out.append(_ln(x, T_["enc.norm.weight"], T_["enc.norm.bias"], eps))
    return np.concatenate(out, 0)
