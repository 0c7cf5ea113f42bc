"""Seeded synthetic GGUF models in jepa.cpp's schema, and the benchmark configurations.

There is no network and no released checkpoint here, so every model the tests and the benchmark
run is generated: weights N(0, 0.02), biases 0, LayerNorm gamma 1 / beta 0, from
numpy.random.default_rng(seed) -- the rule of the benchmark configurations -- or, for the forged
test models, every parameter random (``rand_all``) so that biases, norms and the optional layers
carry signal. Tensor names, shapes and metadata keys follow the hjepa schema
(reference: docs/gguf-schema.md "hjepa", src/jepa-gguf.cpp:480-550, src/hjepa.cpp:96-241) and which
tensors get quantised follows the reference quantiser's rule (tools/jepa-quantize.cpp:90-129).
"""
from __future__ import annotations

import copy
import dataclasses as dc
from typing import Optional

import numpy as np

from .gguf_write import FTYPE, GGML_F32, TYPE_OF_FTYPE, GGUFWriter


@dc.dataclass
class Level:
    embed_dim: int
    n_layer: int
    n_head: int
    ffn_dim: int
    action_dim: int
    pred_dim: int = 0              # 0 = embed_dim
    head_dim: int = 0              # 0 = pred_dim / n_head
    n_frames: int = 3              # rows of pred.pos_embed (the predictor's context window)
    stride: int = 1
    act_embed_hidden: int = 0      # > 0: act_embed.{0,2} MLP present
    act_embed_dim: int = 0         # width of act_embed(a); = action_dim when absent
    enc_kind: str = "vit"          # level 1: vit ; above: latent_mlp | identity
    enc_hidden: int = 0
    enc_out_norm: bool = True
    act_enc_kind: str = "none"     # none (level 1) | mlp | seq
    act_enc_hidden: int = 64
    act_enc_dim: int = 32          # seq encoder width
    act_enc_n_layer: int = 1
    act_enc_n_head: int = 2
    act_enc_out_norm: bool = True
    pred_kind: str = "adaln"       # adaln | adaln_bare
    pact_hidden: int = 0           # adaln_bare: pred.act_embed MLP hidden width
    pact_dim: int = 0              # adaln_bare: its output width (0 = pred_dim)
    out_proj: bool = False
    proj_hidden: int = 0           # > 0: pred.proj.{0,2} MLP present
    act_queue: int = 0             # rows of recorded latent actions (0 = none)

    def P(self) -> int:
        return self.pred_dim or self.embed_dim

    def E(self) -> int:
        return self.act_embed_dim if self.act_embed_hidden else self.action_dim

    def hd(self) -> int:
        return self.head_dim or self.P() // self.n_head


@dc.dataclass
class HJepaSpec:
    levels: list
    ftype: str = "f32"
    enc_dim: int = 0               # encoder stub width (0 = level-1 embed_dim)
    enc_layers: int = 1
    enc_heads: int = 0
    enc_ffn: int = 0
    enc_act: str = "gelu_erf"      # jepa.enc.act of the encoder stub: gelu_erf | gelu_tanh | silu | relu
    enc_qkv_fused: bool = True     # False: the same q / k / v rows written as attn_q, attn_k, attn_v
    rand_all: bool = False         # every parameter random (forged test models)
    w_std: float = 0.02
    cond_std: float = 0.02         # cond_proj / adaln / act_embed init std
    name: str = "synthetic-hjepa"
    proj_kind: str = "identity"    # level-1 projector of the encoder's CLS row: identity | mlp | layernorm
    proj_hidden: int = 0           # mlp projector hidden width (0 = 2 enc_dim)
    proprio_dim: int = 0           # > 0: level 1 is 'vit_proprio' (set its enc_kind), a proprio stream fused in
    proprio_hidden: int = 32
    proprio_out: int = 16          # width of the proprio part of the level-1 state


def _quantizable(name: str) -> bool:
    """tools/jepa-quantize.cpp:90-129 restated: which 2-D weights a quantised file stores quantised."""
    if not name.endswith(".weight"):
        return False
    keep = ("patch_embed", "pos_embed", "cls_token", "reg_tokens", "mask_tokens", "mod_embed", ".adaln.",
            "action_embed", "state_embed", ".ln1.", ".ln2.", ".norm.", "hier_norm", "ln_kv", "head.query",
            ".act_enc.", ".act_embed.", "act_queue")
    if any(k in name for k in keep):
        return False
    if any(c in name for c in (".attn_qkv.", ".attn_q.", ".attn_k.", ".attn_v.", ".attn_out.", ".ffn_up.", ".ffn_down.")):
        return True
    if any(name.startswith(p) for p in ("pred.proj", "pred.embed", "enc.proj.", "head.cls.", "head.xattn.")):
        return True
    if name.startswith("lvl."):
        parts = (".enc.proj.", ".enc.fc1.", ".enc.fc2.", ".pred.proj.", ".pred.in_proj.", ".pred.cond_proj.", ".pred.out_proj.")
        return any(c in name for c in parts)
    return False


class _Gen:
    def __init__(self, spec: HJepaSpec, seed: int):
        self.spec = spec
        self.rng = np.random.default_rng(seed)
        self.w = GGUFWriter()
        self.qtype = TYPE_OF_FTYPE[spec.ftype]

    def tensor(self, name: str, x: np.ndarray) -> None:
        t = self.qtype if (self.qtype != GGML_F32 and x.ndim == 2 and _quantizable(name)) else GGML_F32
        self.w.add_tensor(name, x, t)

    def lin(self, name: str, n_in: int, n_out: int, bias: bool = True, std: Optional[float] = None) -> None:
        s = self.spec.w_std if std is None else std
        self.tensor(name + ".weight", self.rng.normal(0.0, s, (n_out, n_in)).astype(np.float32))
        if bias:
            b = self.rng.normal(0.0, s, n_out) if self.spec.rand_all else np.zeros(n_out)
            self.tensor(name + ".bias", b.astype(np.float32))

    def lin_split(self, names: list, n_in: int, n_out: int) -> None:
        """lin() of one [n_out][n_in] linear (the same draws), written as len(names) linears of equal row slices."""
        s = self.spec.w_std
        wt = self.rng.normal(0.0, s, (n_out, n_in)).astype(np.float32)
        b = (self.rng.normal(0.0, s, n_out) if self.spec.rand_all else np.zeros(n_out)).astype(np.float32)
        k = n_out // len(names)
        for i, nm in enumerate(names):
            self.tensor(nm + ".weight", np.ascontiguousarray(wt[i * k:(i + 1) * k]))
        for i, nm in enumerate(names):
            self.tensor(nm + ".bias", np.ascontiguousarray(b[i * k:(i + 1) * k]))

    def norm(self, name: str, d: int) -> None:
        if self.spec.rand_all:
            self.tensor(name + ".weight", (1.0 + self.rng.normal(0.0, 0.1, d)).astype(np.float32))
            self.tensor(name + ".bias", self.rng.normal(0.0, 0.1, d).astype(np.float32))
        else:
            self.tensor(name + ".weight", np.ones(d, np.float32))
            self.tensor(name + ".bias", np.zeros(d, np.float32))


def write_hjepa(path: str, spec: HJepaSpec, seed: int = 0) -> None:
    """Write one H-JEPA hierarchy (jepa.family = hjepa) with an hfvit encoder stub."""
    g = _Gen(spec, seed)
    w = g.w
    L = spec.levels
    q_pro = spec.proprio_out if spec.proprio_dim else 0
    pixel = L[0].embed_dim - q_pro     # the pixel part of the level-1 state
    Dv = spec.enc_dim or pixel
    eh = spec.enc_heads or max(1, Dv // 64)
    ef = spec.enc_ffn or 4 * Dv
    w.add_kv("general.architecture", "jepa")
    w.add_kv("general.name", spec.name)
    w.add_kv("general.file_type", FTYPE[spec.ftype])
    w.add_kv("jepa.schema_version", 1)
    w.add_kv("jepa.family", "hjepa")
    w.add_kv("jepa.modality", "image")
    for k, v in (("embed_dim", Dv), ("n_layer", spec.enc_layers), ("n_head", eh), ("ffn_dim", ef),
                 ("patch_size", 14), ("tubelet_size", 1), ("img_size", 224), ("n_frames", 1), ("in_chans", 3)):
        w.add_kv("jepa.enc." + k, v)
    w.add_kv("jepa.enc.ln_eps", 1e-12)
    w.add_kv("jepa.enc.act", spec.enc_act)
    w.add_kv("jepa.enc.pos_type", "learned")
    w.add_kv("jepa.enc.cls_token", True)
    w.add_kv("jepa.enc.qkv_fused", spec.enc_qkv_fused)
    # hierarchy metadata: one array entry per level, level 1 first
    w.add_kv("jepa.hjepa.n_levels", len(L))
    w.add_kv("jepa.hjepa.ln_eps", 1e-5)
    w.add_kv("jepa.hjepa.adaln_eps", 1e-6)
    w.add_kv("jepa.hjepa.proj_kind", spec.proj_kind)
    w.add_kv("jepa.hjepa.pixel_dim", pixel)
    w.add_kv("jepa.hjepa.proprio_dim", spec.proprio_dim)
    w.add_kv("jepa.hjepa.raw_action_dim", L[0].action_dim)
    w.add_kv("jepa.hjepa.frameskip", 1)
    arr = {
        "embed_dim": [l.embed_dim for l in L], "stride": [l.stride for l in L], "window": [1] * len(L),
        "target_length": [l.n_frames for l in L], "action_dim": [l.action_dim for l in L],
        "act_embed_dim": [l.E() for l in L],
        "act_enc_dim": [l.act_enc_dim if l.act_enc_kind == "seq" else 0 for l in L],
        "act_enc_n_layer": [l.act_enc_n_layer if l.act_enc_kind == "seq" else 0 for l in L],
        "act_enc_n_head": [l.act_enc_n_head if l.act_enc_kind == "seq" else 0 for l in L],
        "act_enc_max_chunk": [l.stride if l.act_enc_kind == "seq" else 0 for l in L],
        "pred_dim": [l.P() for l in L], "pred_n_layer": [l.n_layer for l in L],
        "pred_n_head": [l.n_head for l in L], "pred_head_dim": [l.hd() for l in L],
        "pred_ffn_dim": [l.ffn_dim for l in L], "pred_n_frames": [l.n_frames for l in L],
    }
    for k, v in arr.items():
        w.add_kv("jepa.hjepa." + k, v)
    w.add_kv("jepa.hjepa.enc_kind", [l.enc_kind for l in L])
    w.add_kv("jepa.hjepa.act_enc_kind", [l.act_enc_kind for l in L])
    w.add_kv("jepa.hjepa.pred_kind", [l.pred_kind for l in L])

    # encoder stub (hfvit layout); the planner never runs it
    n_tok = (224 // 14) ** 2 + 1
    g.lin("enc.patch_embed", 3 * 14 * 14, Dv)
    g.tensor("enc.pos_embed", g.rng.normal(0.0, 0.02, (n_tok, Dv)).astype(np.float32))
    g.tensor("enc.cls_token", g.rng.normal(0.0, 0.02, Dv).astype(np.float32))
    for i in range(spec.enc_layers):
        p = f"enc.blk.{i}."
        g.norm(p + "ln1", Dv)
        if spec.enc_qkv_fused:
            g.lin(p + "attn_qkv", Dv, 3 * Dv)
        else:
            g.lin_split([p + "attn_q", p + "attn_k", p + "attn_v"], Dv, 3 * Dv)
        g.lin(p + "attn_out", Dv, Dv)
        g.norm(p + "ln2", Dv)
        g.lin(p + "ffn_up", Dv, ef)
        g.lin(p + "ffn_down", ef, Dv)
    g.norm("enc.norm", Dv)

    cs = spec.cond_std
    for li, l in enumerate(L):
        k = li + 1
        p = f"lvl.{k}."
        D, P, A, E = l.embed_dim, l.P(), l.action_dim, l.E()
        if k == 1:   # the projector of the encoder's CLS row (and the proprio stream) into the level-1 state
            if spec.proj_kind == "mlp":
                ph = spec.proj_hidden or 2 * Dv
                g.lin(p + "enc.proj.0", Dv, ph)
                g.lin(p + "enc.proj.2", ph, pixel)
            elif spec.proj_kind == "layernorm":
                g.norm(p + "enc.proj_ln", Dv)
            if spec.proprio_dim:
                g.lin(p + "enc.proprio.0", spec.proprio_dim, spec.proprio_hidden)
                g.norm(p + "enc.proprio.ln", spec.proprio_hidden)
                g.lin(p + "enc.proprio.2", spec.proprio_hidden, q_pro)
        if k > 1:
            below = L[li - 1]
            if l.enc_kind == "latent_mlp":
                h = l.enc_hidden or D
                g.norm(p + "enc.in_norm", below.embed_dim)
                g.lin(p + "enc.fc1", below.embed_dim, h)
                g.lin(p + "enc.fc2", h, D)
                if l.enc_out_norm:
                    g.norm(p + "enc.out_norm", D)
            if l.act_enc_kind == "mlp":
                g.lin(p + "act_enc.fc1", l.stride * below.E(), l.act_enc_hidden, std=cs)
                g.lin(p + "act_enc.fc2", l.act_enc_hidden, A, std=cs)
                if l.act_enc_out_norm:
                    g.norm(p + "act_enc.out_norm", A)
            elif l.act_enc_kind == "seq":
                d = l.act_enc_dim
                g.lin(p + "act_enc.step", below.E(), d, std=cs)
                g.tensor(p + "act_enc.pos", g.rng.normal(0.0, cs, (l.stride + 1, d)).astype(np.float32))
                for i in range(l.act_enc_n_layer):
                    q = p + f"act_enc.blk.{i}."
                    g.norm(q + "ln1", d)
                    g.lin(q + "attn_qkv", d, 3 * d, std=cs)
                    g.lin(q + "attn_out", d, d, std=cs)
                    g.norm(q + "ln2", d)
                    g.lin(q + "ffn_up", d, 2 * d, std=cs)
                    g.lin(q + "ffn_down", 2 * d, d, std=cs)
                g.lin(p + "act_enc.head.0", d, d, std=cs)
                g.norm(p + "act_enc.head.ln", d)
                g.lin(p + "act_enc.head.2", d, A, std=cs)
                g.norm(p + "act_enc.out_norm", A)
        if l.act_embed_hidden:
            g.lin(p + "act_embed.0", A, l.act_embed_hidden, std=cs)
            g.lin(p + "act_embed.2", l.act_embed_hidden, E, std=cs)
        if l.act_queue:
            g.tensor(p + "act_queue", g.rng.normal(0.0, 1.0, (l.act_queue, A)).astype(np.float32))
        g.tensor(p + "pred.pos_embed", g.rng.normal(0.0, 0.02, (l.n_frames, D)).astype(np.float32))
        cond = E
        if l.pred_kind == "adaln_bare":
            ph = l.pact_hidden or 2 * E
            cond = l.pact_dim or P
            g.lin(p + "pred.act_embed.0", E, ph, std=cs)
            g.lin(p + "pred.act_embed.2", ph, cond, std=cs)
        if P != D:
            g.lin(p + "pred.in_proj", D, P)
        g.lin(p + "pred.cond_proj", cond, P, std=cs)   # the action Linear(A -> D) of the configs
        inner = l.n_head * l.hd()
        for i in range(l.n_layer):
            q = p + f"pred.blk.{i}."
            g.lin(q + "adaln", P, 6 * P, std=cs)
            if l.pred_kind == "adaln":
                g.norm(q + "ln1", P)
                g.norm(q + "ln2", P)
            g.lin(q + "attn_qkv", P, 3 * inner, bias=spec.rand_all)
            g.lin(q + "attn_out", inner, P)
            g.lin(q + "ffn_up", P, l.ffn_dim)
            g.lin(q + "ffn_down", l.ffn_dim, P)
        g.norm(p + "pred.norm", P)
        out = P
        if l.out_proj or (P != D and not l.proj_hidden):
            out = P if l.proj_hidden else D
            g.lin(p + "pred.out_proj", P, out)
        if l.proj_hidden:
            g.lin(p + "pred.proj.0", out, l.proj_hidden)
            g.lin(p + "pred.proj.2", l.proj_hidden, D)
    w.write(path)


# ---------------------------------------------------------------------------------------------
# V-JEPA 2-AC predictor (jepa.pred.kind = "ac"; reference: src/vjepa2_ac.cpp:86-156, the AC keys of
# src/jepa-gguf.cpp:454-480)
# ---------------------------------------------------------------------------------------------
@dc.dataclass
class ACSpec:
    enc_dim: int = 1408          # width of the encoder latents the predictor reads and writes
    pred_dim: int = 1024
    n_layer: int = 24
    n_head: int = 16
    ffn_dim: int = 4096
    grid: int = 16               # tokens per frame = grid^2
    action_dim: int = 7
    state_dim: int = 7
    n_frames: int = 8            # frame slots (jepa.pred.n_frames)
    ftype: str = "q8_0"
    w_std: float = 0.02
    rand_all: bool = False
    name: str = "synthetic-vjepa2-ac"


def write_ac(path: str, spec: ACSpec, seed: int = 0) -> None:
    """Write a V-JEPA 2-AC predictor bundle (family vjepa2, a 1-layer encoder stub of the right width)."""
    g = _Gen(HJepaSpec(levels=[], ftype=spec.ftype, rand_all=spec.rand_all, w_std=spec.w_std), seed)
    w = g.w
    D, P = spec.enc_dim, spec.pred_dim
    w.add_kv("general.architecture", "jepa")
    w.add_kv("general.name", spec.name)
    w.add_kv("general.file_type", FTYPE[spec.ftype])
    w.add_kv("jepa.schema_version", 1)
    w.add_kv("jepa.family", "vjepa2")
    w.add_kv("jepa.modality", "video")
    for k, v in (("embed_dim", D), ("n_layer", 1), ("n_head", max(1, D // 64)), ("ffn_dim", 4 * D), ("patch_size", 16),
                 ("tubelet_size", 2), ("img_size", 16 * spec.grid), ("n_frames", 64), ("in_chans", 3)):
        w.add_kv("jepa.enc." + k, v)
    w.add_kv("jepa.enc.ln_eps", 1e-6)
    w.add_kv("jepa.enc.act", "gelu_erf")
    w.add_kv("jepa.enc.pos_type", "rope3d")
    w.add_kv("jepa.enc.rope_theta", 10000.0)
    w.add_kv("jepa.enc.rope_freq_layout", "tiled")
    for k, v in (("kind", "ac"), ("embed_dim", P), ("n_layer", spec.n_layer), ("n_head", spec.n_head),
                 ("ffn_dim", spec.ffn_dim), ("out_dim", D), ("grid_size", spec.grid), ("action_dim", spec.action_dim),
                 ("state_dim", spec.state_dim), ("n_cond_tokens", 2), ("cond_order", "action,state"),
                 ("normalize_reps", True), ("norm_reps_eps", 1e-5), ("frame_causal", True), ("n_frames", spec.n_frames),
                 ("ln_eps", 1e-6), ("act", "gelu_erf"), ("rope_freq_layout", "tiled")):
        w.add_kv("jepa.pred." + k, v)
    # encoder stub: the predictor never runs it
    g.lin("enc.patch_embed", 3 * 2 * 16 * 16, D)
    g.norm("enc.norm", D)
    g.lin("pred.embed", D, P)
    g.lin("pred.action_embed", spec.action_dim, P)
    g.lin("pred.state_embed", spec.state_dim, P)
    for i in range(spec.n_layer):
        q = f"pred.blk.{i}."
        g.norm(q + "ln1", P)
        g.lin(q + "attn_qkv", P, 3 * P)
        g.lin(q + "attn_out", P, P)
        g.norm(q + "ln2", P)
        g.lin(q + "ffn_up", P, spec.ffn_dim)
        g.lin(q + "ffn_down", spec.ffn_dim, P)
    g.norm("pred.norm", P)
    g.lin("pred.proj", P, D)
    w.write(path)


@dc.dataclass
class VideoEncSpec:
    """A video encoder bundle: V-JEPA 2 (tiled 3-D RoPE, tubelet 2), V-JEPA 2.1 (interleaved RoPE, modality
    vectors, a one-frame image tokenizer) or LeVJEPA (CLS token, block-causal attention, tubelet 1)."""
    family: str = "vjepa2"
    dim: int = 128
    n_layer: int = 2
    n_head: int = 2
    ffn_dim: int = 256
    patch: int = 16
    tubelet: int = 2
    ftype: str = "f32"
    w_std: float = 0.05
    rope_layout: str = "tiled"
    rope_theta: float = 10000.0
    rope_interpolate: bool = False
    rope_ref_grid: int = 0
    modality_embed: bool = False
    image_patch_embed: bool = False
    cls_token: bool = False
    block_causal: bool = False
    name: str = "synthetic-video-encoder"


def write_video_encoder(path: str, spec: VideoEncSpec, seed: int = 0) -> None:
    """Write an encoder-only video bundle of the given family (every parameter random)."""
    g = _Gen(HJepaSpec(levels=[], ftype=spec.ftype, rand_all=True, w_std=spec.w_std), seed)
    w = g.w
    D, P = spec.dim, spec.patch
    w.add_kv("general.architecture", "jepa")
    w.add_kv("general.name", spec.name)
    w.add_kv("general.file_type", FTYPE[spec.ftype])
    w.add_kv("jepa.schema_version", 1)
    w.add_kv("jepa.family", spec.family)
    w.add_kv("jepa.modality", "video")
    for k, v in (("embed_dim", D), ("n_layer", spec.n_layer), ("n_head", spec.n_head), ("ffn_dim", spec.ffn_dim),
                 ("patch_size", P), ("tubelet_size", spec.tubelet), ("img_size", 256), ("n_frames", 16), ("in_chans", 3)):
        w.add_kv("jepa.enc." + k, v)
    w.add_kv("jepa.enc.ln_eps", 1e-6)
    w.add_kv("jepa.enc.act", "gelu_erf")
    w.add_kv("jepa.enc.pos_type", "rope3d")
    w.add_kv("jepa.enc.rope_theta", spec.rope_theta)
    w.add_kv("jepa.enc.rope_freq_layout", spec.rope_layout)
    if spec.rope_interpolate:
        w.add_kv("jepa.enc.rope_interpolate", True)
        w.add_kv("jepa.enc.rope_ref_grid", spec.rope_ref_grid)
    w.add_kv("jepa.enc.modality_embed", spec.modality_embed)
    w.add_kv("jepa.enc.image_patch_embed", spec.image_patch_embed)
    w.add_kv("jepa.enc.cls_token", spec.cls_token)
    w.add_kv("jepa.enc.attn_mode", "block_causal" if spec.block_causal else "full")
    g.lin("enc.patch_embed", 3 * spec.tubelet * P * P, D)
    if spec.image_patch_embed:
        g.lin("enc.patch_embed_img", 3 * P * P, D)
    if spec.modality_embed:
        g.tensor("enc.mod_embed_video", g.rng.normal(0.0, 0.5, D).astype(np.float32))
        g.tensor("enc.mod_embed_img", g.rng.normal(0.0, 0.5, D).astype(np.float32))
    if spec.cls_token:
        g.tensor("enc.cls_token", g.rng.normal(0.0, 0.5, D).astype(np.float32))
    for i in range(spec.n_layer):
        q = f"enc.blk.{i}."
        g.norm(q + "ln1", D)
        g.lin(q + "attn_qkv", D, 3 * D)
        g.lin(q + "attn_out", D, D)
        g.norm(q + "ln2", D)
        g.lin(q + "ffn_up", D, spec.ffn_dim)
        g.lin(q + "ffn_down", spec.ffn_dim, D)
    g.norm("enc.norm", D)
    w.write(path)


# ---------------------------------------------------------------------------------------------
# benchmark configurations (the BASELINE configs mapped onto the reference architecture)
# ---------------------------------------------------------------------------------------------
def hjepa_config(idx: int) -> tuple[HJepaSpec, list[dict]]:
    """(model spec, per-level plan settings) of BASELINE config `idx` (1-based: 1, 2, 3, 5).

    The plan settings are jepa_hjepa_level_plan fields; n_steps is fixed (early_stop_patience 0) and
    weight decay is 0 ("Adam"), as the measurement rule asks.
    """
    base = dict(pre_decay_horizon=0, lr=0.1, weight_decay=0.0, var_scale=1.0, action_noise=0.0,
                action_clip_sigma=0.0, min_its=0, early_stop_patience=0, early_stop_rel_delta=1e-2,
                intermediate_cost_weight=1.0, action_cost_weight=0.0, horizon_one_goal_upper=0)
    if idx == 1:
        spec = HJepaSpec(levels=[Level(256, 4, 4, 1024, 2)], ftype="f32", name="cfg1-hjepa-1lvl-f32")
        plans = [dict(base, horizon=8, n_samples=64, n_steps=20, cost_last_n=1, num_subgoals=1)]
    elif idx == 2:
        l1 = Level(384, 6, 6, 1536, 2)
        l2 = Level(384, 6, 6, 1536, 8, stride=4, enc_kind="latent_mlp", enc_hidden=384,
                   act_enc_kind="mlp", act_enc_hidden=64)
        spec = HJepaSpec(levels=[l1, l2], ftype="q8_0", name="cfg2-hjepa-2lvl-q8_0")
        plans = [dict(base, horizon=16, n_samples=256, n_steps=50, cost_last_n=4, num_subgoals=1),
                 dict(base, horizon=4, n_samples=256, n_steps=50, cost_last_n=1, num_subgoals=4)]
    elif idx == 3:
        spec = HJepaSpec(levels=[Level(192, 6, 3, 768, 2)], ftype="f16", enc_layers=12, enc_heads=3,
                         enc_ffn=768, name="cfg3-lewm-f16")
        plans = [dict(base, horizon=5, n_samples=1024, n_steps=30, cost_last_n=1, num_subgoals=1)]
    elif idx == 5:
        mk = lambda a, s, ek, aek: Level(768, 12, 12, 3072, a, stride=s, enc_kind=ek, enc_hidden=768,
                                          act_enc_kind=aek, act_enc_hidden=128)
        spec = HJepaSpec(levels=[mk(2, 1, "vit", "none"), mk(8, 4, "latent_mlp", "mlp"),
                                 mk(8, 2, "latent_mlp", "mlp"), mk(8, 2, "latent_mlp", "mlp")],
                         ftype="q8_0", name="cfg5-hjepa-4lvl-q8_0")
        plans = [dict(base, horizon=64, n_samples=4096, n_steps=100, cost_last_n=16, num_subgoals=1),
                 dict(base, horizon=16, n_samples=4096, n_steps=100, cost_last_n=8, num_subgoals=16),
                 dict(base, horizon=8, n_samples=4096, n_steps=100, cost_last_n=4, num_subgoals=8),
                 dict(base, horizon=4, n_samples=4096, n_steps=100, cost_last_n=1, num_subgoals=4)]
    else:
        raise ValueError(f"no H-JEPA config {idx}")
    return spec, plans


def scaled(spec: HJepaSpec, **kw) -> HJepaSpec:
    s = copy.deepcopy(spec)
    for k, v in kw.items():
        setattr(s, k, v)
    return s
