"""ORACLE ONLY -- test infrastructure, never the product path.

A numpy restatement of the reference's H-JEPA gradient planner (src/hjepa-plan.cpp). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import it, and only as the checker.

Parity pin: the restatement is checked against the reference's own planner source compiled
unmodified against a ggml shim (oracle/Makefile -> oracle/_ref/libhjepa_ref.so) and against the golden
vectors that library produced (tests/golden/, written by tests/golden/make_golden.py).

Arithmetic follows the reference: float32 values, LayerNorm statistics and the cost reduction in
float64, the same expression order in the element-wise ops. The matrix products are numpy/BLAS
float32 and therefore differ from the reference's row-by-row axpy in the last bits only.
Weights are dequantised with the `gguf` package (gguf-py 0.19.0, an implementation independent of
both this project and the reference) from the file's own bytes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

f32 = np.float32


# ---------------------------------------------------------------------------------------------
# weights (src/hjepa-plan.cpp:48-206)
# ---------------------------------------------------------------------------------------------
def load_tensors(path: str) -> tuple[dict, dict]:
    """name -> float32 array in PyTorch row-major shape, plus the metadata fields as python values."""
    import gguf
    r = gguf.GGUFReader(path)
    out = {}
    for t in r.tensors:
        shape = tuple(int(x) for x in reversed([int(v) for v in t.shape]))
        data = gguf.quants.dequantize(t.data, t.tensor_type)
        out[t.name] = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(shape))
    meta = {}
    for k, fld in r.fields.items():
        try:
            meta[k] = fld.contents()
        except Exception:
            pass
    return out, meta


@dataclass
class Lin:
    w: np.ndarray            # [out, in]
    b: Optional[np.ndarray]  # [out] or None

    def __call__(self, x):
        y = x @ self.w.T
        if self.b is not None:
            y = y + self.b
        return y.astype(f32)

    def back(self, gy):
        return (gy @ self.w).astype(f32)


@dataclass
class LevelW:
    hp: dict
    pos0: np.ndarray
    act0: Optional[Lin] = None
    act2: Optional[Lin] = None
    pact0: Optional[Lin] = None
    pact2: Optional[Lin] = None
    in_proj: Optional[Lin] = None
    cond_proj: Optional[Lin] = None
    out_proj: Optional[Lin] = None
    proj0: Optional[Lin] = None
    proj2: Optional[Lin] = None
    norm_w: Optional[np.ndarray] = None
    norm_b: Optional[np.ndarray] = None
    blocks: list = field(default_factory=list)
    enc_in_w: Optional[np.ndarray] = None
    enc_in_b: Optional[np.ndarray] = None
    enc_out_w: Optional[np.ndarray] = None
    enc_out_b: Optional[np.ndarray] = None
    enc_fc1: Optional[Lin] = None
    enc_fc2: Optional[Lin] = None
    ae_fc1: Optional[Lin] = None
    ae_fc2: Optional[Lin] = None
    ae_out_w: Optional[np.ndarray] = None
    ae_out_b: Optional[np.ndarray] = None
    ae_step: Optional[Lin] = None             # 'seq' action encoder (hjepa-plan.cpp:183-200)
    ae_pos: Optional[np.ndarray] = None
    ae_blocks: list = field(default_factory=list)
    ae_head0: Optional[Lin] = None
    ae_head2: Optional[Lin] = None
    ae_headln_w: Optional[np.ndarray] = None
    ae_headln_b: Optional[np.ndarray] = None
    queue: Optional[np.ndarray] = None
    pos_all: Optional[np.ndarray] = None        # every row of pred.pos_embed (the multi-frame predictor)


class Model:
    """The planner's f32 view of an H-JEPA file (build_plan_model, src/hjepa-plan.cpp:143-206)."""

    def __init__(self, path: str):
        T, meta = load_tensors(path)
        self.T = T
        g = lambda k, d=None: meta.get("jepa.hjepa." + k, d)
        self.ln_eps = float(g("ln_eps", 1e-5))
        self.adaln_eps = float(g("adaln_eps", 1e-6))
        n = int(g("n_levels"))
        keys = ["embed_dim", "stride", "action_dim", "act_embed_dim", "pred_dim", "pred_n_layer", "pred_n_head",
                "pred_head_dim", "pred_ffn_dim", "pred_n_frames"]
        # the level-1 projector of the encoder's CLS row and the proprio stream (jepa_hjepa_embed)
        self.proj_kind = str(g("proj_kind", "identity"))
        self.proj0, self.proj2 = self.lin("lvl.1.enc.proj.0"), self.lin("lvl.1.enc.proj.2")
        self.proj_ln = (T.get("lvl.1.enc.proj_ln.weight"), T.get("lvl.1.enc.proj_ln.bias"))
        self.pro0, self.pro2 = self.lin("lvl.1.enc.proprio.0"), self.lin("lvl.1.enc.proprio.2")
        self.pro_ln = (T.get("lvl.1.enc.proprio.ln.weight"), T.get("lvl.1.enc.proprio.ln.bias"))
        self.levels = []
        for li in range(n):
            hp = {k: int(g(k)[li]) for k in keys}
            for k in ("enc_kind", "act_enc_kind", "pred_kind"):
                hp[k] = str(g(k)[li])
            p = f"lvl.{li + 1}."
            inner = hp["pred_n_head"] * hp["pred_head_dim"]
            L = LevelW(hp=hp, pos0=T[p + "pred.pos_embed"][0].copy())
            L.pos_all = T[p + "pred.pos_embed"].copy()
            L.act0, L.act2 = self.lin(p + "act_embed.0"), self.lin(p + "act_embed.2")
            L.pact0, L.pact2 = self.lin(p + "pred.act_embed.0"), self.lin(p + "pred.act_embed.2")
            L.in_proj, L.cond_proj = self.lin(p + "pred.in_proj"), self.lin(p + "pred.cond_proj")
            L.out_proj = self.lin(p + "pred.out_proj")
            L.proj0, L.proj2 = self.lin(p + "pred.proj.0"), self.lin(p + "pred.proj.2")
            L.norm_w, L.norm_b = T.get(p + "pred.norm.weight"), T.get(p + "pred.norm.bias")
            for i in range(hp["pred_n_layer"]):
                q = p + f"pred.blk.{i}."
                L.blocks.append(dict(
                    adaln=self.lin(q + "adaln"),
                    v=self.lin(q + "attn_qkv", 2 * inner, inner),      # the value third (hjepa-plan.cpp:170-171)
                    qk=self.lin(q + "attn_qkv", 0, 2 * inner),        # query / key rows (the multi-frame predictor)
                    out=self.lin(q + "attn_out"), up=self.lin(q + "ffn_up"), down=self.lin(q + "ffn_down"),
                    ln1_w=T.get(q + "ln1.weight"), ln1_b=T.get(q + "ln1.bias"),
                    ln2_w=T.get(q + "ln2.weight"), ln2_b=T.get(q + "ln2.bias")))
            L.enc_in_w, L.enc_in_b = T.get(p + "enc.in_norm.weight"), T.get(p + "enc.in_norm.bias")
            L.enc_out_w, L.enc_out_b = T.get(p + "enc.out_norm.weight"), T.get(p + "enc.out_norm.bias")
            L.enc_fc1, L.enc_fc2 = self.lin(p + "enc.fc1"), self.lin(p + "enc.fc2")
            L.ae_fc1, L.ae_fc2 = self.lin(p + "act_enc.fc1"), self.lin(p + "act_enc.fc2")
            L.ae_out_w, L.ae_out_b = T.get(p + "act_enc.out_norm.weight"), T.get(p + "act_enc.out_norm.bias")
            L.ae_step, L.ae_pos = self.lin(p + "act_enc.step"), T.get(p + "act_enc.pos")
            L.ae_head0, L.ae_head2 = self.lin(p + "act_enc.head.0"), self.lin(p + "act_enc.head.2")
            L.ae_headln_w, L.ae_headln_b = T.get(p + "act_enc.head.ln.weight"), T.get(p + "act_enc.head.ln.bias")
            i = 0
            while T.get(p + f"act_enc.blk.{i}.attn_qkv.weight") is not None:
                q = p + f"act_enc.blk.{i}."
                L.ae_blocks.append(dict(qkv=self.lin(q + "attn_qkv"), out=self.lin(q + "attn_out"), up=self.lin(q + "ffn_up"),
                                        down=self.lin(q + "ffn_down"), ln1_w=T.get(q + "ln1.weight"), ln1_b=T.get(q + "ln1.bias"),
                                        ln2_w=T.get(q + "ln2.weight"), ln2_b=T.get(q + "ln2.bias")))
                i += 1
            hp["act_enc_n_head"] = int(g("act_enc_n_head", [0] * n)[li]) if g("act_enc_n_head") is not None else 0
            L.queue = T.get(p + "act_queue")
            self.levels.append(L)

    def lin(self, name, row0=0, rows=None) -> Optional[Lin]:
        w = self.T.get(name + ".weight")
        if w is None:
            return None
        b = self.T.get(name + ".bias")
        rows = w.shape[0] - row0 if rows is None else rows
        return Lin(np.ascontiguousarray(w[row0:row0 + rows]), None if b is None else b[row0:row0 + rows].copy())


# ---------------------------------------------------------------------------------------------
# element-wise ops with their gradients (src/hjepa-plan.cpp:290-475)
# ---------------------------------------------------------------------------------------------
def ln_fwd(x, w, b, eps):
    """Two-pass mean / variance in float64, inverse std rounded to float32 (hjepa-plan.cpp:299-315)."""
    xd = x.astype(np.float64)
    mean = xd.mean(axis=1, keepdims=True)
    var = ((xd - mean) ** 2).mean(axis=1, keepdims=True)
    inv = (1.0 / np.sqrt(var + float(f32(eps)))).astype(f32)
    xhat = (xd - mean).astype(f32) * inv
    y = xhat
    if w is not None:
        y = xhat * w
    if b is not None:
        y = y + b
    return y.astype(f32), (xhat, inv)


def ln_bwd(gy, cache, w):
    xhat, inv = cache
    gh = gy * w if w is not None else gy
    gh = gh.astype(f32)
    m1 = gh.astype(np.float64).mean(axis=1, keepdims=True)
    m2 = (gh.astype(np.float64) * xhat.astype(np.float64)).mean(axis=1, keepdims=True)
    return ((gh.astype(np.float64) - m1 - xhat.astype(np.float64) * m2) * inv.astype(np.float64)).astype(f32)


def _erf(x):
    return np.vectorize(math.erf, otypes=[np.float64])(x)


def act_fwd(x, kind):
    if kind == "silu":
        return (x / (f32(1) + np.exp(-x))).astype(f32)
    if kind == "relu":
        return np.where(x > 0, x, f32(0)).astype(f32)
    return (f32(0.5) * x * (f32(1) + _erf(x * f32(0.70710678118654752)).astype(f32))).astype(f32)


def act_bwd(gy, x, kind):
    if kind == "silu":
        s = (f32(1) / (f32(1) + np.exp(-x))).astype(f32)
        dv = s * (f32(1) + x * (f32(1) - s))
    elif kind == "relu":
        dv = (x > 0).astype(f32)
    else:
        dv = f32(0.5) * (f32(1) + _erf(x * f32(0.70710678118654752)).astype(f32)) + \
            x * f32(0.39894228040143268) * np.exp(f32(-0.5) * x * x)
    return (gy * dv.astype(f32)).astype(f32)


# ---------------------------------------------------------------------------------------------
# one predictor step with a context of one state (build_step, hjepa-plan.cpp:630-651)
# ---------------------------------------------------------------------------------------------
class StepTape:
    """Forward values kept for the backward pass of one step."""


def step_fwd(m: Model, L: LevelW, s, e):
    t = StepTape()
    c = e
    if L.pact0 is not None:
        t.pact_u = L.pact0(c)
        c = L.pact2(act_fwd(t.pact_u, "silu"))
    x = (s + L.pos0).astype(f32)
    if L.in_proj is not None:
        x = L.in_proj(x)
    if L.cond_proj is not None:
        c = L.cond_proj(c)
    t.c = c
    cs = act_fwd(c, "silu")
    D = x.shape[1]
    t.blocks = []
    for B in L.blocks:
        bt = {}
        mod = B["adaln"](cs)
        bt["mod"] = mod
        bt["x0"] = x
        z, bt["ln0a"] = ln_fwd(x, None, None, m.adaln_eps)
        h = (z * (f32(1) + mod[:, D:2 * D]) + mod[:, 0:D]).astype(f32)
        bt["za"] = z
        if B["ln1_w"] is not None:
            bt["fa"] = h
            h, bt["ln1"] = ln_fwd(h, B["ln1_w"], B["ln1_b"], m.ln_eps)
        o = B["out"](B["v"](h))
        bt["o"] = o
        x = (x + o * mod[:, 2 * D:3 * D]).astype(f32)
        bt["x1"] = x
        z, bt["ln0m"] = ln_fwd(x, None, None, m.adaln_eps)
        bt["zm"] = z
        h = (z * (f32(1) + mod[:, 4 * D:5 * D]) + mod[:, 3 * D:4 * D]).astype(f32)
        if B["ln2_w"] is not None:
            h, bt["ln2"] = ln_fwd(h, B["ln2_w"], B["ln2_b"], m.ln_eps)
        u = B["up"](h)
        bt["u"] = u
        dn = B["down"](act_fwd(u, "gelu"))
        bt["dn"] = dn
        x = (x + dn * mod[:, 5 * D:6 * D]).astype(f32)
        t.blocks.append(bt)
    x, t.norm = ln_fwd(x, L.norm_w, L.norm_b, m.ln_eps)
    if L.out_proj is not None:
        x = L.out_proj(x)
    if L.proj0 is not None:
        t.proj_u = L.proj0(x)
        x = L.proj2(act_fwd(t.proj_u, "gelu"))
    return x, t


def step_bwd(m: Model, L: LevelW, t: StepTape, gx):
    """Gradient of one step: d next -> (d s, d e)."""
    if L.proj0 is not None:
        gx = L.proj0.back(act_bwd(L.proj2.back(gx), t.proj_u, "gelu"))
    if L.out_proj is not None:
        gx = L.out_proj.back(gx)
    gx = ln_bwd(gx, t.norm, L.norm_w)
    D = gx.shape[1]
    gcs = None
    for B, bt in reversed(list(zip(L.blocks, t.blocks))):
        mod = bt["mod"]
        gm = np.zeros_like(mod)
        # x2 = x1 + dn * gate_m
        gm[:, 5 * D:6 * D] = gx * bt["dn"]
        gdn = (gx * mod[:, 5 * D:6 * D]).astype(f32)
        gh = B["up"].back(act_bwd(B["down"].back(gdn), bt["u"], "gelu"))
        if B["ln2_w"] is not None:
            gh = ln_bwd(gh, bt["ln2"], B["ln2_w"])
        gm[:, 4 * D:5 * D] = gh * bt["zm"]
        gm[:, 3 * D:4 * D] = gh
        gz = (gh * (f32(1) + mod[:, 4 * D:5 * D])).astype(f32)
        gx = (gx + ln_bwd(gz, bt["ln0m"], None)).astype(f32)
        # x1 = x0 + o * gate_a
        gm[:, 2 * D:3 * D] = gx * bt["o"]
        go = (gx * mod[:, 2 * D:3 * D]).astype(f32)
        gh = B["v"].back(B["out"].back(go))
        if B["ln1_w"] is not None:
            gh = ln_bwd(gh, bt["ln1"], B["ln1_w"])
        gm[:, D:2 * D] = gh * bt["za"]
        gm[:, 0:D] = gh
        gz = (gh * (f32(1) + mod[:, D:2 * D])).astype(f32)
        gx = (gx + ln_bwd(gz, bt["ln0a"], None)).astype(f32)
        g = B["adaln"].back(gm.astype(f32))
        gcs = g if gcs is None else (gcs + g).astype(f32)
    gc = act_bwd(gcs, t.c, "silu")
    if L.cond_proj is not None:
        gc = L.cond_proj.back(gc)
    if L.in_proj is not None:
        gx = L.in_proj.back(gx)
    ge = gc
    if L.pact0 is not None:
        ge = L.pact0.back(act_bwd(L.pact2.back(gc), t.pact_u, "silu"))
    return gx, ge


def act_embed_fwd(L: LevelW, a):
    if L.act0 is None:
        return a, None
    u = L.act0(a)
    return L.act2(act_fwd(u, "silu")), u


def act_embed_bwd(L: LevelW, u, ge):
    if L.act0 is None:
        return ge
    return L.act0.back(act_bwd(L.act2.back(ge), u, "silu"))


def encode_up_fwd(m: Model, up: LevelW, s):
    """build_encode_up (hjepa-plan.cpp:654-660)."""
    if up.hp["enc_kind"] == "identity":
        return s, None
    x, c1 = ln_fwd(s, up.enc_in_w, up.enc_in_b, m.ln_eps)
    u = up.enc_fc1(x)
    x = up.enc_fc2(act_fwd(u, "gelu"))
    c2 = None
    if up.enc_out_w is not None:
        x, c2 = ln_fwd(x, up.enc_out_w, up.enc_out_b, m.ln_eps)
    return x, (c1, u, c2)


def encode_up_bwd(up: LevelW, cache, gx):
    if cache is None:
        return gx
    c1, u, c2 = cache
    if c2 is not None:
        gx = ln_bwd(gx, c2, up.enc_out_w)
    gx = up.enc_fc1.back(act_bwd(up.enc_fc2.back(gx), u, "gelu"))
    return ln_bwd(gx, c1, up.enc_in_w)


# ---------------------------------------------------------------------------------------------
# cost of candidates (chunk_cost, hjepa-plan.cpp:689-810)
# ---------------------------------------------------------------------------------------------
@dataclass
class CostSpec:
    level: int = 1
    horizon: int = 1
    s0: np.ndarray = None
    goal: np.ndarray = None          # [n_goal, D_goal]
    n_goal: int = 1
    goal_level: int = 1
    dense: bool = False
    goal_action: Optional[np.ndarray] = None
    cost_last_n: int = 1
    intermediate_cost_weight: float = 1.0
    action_cost_weight: float = 0.0


def scored_states(m: Model, cs: CostSpec) -> int:
    n = cs.horizon + 1
    for lv in range(cs.level + 1, cs.goal_level + 1):
        stride = 1 if cs.dense else m.levels[lv - 1].hp["stride"]
        n = (n - 1) // stride + 1
    return n - 1


def batch_cost(m: Model, cs: CostSpec, actions, want_grad=True, want_states=False):
    """costs [n], grad [n, T, A] (or None), states [n, T+1, D] (or None) of candidates `actions`."""
    L = m.levels[cs.level - 1]
    n, T, A = actions.shape
    D = L.hp["embed_dim"]
    s = np.broadcast_to(cs.s0.astype(f32), (n, D)).copy()
    preds = [s]
    tapes, emb_u = [], []
    embs = []
    for step in range(T):
        e, u = act_embed_fwd(L, np.ascontiguousarray(actions[:, step, :]).astype(f32))
        emb_u.append(u)
        embs.append(e)
        s, tp = step_fwd(m, L, s, e)
        tapes.append(tp)
        preds.append(s)
    # encode the predicted stream up to the goal's level
    idx = list(range(T + 1))
    vals = list(preds)
    enc_caches = []           # per level above: (kept indices into the previous list, caches)
    for lv in range(cs.level + 1, cs.goal_level + 1):
        up = m.levels[lv - 1]
        stride = 1 if cs.dense else up.hp["stride"]
        keep = list(range(0, len(vals), stride))
        new_vals, caches = [], []
        for k in keep:
            v, c = encode_up_fwd(m, up, vals[k])
            new_vals.append(v)
            caches.append(c)
        enc_caches.append((up, keep, caches))
        vals = new_vals
    scored = vals[1:]
    W = min(max(1, cs.cost_last_n), len(scored))
    costs = np.zeros(n, np.float32)
    gscored = [None] * len(scored)
    for j in range(W):
        k = len(scored) - W + j
        g = cs.goal[0 if cs.n_goal == 1 else j].astype(f32)
        w = f32(cs.intermediate_cost_weight) if (cs.intermediate_cost_weight != 1.0 and W > 1 and j < W - 1) else f32(1)
        diff = (scored[k] - g).astype(f32)
        acc = (diff.astype(np.float64) ** 2).sum(axis=1)
        costs = (costs + w * acc.astype(f32)).astype(f32)
        if want_grad:
            gscored[k] = (f32(2) * w * diff).astype(f32)
    gemb = [None] * T          # extra gradient of each step's action embedding (the action cost)
    if cs.action_cost_weight != 0.0 and cs.goal_action is not None and cs.goal_level == cs.level + 1 and not cs.dense:
        # the candidates pooled into the upper level's macro-actions against the ones it chose (chunk_cost,
        # hjepa-plan.cpp:769-791): whole chunks only, the last Wa of them
        up = m.levels[cs.level]
        stride = up.hp["stride"]
        n_pooled = T // stride
        Wa = min(max(1, cs.cost_last_n), n_pooled, cs.n_goal)
        w = f32(cs.action_cost_weight)
        for j in range(Wa):
            chunk = n_pooled - Wa + j
            steps = list(range(chunk * stride, (chunk + 1) * stride))
            y, cache = action_pool_fwd(m, up, [embs[s] for s in steps])
            g = cs.goal_action[cs.n_goal - Wa + j].astype(f32)
            diff = (y - g).astype(f32)
            acc = (diff.astype(np.float64) ** 2).sum(axis=1)
            costs = (costs + w * acc.astype(f32)).astype(f32)
            if want_grad:
                for s_, ge in zip(steps, action_pool_bwd(up, cache, (f32(2) * w * diff).astype(f32))):
                    gemb[s_] = ge if gemb[s_] is None else (gemb[s_] + ge).astype(f32)
    grad = None
    if want_grad:
        # back through the encoders, top level first
        gvals = [None] + gscored
        for up, keep, caches in reversed(enc_caches):
            prev = [None] * (max(keep) + 1 if keep else 0)
            for k, c, gv in zip(keep, caches, gvals):
                if gv is not None:
                    prev[k] = encode_up_bwd(up, c, gv)
            gvals = prev
        gpred = [None] * (T + 1)
        for k, gv in enumerate(gvals):
            if k <= T:
                gpred[k] = gv
        grad = np.zeros_like(actions, dtype=f32)
        gs = gpred[T] if gpred[T] is not None else np.zeros((n, D), f32)
        for step in reversed(range(T)):
            gs_prev, ge = step_bwd(m, L, tapes[step], gs)
            if gemb[step] is not None:
                ge = (ge + gemb[step]).astype(f32)
            grad[:, step, :] = act_embed_bwd(L, emb_u[step], ge)
            gs = gs_prev
            if gpred[step] is not None:
                gs = (gs + gpred[step]).astype(f32)
    states = np.stack(preds, axis=1) if want_states else None
    return costs, grad, states


# ---------------------------------------------------------------------------------------------
# the upper level's action encoder over one chunk of the level's action embeddings
# (build_action_pool, hjepa-plan.cpp:663-684; op_tokens / op_mha / op_first_of_group :478-619)
# ---------------------------------------------------------------------------------------------
def mha_fwd(qkv, G, n_head):
    """Self-attention inside each group of G rows; qkv [rows][3 d] = [q | k | v] (op_mha, :553-583)."""
    rows, d3 = qkv.shape
    d = d3 // 3
    hd = d // n_head
    n = rows // G
    q = qkv[:, :d].reshape(n, G, n_head, hd).transpose(0, 2, 1, 3)
    k = qkv[:, d:2 * d].reshape(n, G, n_head, hd).transpose(0, 2, 1, 3)
    v = qkv[:, 2 * d:].reshape(n, G, n_head, hd).transpose(0, 2, 1, 3)
    scale = f32(1.0) / f32(math.sqrt(hd))
    s = (np.einsum("nhic,nhjc->nhij", q, k).astype(f32) * scale).astype(f32)
    e = np.exp((s - s.max(-1, keepdims=True)).astype(f32)).astype(f32)
    p = (e / e.sum(-1, keepdims=True, dtype=f32)).astype(f32)
    o = np.einsum("nhij,nhjc->nhic", p, v).astype(f32)
    return o.transpose(0, 2, 1, 3).reshape(rows, d).astype(f32), (q, k, v, p, scale)


def mha_bwd(go, cache, G, n_head):
    """op_mha's backward (:584-617): gv = p go, gs = p (go.v - sum p go.v) scale, gq = gs k, gk = gs q."""
    q, k, v, p, scale = cache
    n, H, _, hd = q.shape
    gon = go.reshape(n, G, H, hd).transpose(0, 2, 1, 3)
    gp = np.einsum("nhic,nhjc->nhij", gon, v).astype(f32)
    gv = np.einsum("nhij,nhic->nhjc", p, gon).astype(f32)
    dotp = (gp * p).sum(-1, keepdims=True, dtype=f32)
    gs = (p * (gp - dotp) * scale).astype(f32)
    gq = np.einsum("nhij,nhjc->nhic", gs, k).astype(f32)
    gk = np.einsum("nhij,nhic->nhjc", gs, q).astype(f32)
    back = lambda x: x.transpose(0, 2, 1, 3).reshape(n * G, H * hd)
    return np.concatenate([back(gq), back(gk), back(gv)], axis=1).astype(f32)


def action_pool_fwd(m: Model, up: LevelW, chunk):
    """chunk: the level's action embeddings of `stride` consecutive steps, each [n][E] -> [n][A_up]."""
    n = chunk[0].shape[0]
    if up.hp["act_enc_kind"] == "mlp":
        x = np.concatenate(chunk, axis=1).astype(f32)
        h = up.ae_fc1(x)
        r = act_fwd(h, "relu")
        y = up.ae_fc2(r)
        c_out = None
        if up.ae_out_w is not None:
            y, c_out = ln_fwd(y, up.ae_out_w, up.ae_out_b, m.ln_eps)
        return y, ("mlp", h, c_out)
    steps = [up.ae_step(e) for e in chunk]
    L, d = len(steps), steps[0].shape[1]
    G = L + 1
    x = np.zeros((n, G, d), f32)
    x[:, 0, :] = up.ae_pos[0]
    for l in range(L):
        x[:, l + 1, :] = (steps[l] + up.ae_pos[l + 1]).astype(f32)
    x = x.reshape(n * G, d)
    bc = []
    for B in up.ae_blocks:
        h, c1 = ln_fwd(x, B["ln1_w"], B["ln1_b"], m.ln_eps)
        qkv = B["qkv"](h)
        o, cm = mha_fwd(qkv, G, up.hp["act_enc_n_head"])
        x = (x + B["out"](o)).astype(f32)
        h2, c2 = ln_fwd(x, B["ln2_w"], B["ln2_b"], m.ln_eps)
        u = B["up"](h2)
        x = (x + B["down"](act_fwd(u, "relu"))).astype(f32)
        bc.append((c1, cm, c2, u))
    y0 = x.reshape(n, G, d)[:, 0, :].copy()
    z = up.ae_head0(y0)
    zg = act_fwd(z, "gelu")
    zl, ch = ln_fwd(zg, up.ae_headln_w, up.ae_headln_b, m.ln_eps)
    y2 = up.ae_head2(zl)
    y, co = ln_fwd(y2, up.ae_out_w, up.ae_out_b, 1e-6)
    return y, ("seq", G, d, bc, z, ch, co)


def action_pool_bwd(up: LevelW, cache, gy):
    """Gradient of the pooled action with respect to each embedding of the chunk: list of [n][E]."""
    if cache[0] == "mlp":
        _, h, c_out = cache
        if c_out is not None:
            gy = ln_bwd(gy, c_out, up.ae_out_w)
        gx = up.ae_fc1.back(act_bwd(up.ae_fc2.back(gy), h, "relu"))
        E = gx.shape[1] // up.hp["stride"]
        return [np.ascontiguousarray(gx[:, i * E:(i + 1) * E]) for i in range(up.hp["stride"])]
    _, G, d, bc, z, ch, co = cache
    g = ln_bwd(gy, co, up.ae_out_w)
    g = up.ae_head2.back(g)
    g = ln_bwd(g, ch, up.ae_headln_w)
    g = up.ae_head0.back(act_bwd(g, z, "gelu"))
    n = g.shape[0]
    gx = np.zeros((n, G, d), f32)
    gx[:, 0, :] = g
    gx = gx.reshape(n * G, d)
    for B, (c1, cm, c2, u) in zip(reversed(up.ae_blocks), reversed(bc)):
        gu = act_bwd(B["down"].back(gx), u, "relu")
        gx = (gx + ln_bwd(B["up"].back(gu), c2, B["ln2_w"])).astype(f32)
        gq = mha_bwd(B["out"].back(gx), cm, G, up.hp["act_enc_n_head"])
        gx = (gx + ln_bwd(B["qkv"].back(gq), c1, B["ln1_w"])).astype(f32)
    gx = gx.reshape(n, G, d)
    return [up.ae_step.back(np.ascontiguousarray(gx[:, l + 1, :])) for l in range(G - 1)]


# ---------------------------------------------------------------------------------------------
# one level's solve (solve_level, hjepa-plan.cpp:904-959)
# ---------------------------------------------------------------------------------------------
def prior_of(L: LevelW, clip_sigma: float):
    A = L.hp["action_dim"]
    q = L.queue
    mean = np.zeros(A, f32)
    std = np.ones(A, f32)
    lo = hi = None
    if q is not None and q.size:
        qd = q.astype(np.float64)
        mu = qd.mean(axis=0)
        var = ((qd - mu) ** 2).sum(axis=0) / qd.shape[0]
        mean = mu.astype(f32)
        std = np.maximum(np.sqrt(var).astype(f32), f32(1e-4))
    if clip_sigma > 0:
        lo = (mean - f32(clip_sigma) * std).astype(f32)
        hi = (mean + f32(clip_sigma) * std).astype(f32)
    elif q is not None and q.size:
        n = q.shape[0]
        lo, hi = np.zeros(A, f32), np.zeros(A, f32)
        for a in range(A):
            col = np.sort(q[:, a].astype(f32))

            def quant(p):
                pos = p * (n - 1)
                i0 = int(math.floor(pos))
                i1 = min(i0 + 1, n - 1)
                fr = pos - i0
                return f32(float(col[i0]) + (float(col[i1]) - float(col[i0])) * fr)
            lo[a], hi[a] = quant(0.02), quant(0.98)
    return mean, std, lo, hi


def solve_level(m: Model, cs: CostSpec, lp: dict, noise):
    """`noise(n)` returns n standard-normal draws (the jepa_randn_fn). Returns actions, states, cost, iters."""
    L = m.levels[cs.level - 1]
    A, T, S = L.hp["action_dim"], cs.horizon, max(1, lp["n_samples"])
    mean, std, lo, hi = prior_of(L, lp["action_clip_sigma"])
    x = np.broadcast_to(mean, (S, T, A)).astype(f32).copy()
    if S > 1:
        z = noise((S - 1) * T * A).reshape(S - 1, T, A).astype(f32)
        x[1:] = (x[1:] + z * std * f32(lp["var_scale"])).astype(f32)
    b1, b2, eps = f32(0.9), f32(0.999), f32(1e-8)
    mm = np.zeros_like(x)
    vv = np.zeros_like(x)
    best, stalled, iters = math.inf, 0, 0
    lr, wd = f32(lp["lr"]), f32(lp["weight_decay"])
    for step in range(lp["n_steps"]):
        costs, g, _ = batch_cost(m, cs, x, want_grad=True)
        c1 = f32(1) - np.power(b1, f32(step + 1), dtype=f32)
        c2 = f32(1) - np.power(b2, f32(step + 1), dtype=f32)
        step_size = f32(lr / c1)
        c2s = np.sqrt(c2, dtype=f32)
        x = (x * (f32(1) - lr * wd)).astype(f32)
        mm = (b1 * mm + (f32(1) - b1) * g).astype(f32)
        vv = (b2 * vv + (f32(1) - b2) * g * g).astype(f32)
        x = (x - step_size * mm / (np.sqrt(vv) / c2s + eps)).astype(f32)
        if lp["action_noise"] > 0:
            z = noise(S * T * A).reshape(S, T, A).astype(f32)
            x = (x + z * f32(lp["action_noise"])).astype(f32)
        if lo is not None:
            x = np.minimum(np.maximum(x, lo), hi).astype(f32)
        iters = step + 1
        if lp["early_stop_patience"] > 0:
            score = float(costs.min())
            improved = (not math.isfinite(best)) or (best - score > lp["early_stop_rel_delta"] * max(abs(best), 1e-12))
            if improved:
                best, stalled = score, 0
            else:
                stalled += 1
                if stalled >= lp["early_stop_patience"] and step + 1 >= lp["min_its"]:
                    break
    costs, _, states = batch_cost(m, cs, x, want_grad=False, want_states=True)
    top = int(np.argmin(costs))
    return x[top].copy(), states[top].copy(), float(costs[top]), iters


def plan(m: Model, states, goals, levels: list, noise_for_level):
    """jepa_hjepa_plan (hjepa-plan.cpp:1165-1256): the levels top-down. `noise_for_level(lv)` gives
    that level's jepa_randn_fn. Returns (level-1 actions, info dict)."""
    n_levels = len(m.levels)
    info = {"planned": [0] * n_levels, "cost": [0.0] * n_levels, "iters": [0] * n_levels, "goal_level": [0] * n_levels}
    upper = None
    skipped_goal_level = 0
    upper_anchored = True
    for lv in range(n_levels, 0, -1):
        lp = levels[lv - 1]
        if lv > 1 and lp["horizon"] == 1:
            skipped_goal_level = (skipped_goal_level or lv) if lp["horizon_one_goal_upper"] else 0
            upper = None
            continue
        cs = CostSpec(level=lv, horizon=lp["horizon"], s0=states[lv - 1], cost_last_n=lp["cost_last_n"],
                      intermediate_cost_weight=lp["intermediate_cost_weight"],
                      action_cost_weight=lp["action_cost_weight"])
        if upper is None:
            cs.goal_level = skipped_goal_level or lv
            cs.goal = np.asarray(goals[cs.goal_level - 1], f32).reshape(1, -1)
            cs.n_goal = 1
            cs.dense = cs.goal_level > lv
            anchored = True
        else:
            up = m.levels[lv]
            u_act, u_states = upper
            n_up = u_states.shape[0]
            n_sub = min(levels[lv]["num_subgoals"], n_up - 1)
            gb = u_states[1:1 + n_sub].copy()
            anchored = False
            if 1 + levels[lv]["num_subgoals"] >= n_up and upper_anchored:
                gb[n_sub - 1] = goals[lv]
                anchored = True
            cs.goal_level, cs.goal, cs.n_goal = lv + 1, gb, n_sub
            cs.goal_action = u_act[:n_sub].copy()
            if n_sub > 1:
                expected = (lp["horizon"] + up.hp["stride"]) // up.hp["stride"] - 1
                if n_sub != expected:
                    raise ValueError("subgoal count does not match the horizon")
        a, st, c, it = solve_level(m, cs, lp, noise_for_level(lv))
        upper = (a, st)
        info["planned"][lv - 1], info["cost"][lv - 1], info["iters"][lv - 1] = 1, c, it
        info["goal_level"][lv - 1] = cs.goal_level
        upper_anchored = anchored
        skipped_goal_level = 0
    return upper[0], info


def replay(draws):
    """A noise source over recorded draws (the jepa_randn_fn of the reference's tests)."""
    buf = np.asarray(draws, f32).ravel()
    pos = [0]

    def fn(n):
        out = np.zeros(n, f32)
        k = min(n, buf.size - pos[0])
        out[:k] = buf[pos[0]:pos[0] + k]
        pos[0] += k
        return out
    return fn


# ---------------------------------------------------------------------------------------------
# the multi-frame predictor: jepa_hjepa_predict / jepa_hjepa_rollout (src/hjepa.cpp:566-667) over the
# adaLN-zero transformer jepa_build_adaln (src/lewm.cpp:33-95): causal softmax attention across frames
# ---------------------------------------------------------------------------------------------
def causal_attention(q, k, v, n_head):
    """Per head softmax(q k^T / sqrt(hd)) v with keys 0..t for query t (jepa_causal_mask_f16, src/lewm.cpp:97-103)."""
    T_, inner = q.shape
    hd = inner // n_head
    split = lambda x: x.reshape(T_, n_head, hd).transpose(1, 0, 2)
    qh, kh, vh = split(q), split(k), split(v)
    s = (qh @ kh.transpose(0, 2, 1)).astype(f32) * f32(1.0 / math.sqrt(hd))
    s = np.where(np.triu(np.ones((T_, T_), bool), 1)[None], -np.inf, s).astype(f32)
    e = np.exp((s - s.max(-1, keepdims=True)).astype(f32)).astype(f32)
    p = (e / e.sum(-1, keepdims=True, dtype=f32)).astype(f32)
    return (p @ vh).astype(f32).transpose(1, 0, 2).reshape(T_, inner)


def predict(m: Model, level: int, states, actions):
    """states [T][D], actions [T][A] -> [T][D_out]; row t is the state predicted after frames 0..t."""
    L = m.levels[level - 1]
    T_ = states.shape[0]
    D = L.hp["pred_dim"] or L.hp["embed_dim"]
    c, _ = act_embed_fwd(L, np.asarray(actions, f32))
    if L.pact0 is not None:
        c = L.pact2(act_fwd(L.pact0(c), "silu"))
    x = (np.asarray(states, f32) + L.pos_all[:T_]).astype(f32)
    if L.in_proj is not None:
        x = L.in_proj(x)
    if L.cond_proj is not None:
        c = L.cond_proj(c)
    cs = act_fwd(c, "silu")
    P = x.shape[1]
    for B in L.blocks:
        mod = B["adaln"](cs)
        z, _ = ln_fwd(x, None, None, m.adaln_eps)
        h = (z * (f32(1) + mod[:, P:2 * P]) + mod[:, 0:P]).astype(f32)
        if B["ln1_w"] is not None:
            h, _ = ln_fwd(h, B["ln1_w"], B["ln1_b"], m.ln_eps)
        qk = B["qk"](h)
        inner = qk.shape[1] // 2
        o = causal_attention(qk[:, :inner], qk[:, inner:], B["v"](h), L.hp["pred_n_head"])
        x = (x + B["out"](o) * mod[:, 2 * P:3 * P]).astype(f32)
        z, _ = ln_fwd(x, None, None, m.adaln_eps)
        h = (z * (f32(1) + mod[:, 4 * P:5 * P]) + mod[:, 3 * P:4 * P]).astype(f32)
        if B["ln2_w"] is not None:
            h, _ = ln_fwd(h, B["ln2_w"], B["ln2_b"], m.ln_eps)
        x = (x + B["down"](act_fwd(B["up"](h), "gelu")) * mod[:, 5 * P:6 * P]).astype(f32)
    x, _ = ln_fwd(x, L.norm_w, L.norm_b, m.ln_eps)
    if L.out_proj is not None:
        x = L.out_proj(x)
    if L.proj0 is not None:
        x = L.proj2(act_fwd(L.proj0(x), "gelu"))
    return x


def rollout(m: Model, level: int, seeds, actions, n_steps: int, history: int):
    """seeds [n_seed][D], actions [n_seed + n_steps - 1][A] -> the n_steps predicted states: step j reads the
    last `history` frames of the growing sequence (seeds, then predictions) and their actions."""
    seq = [np.asarray(s, f32) for s in seeds]
    out = []
    for _ in range(n_steps):
        have = len(seq)
        w = min(history, have)
        nxt = predict(m, level, np.stack(seq[have - w:have]), actions[have - w:have])[-1]
        seq.append(nxt)
        out.append(nxt)
    return np.stack(out)


# ---------------------------------------------------------------------------------------------
# the state and action encoders of the API: jepa_hjepa_embed / _lift / _action_embed / _action_encode
# (src/hjepa.cpp:374-561)
# ---------------------------------------------------------------------------------------------
def embed(m: Model, cls, proprio=None):
    """Level-1 states from the encoder's CLS rows [n][Dv] (and the proprio stream [n][P]): the projector
    (mlp with GELU / layernorm / identity), then [pixel | proprio] for 'vit_proprio' (hjepa.cpp:374-414)."""
    x = np.asarray(cls, f32)
    if m.proj_kind == "mlp":
        x = m.proj2(act_fwd(m.proj0(x), "gelu"))
    elif m.proj_kind == "layernorm":
        x, _ = ln_fwd(x, m.proj_ln[0], m.proj_ln[1], m.ln_eps)
    if m.levels[0].hp["enc_kind"] == "vit_proprio":
        h, _ = ln_fwd(m.pro0(np.asarray(proprio, f32)), m.pro_ln[0], m.pro_ln[1], m.ln_eps)
        x = np.concatenate([x, m.pro2(act_fwd(h, "gelu"))], axis=1).astype(f32)
    return x


def lift(m: Model, level: int, below):
    """Level-k states: the state encoder on every stride-th state of level k-1 (hjepa.cpp:416-448)."""
    up = m.levels[level - 1]
    x = np.ascontiguousarray(np.asarray(below, f32)[::up.hp["stride"]])
    y, _ = encode_up_fwd(m, up, x)
    return y


def action_embed(m: Model, level: int, actions):
    """The level's actions through act_embed (identity when absent) (hjepa.cpp:454-467)."""
    e, _ = act_embed_fwd(m.levels[level - 1], np.asarray(actions, f32))
    return e


def action_encode(m: Model, level: int, below_emb):
    """Latent actions of level k from the level below's action embeddings [n][E]: chunks of `stride` rows,
    a short trailing chunk zero-padded for 'mlp' and run at its own length for 'seq' (hjepa.cpp:508-561)."""
    up = m.levels[level - 1]
    S = up.hp["stride"]
    emb = np.asarray(below_emb, f32)
    n = emb.shape[0]
    n_out = (n + S - 1) // S
    if up.hp["act_enc_kind"] == "mlp":
        pad = np.zeros((n_out * S, emb.shape[1]), f32)
        pad[:n] = emb
        chunks = [np.ascontiguousarray(pad[i::S]) for i in range(S)]   # step i of every chunk
        y, _ = action_pool_fwd(m, up, chunks)
        return y
    out = []
    for c in range(n_out):
        rows = emb[c * S:min(n, (c + 1) * S)]
        y, _ = action_pool_fwd(m, up, [rows[i:i + 1] for i in range(rows.shape[0])])
        out.append(y[0])
    return np.stack(out).astype(f32)
