"""ORACLE ONLY -- test infrastructure, never the product path.

A numpy restatement of the reference's V-JEPA 2-AC world model and CEM planner. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import it, and only as the checker.

  predictor forward   src/vjepa2_ac.cpp:86-156 (jepa_build_ac) over the pre-LN block of src/jepa.cpp:444-471,
                      following the reference's executable spec scripts/jepa_convert/selftest.py:304-395
                      (ac_block_causal_mask, ac_token_ids, ac_predictor_forward)
  3-D RoPE tables     src/rope3d.cpp:9-134 (tiled layout, float32 angle products, sign folded into sin)
  rollout             src/vjepa2_ac.cpp:455-577 (ac_rollout: seed frames, per-step actions / poses,
                      normalize_reps between steps)
  pose update         src/vjepa2_ac.cpp:207-251 (jepa_ac_next_state)
  energy              src/vjepa2_ac.cpp:253-263 (jepa_ac_energy)
  CEM                 src/vjepa2_ac.cpp:829-946 (jepa_ac_plan with explicit noise)

Parity pin: tests/golden/ac_spec.npz holds outputs of the reference's own numpy spec
(selftest.ac_predictor_forward), written by tests/golden/make_golden_ac.py; tests/vectors of the
reference (rope3d hd64 "hf" cases) pin the RoPE tables -- copied as tests/golden/rope3d_hf.npz.
"""
from __future__ import annotations

import math

import numpy as np

from hjepa_oracle import load_tensors

f32 = np.float32


class ACModel:
    def __init__(self, path: str):
        self.T, meta = load_tensors(path)
        g = lambda k, d=None: meta.get(k, d)
        self.enc_dim = int(g("jepa.enc.embed_dim"))
        self.D = int(g("jepa.pred.embed_dim"))
        self.n_layer = int(g("jepa.pred.n_layer"))
        self.n_head = int(g("jepa.pred.n_head"))
        self.hd = self.D // self.n_head
        self.grid = int(g("jepa.pred.grid_size"))
        self.HW = self.grid * self.grid
        self.A = int(g("jepa.pred.action_dim"))
        self.S = int(g("jepa.pred.state_dim"))
        self.n_cond = int(g("jepa.pred.n_cond_tokens"))
        self.eps = float(g("jepa.pred.ln_eps", 1e-6))
        self.norm_eps = float(g("jepa.pred.norm_reps_eps", 1e-5))
        self.normalize_reps = bool(g("jepa.pred.normalize_reps", False))
        self.frame_causal = bool(g("jepa.pred.frame_causal", False))
        self.theta = float(g("jepa.enc.rope_theta", 10000.0))
        self.layout = str(g("jepa.pred.rope_freq_layout", "tiled"))

    def w(self, name):
        return self.T[name]

    def b(self, name):
        return self.T.get(name)


def layer_norm(x, w, b, eps):
    """float32 LayerNorm (the spec's numpy layer_norm, selftest.py:81-90)."""
    x = x.astype(f32)
    mu = x.mean(-1, keepdims=True, dtype=np.float64).astype(f32)
    var = ((x - mu) ** 2).mean(-1, keepdims=True, dtype=np.float64).astype(f32)
    y = (x - mu) / np.sqrt(var + f32(eps))
    if w is not None:
        y = y * w
    if b is not None:
        y = y + b
    return y.astype(f32)


def gelu(x):
    """GELU with the exact erf, evaluated in double (scipy's vectorised erf when present, else math.erf)."""
    z = x.astype(np.float64) / math.sqrt(2.0)
    try:
        from scipy.special import erf as verf
        e = verf(z)
    except ImportError:
        from math import erf
        e = np.vectorize(erf, otypes=[np.float64])(z)
    return (0.5 * x * (1.0 + e)).astype(f32)


def linear(x, w, b):
    y = x.astype(f32) @ w.T.astype(f32)
    return (y + b if b is not None else y).astype(f32)


# ---------------------------------------------------------------------------------------------
# 3-D RoPE (src/rope3d.cpp:9-134): per-axis width d = 2 ((hd / 3) / 2), dims [0,d) rotate with t,
# [d,2d) with h, [2d,3d) with w; omega_k = 1 / theta^(k / (d/2)), angle = pos * omega (float32);
# tiled layout uses omega[j mod d/2]; the sign of the rotation is folded into sin (even lanes negated)
# ---------------------------------------------------------------------------------------------
def rope_tables(ids, grid, hd, theta, layout="tiled"):
    ids = np.asarray(ids, np.int64)
    d = 2 * ((hd // 3) // 2)
    half = d // 2
    omega = np.array([f32(1.0) / np.power(f32(theta), f32(k) / f32(half), dtype=f32) for k in range(half)], f32)
    per = grid * grid
    pos = [(ids // per).astype(f32), ((ids % per) // grid).astype(f32), (ids % grid).astype(f32)]
    N = ids.size
    cos = np.ones((N, hd), f32)
    sin = np.zeros((N, hd), f32)
    for ax in range(3):
        for j in range(d):
            k = (j % half) if layout == "tiled" else (j // 2)
            ang = (pos[ax] * omega[k]).astype(f32)
            cos[:, ax * d + j] = np.cos(ang)
            sin[:, ax * d + j] = np.sin(ang)
    sin[:, 0::2] = -sin[:, 0::2]
    return cos, sin


def rope_apply(x, cos, sin):
    """x [..., N, hd]: out = x * C + swap(x) * S' (swap exchanges lanes 2k and 2k+1)."""
    sw = np.empty_like(x)
    sw[..., 0::2] = x[..., 1::2]
    sw[..., 1::2] = x[..., 0::2]
    return (x * cos + sw * sin).astype(f32)


def token_ids(T, grid, n_cond):
    ids = []
    for t in range(T):
        base = t * grid * grid
        ids += [base] * n_cond + [base + i for i in range(grid * grid)]
    return np.asarray(ids, np.int64)


# ---------------------------------------------------------------------------------------------
# predictor forward (one item)
# ---------------------------------------------------------------------------------------------
def predict_all(m: ACModel, context, actions, states):
    """context [T HW, enc_dim], actions [T, A], states [T, S] -> [T HW, enc_dim]: row block t is the
    prediction of frame t+1 given frames 0..t (jepa_ac_predict_all)."""
    T = context.shape[0] // m.HW
    D, H, hd = m.D, m.n_head, m.hd
    x = linear(context, m.w("pred.embed.weight"), m.b("pred.embed.bias")).reshape(T, m.HW, D)
    a = linear(actions, m.w("pred.action_embed.weight"), m.b("pred.action_embed.bias"))
    s = linear(states, m.w("pred.state_embed.weight"), m.b("pred.state_embed.bias"))
    seq = np.concatenate([a[:, None, :], s[:, None, :], x], axis=1).reshape(T * (m.n_cond + m.HW), D).astype(f32)
    N = seq.shape[0]
    cos, sin = rope_tables(token_ids(T, m.grid, m.n_cond), m.grid, hd, m.theta, m.layout)
    frame = np.arange(N) // (m.n_cond + m.HW)
    mask = (frame[:, None] >= frame[None, :]) if (m.frame_causal and T > 1) else None
    for i in range(m.n_layer):
        p = f"pred.blk.{i}."
        h = layer_norm(seq, m.w(p + "ln1.weight"), m.b(p + "ln1.bias"), m.eps)
        qkv = linear(h, m.w(p + "attn_qkv.weight"), m.b(p + "attn_qkv.bias"))
        q = qkv[:, :D].reshape(N, H, hd).transpose(1, 0, 2)
        k = qkv[:, D:2 * D].reshape(N, H, hd).transpose(1, 0, 2)
        v = qkv[:, 2 * D:].reshape(N, H, hd).transpose(1, 0, 2)
        q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
        att = (q @ k.transpose(0, 2, 1)).astype(f32) / f32(math.sqrt(hd))
        if mask is not None:
            att = np.where(mask[None], att, -np.inf)
        att = np.exp(att - att.max(-1, keepdims=True))
        att = att / att.sum(-1, keepdims=True)
        o = (att @ v).transpose(1, 0, 2).reshape(N, D).astype(f32)
        seq = (seq + linear(o, m.w(p + "attn_out.weight"), m.b(p + "attn_out.bias"))).astype(f32)
        h = layer_norm(seq, m.w(p + "ln2.weight"), m.b(p + "ln2.bias"), m.eps)
        u = gelu(linear(h, m.w(p + "ffn_up.weight"), m.b(p + "ffn_up.bias")))
        seq = (seq + linear(u, m.w(p + "ffn_down.weight"), m.b(p + "ffn_down.bias"))).astype(f32)
    rows = seq.reshape(T, m.n_cond + m.HW, D)[:, m.n_cond:, :].reshape(T * m.HW, D)
    rows = layer_norm(rows, m.w("pred.norm.weight"), m.b("pred.norm.bias"), m.eps)
    return linear(rows, m.w("pred.proj.weight"), m.b("pred.proj.bias"))


def normalize(m: ACModel, rows):
    """jepa_ac_normalize (src/vjepa2_ac.cpp:182-196): float64 mean / variance, float inverse std of
    (float) var + eps, then (x - (float) mean) * inv."""
    rows = rows.astype(f32)
    mu = rows.astype(np.float64).mean(-1, keepdims=True)
    var = ((rows.astype(np.float64) - mu) ** 2).mean(-1, keepdims=True)
    inv = (f32(1.0) / np.sqrt(var.astype(f32) + f32(m.norm_eps))).astype(f32)
    return ((rows - mu.astype(f32)) * inv).astype(f32)


def next_state(state, action):
    """jepa_ac_next_state: xyz added; R(action) R(pose) as extrinsic-xyz Euler; gripper clipped."""
    def rot(e):
        a, b, c = (float(v) for v in e)
        ca, sa, cb, sb, cc, sc = math.cos(a), math.sin(a), math.cos(b), math.sin(b), math.cos(c), math.sin(c)
        return np.array([[cb * cc, sa * sb * cc - ca * sc, ca * sb * cc + sa * sc],
                         [cb * sc, sa * sb * sc + ca * cc, ca * sb * sc - sa * cc],
                         [-sb, sa * cb, ca * cb]])
    Dm, P = rot(action[3:6]), rot(state[3:6])
    # R = Dm P, each entry summed left to right in double (no fused multiply-add)
    R = np.array([[Dm[i, 0] * P[0, j] + Dm[i, 1] * P[1, j] + Dm[i, 2] * P[2, j] for j in range(3)] for i in range(3)])
    s = max(-1.0, min(1.0, -R[2, 0]))
    beta = math.asin(s)
    if abs(s) < 1.0 - 1e-9:
        alpha, gamma = math.atan2(R[2, 1], R[2, 2]), math.atan2(R[1, 0], R[0, 0])
    else:
        alpha, gamma = math.atan2(-R[1, 2], R[1, 1]), 0.0
    out = np.array(state, f32).copy()
    out[:3] = (np.asarray(state[:3], f32) + np.asarray(action[:3], f32)).astype(f32)
    out[3], out[4], out[5] = f32(alpha), f32(beta), f32(gamma)
    out[6] = min(max(f32(state[6]) + f32(action[6]), f32(0)), f32(1))
    return out


def rollout(m: ACModel, latents, n_seed, seed_actions, seed_states, actions, states=None):
    """ac_rollout for K candidates: latents [n_seed HW, enc], actions [K, H, A] -> [K, H, HW, enc]."""
    K, H, A = actions.shape
    HW, E = m.HW, m.enc_dim
    n_seq = n_seed + H - 1
    out = np.zeros((K, H, HW, E), f32)
    for c in range(K):
        st = np.zeros((n_seq, m.S), f32)
        st[:n_seed] = seed_states
        act = np.zeros((n_seq, A), f32)
        tail = []
        for step in range(H):
            T = n_seed + step
            for j in range(T):
                if j < n_seed - 1:
                    act[j] = seed_actions[j] if seed_actions is not None else actions[c, 0]
                    continue
                k = min(j - (n_seed - 1), step)
                act[j] = actions[c, k]
                if j >= n_seed:
                    st[j] = states[c, j - n_seed] if states is not None else next_state(st[j - 1], act[j - 1])
            ctx = np.concatenate([latents] + tail, axis=0) if tail else latents
            pred = predict_all(m, ctx, act[:T], st[:T])[-HW:]
            if m.normalize_reps:
                pred = normalize(m, pred)
            out[c, step] = pred
            tail.append(pred)
    return out


def energy(pred, goal):
    """jepa_ac_energy: mean |pred - goal| per item, double accumulation."""
    K = pred.shape[0]
    d = np.abs(pred.reshape(K, -1).astype(np.float64) - goal.reshape(1, -1).astype(np.float64))
    return (d.sum(1) / d.shape[1]).astype(f32)


def cem_draws(seed: int, n: int) -> np.ndarray:
    """The normal draws jepa_ac_plan makes when it is given no noise (src/vjepa2_ac.cpp:804-826): xorshift128+
    with shifts 23 / 17 / 26, state (0x9E3779B97F4A7C15 ^ seed, 0xBF58476D1CE4E5B9 + seed) advanced by 8
    outputs; a uniform in (0, 1] from the top 53 bits of an output, ((x >> 11) + 1) / (2^53 + 1) in double
    rounded to float; one normal from two uniforms, sqrtf(-2 logf(u1)) * cosf(2 pi u2) in float. The float
    functions are the C library's own (logf, cosf, sqrtf through ctypes), as in the reference's host code."""
    import ctypes
    libm = ctypes.CDLL("libm.so.6")
    for fn in ("logf", "cosf", "sqrtf"):
        getattr(libm, fn).restype = ctypes.c_float
        getattr(libm, fn).argtypes = [ctypes.c_float]
    mask = (1 << 64) - 1
    s = [(0x9E3779B97F4A7C15 ^ seed) & mask, (0xBF58476D1CE4E5B9 + seed) & mask]

    def advance():
        x, y = s
        s[0] = y
        x ^= (x << 23) & mask
        s[1] = x ^ y ^ (x >> 17) ^ (y >> 26)
        return (s[1] + y) & mask

    for _ in range(8):
        advance()
    two_pi = f32(6.2831853071795864769)
    out = np.empty(n, f32)
    for i in range(n):
        u1 = f32(((advance() >> 11) + 1) * (1.0 / 9007199254740993.0))
        u2 = f32(((advance() >> 11) + 1) * (1.0 / 9007199254740993.0))
        r = f32(libm.sqrtf(float(f32(-2.0) * f32(libm.logf(float(u1))))))
        out[i] = r * f32(libm.cosf(float(two_pi * u2)))
    return out


def cem(m: ACModel, latents, n_seed, seed_actions, seed_states, goal, p: dict, noise, rollout_fn=None, A=None,
        energy_fn=None):
    """jepa_ac_plan with explicit noise [cem_steps, H, K, 4] (src/vjepa2_ac.cpp:829-946). Returns
    (actions [H, A], best energy per iteration, elite index sets per iteration).

    rollout_fn(acts [K, H, A]) -> [K, H, HW, E] replaces the numpy rollout (a test drives the refit with the
    GPU's predictions to check the CEM arithmetic on its own); energy_fn(acts) -> [K] replaces rollout and
    energy together (the sharding protocol test gathers per-rank energies through it). The refit follows the reference's float /
    double mix exactly: elite sums and squared deviations accumulate in double in elite order, the
    momentum terms multiply two floats in float (mn * momentum) before the double sum."""
    K, H = p["samples"], p["horizon"]
    A = A if A is not None else m.A
    mm, ms = f32(p["momentum_mean"]), f32(p["momentum_std"])
    mmg, msg = f32(p["momentum_mean_gripper"]), f32(p["momentum_std_gripper"])
    maxnorm, gclamp = f32(p["maxnorm"]), f32(p["gripper_clamp"])
    mean = np.zeros((H, 4), f32)
    sd = np.zeros((H, 4), f32)
    sd[:, :3] = maxnorm
    sd[:, 3] = f32(1.0)
    best, elites = [], []
    topk = p["topk"]
    for it in range(p["cem_steps"]):
        acts = np.zeros((K, H, A), f32)
        for h in range(H):
            z = noise[it, h].astype(f32)                     # [K, 4]
            v = (z * sd[h] + mean[h]).astype(f32)
            v[:, :3] = np.minimum(np.maximum(v[:, :3], -maxnorm), maxnorm)
            v[:, 3] = np.minimum(np.maximum(v[:, 3], -gclamp), gclamp)
            acts[:, h, 0:3] = v[:, :3]
            acts[:, h, 6] = v[:, 3]
        if energy_fn is not None:
            e = np.asarray(energy_fn(acts), np.float32)
        else:
            roll = rollout_fn(acts) if rollout_fn is not None else rollout(m, latents, n_seed, seed_actions, seed_states, acts)
            e = energy(roll[:, H - 1], goal)
        order = np.argsort(e, kind="stable")
        best.append(float(e[order[0]]))
        elites.append(order[:topk].copy())
        for h in range(H):
            el = [[float(acts[c, h, 0]), float(acts[c, h, 1]), float(acts[c, h, 2]), float(acts[c, h, 6])] for c in order[:topk]]
            mu = [0.0] * 4
            for row in el:
                for j in range(4):
                    mu[j] += row[j]
            mu = [x / float(topk) for x in mu]
            var = [0.0] * 4
            for row in el:
                for j in range(4):
                    d = row[j] - mu[j]
                    var[j] += d * d
            denom = float(topk - 1) if topk > 1 else 1.0
            var = [math.sqrt(x / denom) for x in var]
            for j in range(3):
                mean[h, j] = f32(mu[j] * (1.0 - float(mm)) + float(f32(mean[h, j] * mm)))
                sd[h, j] = f32(var[j] * (1.0 - float(ms)) + float(f32(sd[h, j] * ms)))
            mean[h, 3] = f32(mu[3] * (1.0 - float(mmg)) + float(f32(mean[h, 3] * mmg)))
            sd[h, 3] = f32(var[3] * (1.0 - float(msg)) + float(f32(sd[h, 3] * msg)))
    out = np.zeros((H, A), f32)
    out[:, 0:3] = mean[:, 0:3]
    g = mean[:, 3]
    out[:, 6] = np.where(np.abs(g) < f32(p["round_gripper"]), f32(0.0), g)
    return out, np.array(best, f32), elites
