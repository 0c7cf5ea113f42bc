"""Python view of the engine's H-JEPA planner through its C ABI (libjepa.so), mirroring the planner
calls of the reference's binding (python/src/jepa_cpp/model.py:994-1127): one model + context, costs
and gradients of candidates, one level's solve, the top-down hierarchy. Host numpy arrays in and out.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import numpy as np

from . import capi
from . import lib as jlib


class _Output(C.Structure):
    _fields_ = [("data", capi.FP), ("n_tokens", C.c_int64), ("dim", C.c_int64)]


class _Input(C.Structure):
    _fields_ = [("data", capi.FP), ("n_batch", C.c_int), ("n_chans", C.c_int), ("n_frames", C.c_int),
                ("height", C.c_int), ("width", C.c_int)]


class Planner:
    def __init__(self, path: str, device: int = -1, verbose: bool = False):
        self.lib = L = jlib.load()
        L.jepa_model_load.restype = C.c_void_p
        L.jepa_model_load.argtypes = [C.c_char_p, C.c_bool]
        L.jepa_context_new.restype = C.c_void_p
        L.jepa_context_new.argtypes = [C.c_void_p, _CtxParams]
        L.jepa_context_default_params.restype = _CtxParams
        L.jepa_hjepa_embed_dim.argtypes = [C.c_void_p, C.c_int]
        L.jepa_hjepa_action_dim.argtypes = [C.c_void_p, C.c_int]
        L.jepa_hjepa_n_levels.argtypes = [C.c_void_p]
        L.jepa_error_reset()
        if device >= 0:
            L.jepa_model_load_ex.restype = C.c_void_p
            L.jepa_model_load_ex.argtypes = [C.c_char_p, C.POINTER(_ModelParams)]
            mp = _ModelParams(verbose, device)
            self.model = L.jepa_model_load_ex(path.encode(), C.byref(mp))
        else:
            self.model = L.jepa_model_load(path.encode(), verbose)
        if not self.model:
            raise RuntimeError(f"jepa_model_load({path}) failed: {jlib.error_text()}")
        self.ctx = L.jepa_context_new(self.model, L.jepa_context_default_params())
        if not self.ctx:
            raise RuntimeError(f"jepa_context_new failed: {jlib.error_text()}")
        self.n_levels = L.jepa_hjepa_n_levels(self.model)

    def close(self) -> None:
        if getattr(self, "ctx", None):
            self.lib.jepa_context_free(C.c_void_p(self.ctx))
            self.lib.jepa_model_free(C.c_void_p(self.model))
            self.ctx = self.model = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def embed_dim(self, level: int) -> int:
        return self.lib.jepa_hjepa_embed_dim(self.model, level)

    def action_dim(self, level: int) -> int:
        return self.lib.jepa_hjepa_action_dim(self.model, level)

    def set_shard(self, rank: int, world: int, nccl_id: Optional[bytes]) -> None:
        buf = C.create_string_buffer(nccl_id, 128) if nccl_id is not None else None
        if self.lib.jepa_b200_context_set_shard(self.ctx, rank, world, buf) != 0:
            raise RuntimeError(f"jepa_b200_context_set_shard failed: {jlib.error_text()}")

    def predict(self, level: int, states, actions) -> np.ndarray:
        """jepa_hjepa_predict: states [T, D], actions [T, A] -> [T, D_out], row t predicted after frames 0..t."""
        states = np.ascontiguousarray(states, np.float32)
        actions = np.ascontiguousarray(actions, np.float32)
        out = _Output()
        fn = self.lib.jepa_hjepa_predict
        fn.argtypes = [C.c_void_p, C.c_int, capi.FP, capi.FP, C.c_int, C.POINTER(_Output)]
        if fn(self.ctx, level, capi.fptr(states), capi.fptr(actions), states.shape[0], C.byref(out)) != 0:
            raise RuntimeError(f"jepa_hjepa_predict failed: {jlib.error_text()}")
        try:
            res = np.ctypeslib.as_array(out.data, shape=(out.n_tokens * out.dim,)).copy()
        finally:
            self.lib.jepa_free.argtypes = [C.c_void_p]
            self.lib.jepa_free(C.cast(out.data, C.c_void_p))
        return res.reshape(out.n_tokens, out.dim)

    def _output(self, fn_name: str, call) -> np.ndarray:
        out = _Output()
        if call(C.byref(out)) != 0:
            raise RuntimeError(f"{fn_name} failed: {jlib.error_text()}")
        try:
            res = np.ctypeslib.as_array(out.data, shape=(out.n_tokens * out.dim,)).copy()
        finally:
            self.lib.jepa_free.argtypes = [C.c_void_p]
            self.lib.jepa_free(C.cast(out.data, C.c_void_p))
        return res.reshape(out.n_tokens, out.dim)

    def encode(self, images) -> np.ndarray:
        """jepa_encode: images [B, C, H, W] (or [B, C, T, H, W]) -> [B (T) N, D], final norm applied."""
        x = np.ascontiguousarray(images, np.float32)
        if x.ndim == 4:
            x = x[:, :, None]
        inp = _Input(capi.fptr(x), x.shape[0], x.shape[1], x.shape[2], x.shape[3], x.shape[4])
        fn = self.lib.jepa_encode
        fn.argtypes = [C.c_void_p, C.POINTER(_Input), C.POINTER(_Output)]
        return self._output("jepa_encode", lambda o: fn(self.ctx, C.byref(inp), o))

    def pool(self, kind: str, enc: np.ndarray) -> np.ndarray:
        """jepa_pool_cls / jepa_pool_mean of one item's encoder rows [N, D]."""
        enc = np.ascontiguousarray(enc, np.float32)
        src = _Output(capi.fptr(enc), enc.shape[0], enc.shape[1])
        fn = getattr(self.lib, "jepa_pool_" + kind)
        fn.argtypes = [C.c_void_p, C.POINTER(_Output), C.POINTER(_Output)]
        return self._output("jepa_pool_" + kind, lambda o: fn(self.model, C.byref(src), o))[0]

    def encode_states(self, cls_rows, proprio=None) -> np.ndarray:
        """jepa_hjepa_embed: the encoder's CLS rows [n, Dv] (and the proprio stream [n, P]) -> level-1 states."""
        cls_rows = np.ascontiguousarray(cls_rows, np.float32)
        pr = None if proprio is None else np.ascontiguousarray(proprio, np.float32)
        fn = self.lib.jepa_hjepa_embed
        fn.argtypes = [C.c_void_p, capi.FP, capi.FP, C.c_int, C.POINTER(_Output)]
        return self._output("jepa_hjepa_embed",
                            lambda o: fn(self.ctx, capi.fptr(cls_rows), capi.fptr(pr), cls_rows.shape[0], o))

    def encoder(self, kind: str, level: int, rows) -> np.ndarray:
        """jepa_hjepa_lift / _action_embed / _action_encode ('lift', 'action_embed', 'action_encode') of rows [n, *]."""
        rows = np.ascontiguousarray(rows, np.float32)
        name = {"lift": "jepa_hjepa_lift", "action_embed": "jepa_hjepa_action_embed",
                "action_encode": "jepa_hjepa_action_encode"}[kind]
        fn = getattr(self.lib, name)
        fn.argtypes = [C.c_void_p, C.c_int, capi.FP, C.c_int, C.POINTER(_Output)]
        return self._output(name, lambda o: fn(self.ctx, level, capi.fptr(rows), rows.shape[0], o))

    def rollout(self, level: int, seeds, actions, n_steps: int, history: int) -> np.ndarray:
        """jepa_hjepa_rollout: seeds [n_seed, D], actions [n_seed + n_steps - 1, A] -> [n_steps, D]."""
        seeds = np.ascontiguousarray(np.atleast_2d(seeds), np.float32)
        actions = np.ascontiguousarray(actions, np.float32)
        out = np.zeros((n_steps, seeds.shape[1]), np.float32)
        fn = self.lib.jepa_hjepa_rollout
        fn.argtypes = [C.c_void_p, C.c_int, capi.FP, C.c_int, capi.FP, C.c_int, C.c_int, capi.FP]
        if fn(self.ctx, level, capi.fptr(seeds), seeds.shape[0], capi.fptr(actions), n_steps, history, capi.fptr(out)) != 0:
            raise RuntimeError(f"jepa_hjepa_rollout failed: {jlib.error_text()}")
        return out

    def set_streams(self, n: int) -> None:
        """Candidate streams of the solves (0 = automatic); results do not depend on it."""
        if self.lib.jepa_b200_hjepa_set_streams(self.ctx, int(n)) != 0:
            raise RuntimeError(f"jepa_b200_hjepa_set_streams failed: {jlib.error_text()}")

    def set_step_modulation(self, mode: int) -> None:
        """0: every step's adaLN modulation kept when it fits (automatic); 1: one step at a time."""
        if self.lib.jepa_b200_hjepa_set_step_modulation(self.ctx, int(mode)) != 0:
            raise RuntimeError(f"jepa_b200_hjepa_set_step_modulation failed: {jlib.error_text()}")

    def last_ms(self) -> float:
        return self.lib.jepa_b200_last_plan_ms(self.ctx)

    def last_launches(self) -> int:
        return self.lib.jepa_b200_last_plan_launches(self.ctx)

    def plan_cost(self, level, state, goal, actions, goal_level=0, dense=0, plan: Optional[dict] = None,
                  want_grad=True, goal_actions=None):
        actions = np.ascontiguousarray(actions, np.float32)
        S, T, _ = actions.shape
        state = np.ascontiguousarray(state, np.float32)
        goal = np.ascontiguousarray(np.atleast_2d(goal), np.float32)
        ga = None if goal_actions is None else np.ascontiguousarray(goal_actions, np.float32)
        g = capi.Goal(capi.fptr(goal), goal.shape[0], goal_level, dense, capi.fptr(ga))
        lp = capi.LevelPlan.of(**plan) if plan is not None else None
        costs = np.zeros(S, np.float32)
        grad = np.zeros_like(actions) if want_grad else None
        rc = self.lib.jepa_hjepa_plan_cost(self.ctx, level, capi.fptr(state), C.byref(g),
                                           C.byref(lp) if lp is not None else None, capi.fptr(actions), S, T,
                                           capi.fptr(costs), capi.fptr(grad))
        if rc != 0:
            raise RuntimeError(f"jepa_hjepa_plan_cost failed: {jlib.error_text()}")
        return costs, grad

    def solve(self, level, state, goal, plan: dict, noise=None, goal_level=0, n_goal=None):
        goal = np.ascontiguousarray(np.atleast_2d(goal), np.float32)
        state = np.ascontiguousarray(state, np.float32)
        g = capi.Goal(capi.fptr(goal), n_goal or goal.shape[0], goal_level, 0, capi.fptr(None))
        lp = capi.LevelPlan.of(**plan)
        T, A, D = plan["horizon"], self.action_dim(level), self.embed_dim(level)
        act = np.zeros((T, A), np.float32)
        st = np.zeros((T + 1, D), np.float32)
        cost, it = C.c_float(), C.c_int()
        rp = capi.Replay(noise) if noise is not None else None
        fn = rp.fn if rp is not None else capi.RANDN_FN()
        rc = self.lib.jepa_hjepa_solve(self.ctx, level, capi.fptr(state), C.byref(g), C.byref(lp), fn, None,
                                       capi.fptr(act), capi.fptr(st), C.byref(cost), C.byref(it))
        if rc != 0:
            raise RuntimeError(f"jepa_hjepa_solve failed: {jlib.error_text()}")
        return act, st, cost.value, it.value, (rp.pos if rp is not None else None)

    def plan(self, states: Sequence[np.ndarray], goals: Sequence[np.ndarray], plans: Sequence[dict], noise=None):
        n = len(plans)
        sts = [np.ascontiguousarray(s, np.float32) for s in states]
        gls = [np.ascontiguousarray(g, np.float32) for g in goals]
        SP = (capi.FP * n)(*[capi.fptr(s) for s in sts])
        GP = (capi.FP * n)(*[capi.fptr(g) for g in gls])
        lps = (capi.LevelPlan * n)(*[capi.LevelPlan.of(**p) for p in plans])
        out = np.zeros((plans[0]["horizon"], self.action_dim(1)), np.float32)
        info = capi.PlanInfo()
        rp = capi.Replay(noise) if noise is not None else None
        fn = rp.fn if rp is not None else capi.RANDN_FN()
        rc = self.lib.jepa_hjepa_plan(self.ctx, SP, GP, lps, n, fn, None, capi.fptr(out), C.byref(info))
        if rc != 0:
            raise RuntimeError(f"jepa_hjepa_plan failed: {jlib.error_text()}")
        return out, info, (rp.pos if rp is not None else None)


class _CtxParams(C.Structure):
    _fields_ = [("n_threads", C.c_int), ("use_flash_attn", C.c_bool), ("verbose", C.c_bool), ("flash_kv", C.c_int)]


class _ModelParams(C.Structure):
    _fields_ = [("verbose", C.c_bool), ("device", C.c_int)]
