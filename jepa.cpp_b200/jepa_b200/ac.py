"""Python view of the engine's V-JEPA 2-AC world model and CEM planner through its C ABI (libjepa.so),
with the argument meaning of the reference's binding (python/src/jepa_cpp/_api.py:362-395): predict /
predict_all, rollout / rollout_ex, the cached context handle, and jepa_ac_plan. Host numpy arrays in and out.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import capi
from . import lib as jlib
from .hjepa import _CtxParams, _ModelParams

FP = capi.FP


class _Output(C.Structure):
    _fields_ = [("data", FP), ("n_tokens", C.c_int64), ("dim", C.c_int64)]


def _declare(L: C.CDLL) -> None:
    vp = C.c_void_p
    sig = {
        "jepa_model_load_ex": (vp, [C.c_char_p, C.POINTER(_ModelParams)]),
        "jepa_context_new": (vp, [vp, _CtxParams]),
        "jepa_context_default_params": (_CtxParams, []),
        "jepa_ac_tokens_per_frame": (C.c_int, [vp]),
        "jepa_ac_action_dim": (C.c_int, [vp]),
        "jepa_ac_state_dim": (C.c_int, [vp]),
        "jepa_ac_max_frames": (C.c_int, [vp]),
        "jepa_ac_normalize_reps": (C.c_bool, [vp]),
        "jepa_ac_normalize": (None, [vp, FP, C.c_int64, C.c_int64]),
        "jepa_ac_predict": (C.c_int, [vp, FP, C.c_int, C.c_int, FP, FP, C.POINTER(_Output)]),
        "jepa_ac_predict_all": (C.c_int, [vp, FP, C.c_int, C.c_int, FP, FP, C.POINTER(_Output)]),
        "jepa_ac_rollout": (C.c_int, [vp, FP, C.c_int, FP, FP, FP, C.c_int, C.c_int, FP]),
        "jepa_ac_rollout_ex": (C.c_int, [vp, FP, C.c_int, FP, FP, FP, FP, C.c_int, C.c_int, FP]),
        "jepa_ac_context_new": (vp, [vp, FP, C.c_int, FP, FP]),
        "jepa_ac_context_free": (None, [vp]),
        "jepa_ac_context_n_frames": (C.c_int, [vp]),
        "jepa_ac_context_capacity": (C.c_int, [vp]),
        "jepa_ac_context_update": (C.c_int, [vp, FP, FP, FP]),
        "jepa_ac_context_trim": (C.c_int, [vp, C.c_int]),
        "jepa_ac_rollout_cached": (C.c_int, [vp, vp, FP, FP, C.c_int, C.c_int, FP]),
        "jepa_ac_cem_default_params": (capi.CemParams, []),
        "jepa_ac_plan": (C.c_int, [vp, vp, FP, C.POINTER(capi.CemParams), FP, FP, FP]),
        "jepa_ac_energy": (None, [FP, FP, C.c_int, C.c_int64, C.c_int64, FP]),
        "jepa_free": (None, [vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, np.float32)


class ACWorldModel:
    """One V-JEPA 2-AC model and context on one GPU."""

    def __init__(self, path: str, device: int = 0, verbose: bool = False):
        self.lib = L = jlib.load()
        _declare(L)
        L.jepa_error_reset()
        mp = _ModelParams(verbose, device)
        self.model = L.jepa_model_load_ex(path.encode(), C.byref(mp))
        if not self.model:
            raise RuntimeError(f"jepa_model_load({path}) failed: {jlib.error_text()}")
        self.ctx = L.jepa_context_new(self.model, L.jepa_context_default_params())
        if not self.ctx:
            raise RuntimeError(f"jepa_context_new failed: {jlib.error_text()}")
        self.HW = L.jepa_ac_tokens_per_frame(self.model)
        self.A = L.jepa_ac_action_dim(self.model)
        self.S = L.jepa_ac_state_dim(self.model)
        self.max_frames = L.jepa_ac_max_frames(self.model)
        self.handles = []

    def close(self) -> None:
        if getattr(self, "ctx", None):
            for h in self.handles:
                self.lib.jepa_ac_context_free(C.c_void_p(h))
            self.handles = []
            self.lib.jepa_context_free(C.c_void_p(self.ctx))
            self.lib.jepa_model_free(C.c_void_p(self.model))
            self.ctx = self.model = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what} failed: {jlib.error_text()}")

    def set_shard(self, rank: int, world: int, nccl_id: Optional[bytes]) -> None:
        buf = C.create_string_buffer(nccl_id, 128) if nccl_id is not None else None
        self._check(self.lib.jepa_b200_context_set_shard(self.ctx, rank, world, buf), "jepa_b200_context_set_shard")

    def last_ms(self) -> float:
        return self.lib.jepa_b200_last_plan_ms(self.ctx)

    def predict(self, context, actions, states, all_frames: bool = False) -> np.ndarray:
        """context [B, T HW, E], actions [B, T, A], states [B, T, S] -> [B, n_out HW, out_dim]."""
        context, actions, states = _f32(context), _f32(actions), _f32(states)
        B, T = actions.shape[0], actions.shape[1]
        out = _Output()
        fn = self.lib.jepa_ac_predict_all if all_frames else self.lib.jepa_ac_predict
        self._check(fn(self.ctx, capi.fptr(context), T, B, capi.fptr(actions), capi.fptr(states), C.byref(out)),
                    "jepa_ac_predict")
        try:
            n = out.n_tokens * out.dim
            res = np.ctypeslib.as_array(out.data, shape=(n,)).copy()
        finally:
            self.lib.jepa_free(C.cast(out.data, C.c_void_p))
        return res.reshape(B, -1, out.dim)

    def rollout(self, context, n_seed, seed_states, actions, states=None, seed_actions=None) -> np.ndarray:
        """context [n_seed HW, E]; actions [K, H, A] -> [K, H, HW, E] (jepa_ac_rollout_ex)."""
        context, seed_states, actions = _f32(context), _f32(seed_states), _f32(actions)
        states, seed_actions = _f32(states), _f32(seed_actions)
        K, H = actions.shape[0], actions.shape[1]
        E = context.shape[-1]
        out = np.zeros((K, H, self.HW, E), np.float32)
        self._check(self.lib.jepa_ac_rollout_ex(self.ctx, capi.fptr(context), n_seed, capi.fptr(seed_actions),
                                                capi.fptr(seed_states), capi.fptr(actions), capi.fptr(states), K, H,
                                                capi.fptr(out)), "jepa_ac_rollout_ex")
        return out

    def context_new(self, latents, n_frames, actions, states) -> int:
        latents, actions, states = _f32(latents), _f32(actions), _f32(states)
        h = self.lib.jepa_ac_context_new(self.ctx, capi.fptr(latents), n_frames, capi.fptr(actions), capi.fptr(states))
        if not h:
            raise RuntimeError(f"jepa_ac_context_new failed: {jlib.error_text()}")
        self.handles.append(h)
        return h

    def context_free(self, h: int) -> None:
        self.lib.jepa_ac_context_free(C.c_void_p(h))
        self.handles.remove(h)

    def context_update(self, h, latents, action, state) -> None:
        latents, action, state = _f32(latents), _f32(action), _f32(state)
        self._check(self.lib.jepa_ac_context_update(C.c_void_p(h), capi.fptr(latents), capi.fptr(action), capi.fptr(state)),
                    "jepa_ac_context_update")

    def context_trim(self, h, n_keep) -> None:
        self._check(self.lib.jepa_ac_context_trim(C.c_void_p(h), n_keep), "jepa_ac_context_trim")

    def rollout_cached(self, h, actions, states=None, E: int = 0) -> np.ndarray:
        actions, states = _f32(actions), _f32(states)
        K, H = actions.shape[0], actions.shape[1]
        out = np.zeros((K, H, self.HW, E), np.float32)
        self._check(self.lib.jepa_ac_rollout_cached(self.ctx, C.c_void_p(h), capi.fptr(actions), capi.fptr(states), K, H,
                                                    capi.fptr(out)), "jepa_ac_rollout_cached")
        return out

    def cem_params(self, **kw) -> capi.CemParams:
        p = self.lib.jepa_ac_cem_default_params()
        for k, v in kw.items():
            setattr(p, k, v)
        return p

    def plan(self, h, goal, params: capi.CemParams, noise=None):
        goal, noise = _f32(goal), _f32(noise)
        out = np.zeros((params.horizon, self.A), np.float32)
        energy = np.zeros(params.cem_steps, np.float32)
        self._check(self.lib.jepa_ac_plan(self.ctx, C.c_void_p(h), capi.fptr(goal), C.byref(params), capi.fptr(noise),
                                          capi.fptr(out), capi.fptr(energy)), "jepa_ac_plan")
        return out, energy
