"""ctypes view of the planner block of the jepa.cpp C API (include/jepa.h).

Struct layouts mirror the reference header field for field (reference: include/jepa.h:286-362 for
the H-JEPA planner, :480-491 for the CEM parameters): the same `libjepa.so` ABI that the reference's
Python binding binds (python/src/jepa_cpp/_api.py:216-409), so one set of definitions serves both
this engine's library and the reference planner built as the oracle.
"""
from __future__ import annotations

import ctypes as C
import os

MAX_PLAN_LEVELS = 8


class LevelPlan(C.Structure):
    """jepa_hjepa_level_plan (include/jepa.h:286-310)."""
    _fields_ = [
        ("horizon", C.c_int), ("pre_decay_horizon", C.c_int), ("n_samples", C.c_int), ("n_steps", C.c_int),
        ("lr", C.c_float), ("weight_decay", C.c_float), ("var_scale", C.c_float), ("action_noise", C.c_float),
        ("action_clip_sigma", C.c_float), ("min_its", C.c_int), ("early_stop_patience", C.c_int),
        ("early_stop_rel_delta", C.c_float), ("cost_last_n", C.c_int), ("intermediate_cost_weight", C.c_float),
        ("action_cost_weight", C.c_float), ("num_subgoals", C.c_int), ("horizon_one_goal_upper", C.c_int),
    ]

    @classmethod
    def of(cls, **kw) -> "LevelPlan":
        p = cls()
        for k, v in kw.items():
            setattr(p, k, v)
        return p


class Goal(C.Structure):
    """jepa_hjepa_goal (include/jepa.h:320-328)."""
    _fields_ = [("states", C.POINTER(C.c_float)), ("n_states", C.c_int), ("level", C.c_int),
                ("dense", C.c_int), ("actions", C.POINTER(C.c_float))]


class PlanInfo(C.Structure):
    """jepa_hjepa_plan_info (include/jepa.h:357-362); sizeof == 128."""
    _fields_ = [("planned", C.c_int * MAX_PLAN_LEVELS), ("goal_level", C.c_int * MAX_PLAN_LEVELS),
                ("iters", C.c_int * MAX_PLAN_LEVELS), ("cost", C.c_float * MAX_PLAN_LEVELS)]


class CemParams(C.Structure):
    """jepa_ac_cem_params (include/jepa.h:480-491)."""
    _fields_ = [("samples", C.c_int), ("topk", C.c_int), ("cem_steps", C.c_int), ("horizon", C.c_int),
                ("maxnorm", C.c_float), ("gripper_clamp", C.c_float), ("momentum_mean", C.c_float),
                ("momentum_std", C.c_float), ("momentum_mean_gripper", C.c_float),
                ("momentum_std_gripper", C.c_float), ("round_gripper", C.c_float), ("seed", C.c_uint32)]


RANDN_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(C.c_float), C.c_size_t)
FP = C.POINTER(C.c_float)


def fptr(a) -> "C._Pointer":
    """Pointer to the data of a C-contiguous float32 numpy array (or NULL for None)."""
    if a is None:
        return C.cast(None, FP)
    assert a.dtype.name == "float32" and a.flags["C_CONTIGUOUS"], "need a C-contiguous float32 array"
    return a.ctypes.data_as(FP)


def declare_planner(lib: C.CDLL) -> C.CDLL:
    """Argument and return types of the H-JEPA planner entry points (include/jepa.h:313-373) that `lib` exports."""
    vp = C.c_void_p
    sigs = {
        "jepa_hjepa_level_plan_default": (LevelPlan, []),
        "jepa_hjepa_plan_cost": (C.c_int, [vp, C.c_int, FP, C.POINTER(Goal), C.POINTER(LevelPlan), FP, C.c_int,
                                           C.c_int, FP, FP]),
        "jepa_hjepa_solve": (C.c_int, [vp, C.c_int, FP, C.POINTER(Goal), C.POINTER(LevelPlan), RANDN_FN, vp,
                                       FP, FP, FP, C.POINTER(C.c_int)]),
        "jepa_hjepa_horizons": (C.c_int, [vp, C.POINTER(LevelPlan), C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.POINTER(C.c_int)]),
        "jepa_hjepa_plan": (C.c_int, [vp, C.POINTER(FP), C.POINTER(FP), C.POINTER(LevelPlan), C.c_int, RANDN_FN,
                                      vp, FP, C.POINTER(PlanInfo)]),
    }
    for name, (res, args) in sigs.items():
        if hasattr(lib, name):
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
    return lib


class Replay:
    """A jepa_randn_fn that hands back pre-recorded draws in order (reference: tests/test-predictor.cpp:183-194).

    Keep the object alive for the duration of the call: `fn` holds the ctypes callback.
    """

    def __init__(self, data):
        import numpy as np
        self.data = np.ascontiguousarray(data, dtype=np.float32).ravel()
        self.pos = 0
        self.overrun = False

        def _cb(user, out, n):
            k = min(n, self.data.size - self.pos)
            if k > 0:
                C.memmove(out, self.data[self.pos:self.pos + k].ctypes.data, 4 * k)
            if k < n:
                C.memset(C.addressof(out.contents) + 4 * k, 0, 4 * (n - k))
                self.overrun = True
            self.pos += k
        self.fn = RANDN_FN(_cb)

    def exact(self) -> bool:
        return not self.overrun and self.pos == self.data.size


def repo_root() -> str:
    return os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
