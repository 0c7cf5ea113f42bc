"""Loads the engine's shared library (jepa.cpp_b200/lib/libjepa.so) through ctypes.

There is no fallback: when the library is missing or cannot be loaded, the import fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os

from . import capi

LIB_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "lib", "libjepa.so")

_lib = None


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} is not built: run python jepa.cpp_b200/build.py (or __graft_entry__.build())")
    lib = C.CDLL(LIB_PATH)
    capi.declare_planner(lib)
    vp, FP = C.c_void_p, capi.FP
    decl = {
        "jepa_b200_version": (C.c_char_p, []),
        "jepa_b200_gemm": (C.c_int, [FP, FP, C.c_int, C.c_int, C.c_int, FP]),
        "jepa_b200_gemm_bench": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]),
        "jepa_b200_dequant": (C.c_int, [C.c_uint32, vp, C.c_int64, C.c_int64, FP]),
        "jepa_error_reset": (None, []),
        "jepa_error_text": (C.c_char_p, []),
    }
    optional = {
        "jepa_model_load": (vp, [C.c_char_p, C.c_bool]),
        "jepa_model_free": (None, [vp]),
        "jepa_context_default_params": (None, []),
        "jepa_context_free": (None, [vp]),
        "jepa_b200_nccl_unique_id": (C.c_int, [vp]),
        "jepa_b200_context_set_shard": (C.c_int, [vp, C.c_int, C.c_int, vp]),
        "jepa_b200_last_plan_ms": (C.c_double, [vp]),
        "jepa_b200_hjepa_set_streams": (C.c_int, [vp, C.c_int]),
        "jepa_b200_hjepa_set_step_modulation": (C.c_int, [vp, C.c_int]),
        "jepa_b200_last_plan_launches": (C.c_longlong, [vp]),
        "jepa_b200_context_new": (vp, [vp, C.c_int]),
    }
    for name, (res, args) in list(decl.items()) + list(optional.items()):
        if hasattr(lib, name):
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        elif name in decl:
            raise OSError(f"{LIB_PATH} does not export {name}")
    _lib = lib
    return lib


def error_text() -> str:
    return (load().jepa_error_text() or b"").decode(errors="replace")
