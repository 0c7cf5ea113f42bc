"""Test infrastructure: ctypes handle on the reference's own planner built by oracle/Makefile.

ORACLE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may
use this module, and only as the checker or the timed baseline -- never as the product path.

`_ref/libhjepa_ref.so` is src/hjepa-plan.cpp of the reference, compiled unmodified against the shim in
oracle/shim/; its entry points are the reference's jepa_hjepa_plan_cost / _solve / _plan / _horizons.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libhjepa_ref.so")
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "jepa.cpp_b200"))

from jepa_b200 import capi  # noqa: E402  (ABI struct definitions only)


def available() -> bool:
    return os.path.exists(LIB_PATH)


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"{LIB_PATH} is not built (make -C oracle with the reference tree present)")
        _lib = capi.declare_planner(C.CDLL(LIB_PATH))
        _lib.ref_model_load.restype = C.c_void_p
        _lib.ref_model_load.argtypes = [C.c_char_p]
        _lib.ref_model_free.argtypes = [C.c_void_p]
        _lib.ref_context_new.restype = C.c_void_p
        _lib.ref_context_new.argtypes = [C.c_void_p, C.c_int]
        _lib.ref_context_free.argtypes = [C.c_void_p]
    return _lib


class RefPlanner:
    """The reference planner over one GGUF file, with `n_threads` host threads."""

    def __init__(self, path: str, n_threads: int = 1):
        L = lib()
        self.model = L.ref_model_load(path.encode())
        if not self.model:
            raise RuntimeError(f"reference shim could not load {path}")
        self.ctx = L.ref_context_new(self.model, n_threads)
        self.lib = L

    def close(self) -> None:
        if self.ctx:
            self.lib.ref_context_free(self.ctx)
            self.lib.ref_model_free(self.model)
            self.ctx = self.model = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
