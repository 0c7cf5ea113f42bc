"""The drop-in boundary, checked without a GPU: the library loads, exports every function that
include/jepa.h and include/jepa_b200.h declare (the reference's Python binding resolves every one of
them at import, reference: python/src/jepa_cpp/_api.py:413-418), and the structs keep the reference's
layout (sizeof(jepa_hjepa_plan_info) == 128, reference: python/tests/test_api_coverage.py:134)."""
import ctypes as C
import os
import re

from jepa_b200 import capi, lib as jlib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"//[^\n]*", "", src)
    return re.findall(r"\b(jepa_\w+)\s*\(", src)


def test_every_declared_function_is_exported():
    lib = jlib.load()
    names = set(declared("jepa.h")) | set(declared("jepa_b200.h"))
    names.discard("jepa_randn_fn")
    missing = sorted(n for n in names if not hasattr(lib, n))
    assert not missing, missing
    assert len(set(declared("jepa.h"))) >= 114


def test_reference_python_binding_probe():
    lib = jlib.load()
    lib.jepa_cpp_shared_abi.restype = C.c_char_p
    lib.jepa_version.restype = C.c_char_p
    assert lib.jepa_cpp_shared_abi() == lib.jepa_version()


def test_struct_layouts():
    assert C.sizeof(capi.PlanInfo) == 128
    assert C.sizeof(capi.LevelPlan) == 68
    assert C.sizeof(capi.Goal) == 32
    assert C.sizeof(capi.CemParams) == 48


def test_level_plan_defaults_match_reference():
    p = jlib.load().jepa_hjepa_level_plan_default()
    # src/hjepa-plan.cpp:1066-1086
    assert (p.horizon, p.n_samples, p.n_steps, p.min_its, p.early_stop_patience, p.cost_last_n, p.num_subgoals) == \
        (1, 100, 90, 30, 5, 1, 1)
    assert abs(p.lr - 0.1) < 1e-7 and abs(p.weight_decay - 0.01) < 1e-7 and abs(p.early_stop_rel_delta - 1e-2) < 1e-9


def test_error_text_capture():
    lib = jlib.load()
    lib.jepa_error_reset()
    assert lib.jepa_error_text() == b""
    lib.jepa_hjepa_plan_cost.restype = C.c_int
    assert lib.jepa_hjepa_plan_cost(None, 1, None, None, None, None, 1, 1, None, None) == -1
