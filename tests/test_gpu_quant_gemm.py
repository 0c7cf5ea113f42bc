"""Weights dequantised inside the GEMM mainloop (GPU, through the C ABI).

The planner keeps each q8_0 / q4_0 / f16 linear in its block values (int8, 4-bit or f16 planes in both
orientations plus one f16 scale array). The GEMM's converter warps turn a TMA-staged raw tile into the split
operand in shared memory. The values are those of the reference's load-time dequantisation
(src/hjepa-plan.cpp:61-79 decodes every weight to f32 once; d * q is exact in f32, and so is its hi / lo split).
So the product must equal the same GEMM on the dequantised weight bit for bit:
- forward (C = A W^T) and transposed (C = A W, the backward product against the same weight);
- the 64-wide split-K cluster kernel (N or K below 768) and the persistent 128-wide kernel;
- the planner's K-split configuration.
The dequantised weight comes from gguf-py, the block formats' published decoder.
"""
import ctypes as C

import numpy as np
import pytest

from jepa_b200 import capi
from jepa_b200 import lib as jlib
from jepa_b200.gguf_write import quantize_q4_0, quantize_q8_0

pytestmark = pytest.mark.gpu

TYPES = {8: "q8_0", 2: "q4_0", 1: "f16"}


def _dequant(t, raw, rows, ne0):
    import gguf
    qt = {1: gguf.GGMLQuantizationType.F16, 2: gguf.GGMLQuantizationType.Q4_0, 8: gguf.GGMLQuantizationType.Q8_0}[t]
    return np.asarray(gguf.quants.dequantize(np.frombuffer(raw, np.uint8).reshape(rows, -1), qt), np.float32).reshape(rows, ne0)


def _lib():
    L = jlib.load()
    L.jepa_b200_gemm_quant.argtypes = [C.c_uint32, C.c_void_p, C.c_int, C.c_int, C.c_int, capi.FP, C.c_int, capi.FP, C.c_int]
    L.jepa_b200_gemm_ksplit.argtypes = [capi.FP, capi.FP, C.c_int, C.c_int, C.c_int, capi.FP]
    return L


def _weight(t, rows, ne0, seed):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.05, (rows, ne0)).astype(np.float32)
    raw = {1: w.astype(np.float16).tobytes(), 2: quantize_q4_0(w), 8: quantize_q8_0(w)}[t]
    return raw, _dequant(t, raw, rows, ne0)


# (rows, ne0, M): W [rows][ne0]. Forward N = rows, K = ne0; transposed N = ne0, K = rows.
SHAPES = [
    (384, 384, 256),     # config 2's value/output: 64-wide split-K clusters both ways
    (1536, 384, 200),    # config 2's up (transposed: its backward, K = 1536), ragged M
    (768, 768, 300),     # config 5's widths: persistent kernel, ragged M
    (3072, 768, 256),    # up (N = 3072) / its transposed backward (K = 3072: K split in the planner's configuration)
    (768, 3072, 130),    # down / its transposed backward (N = 3072)
    (4608, 768, 128),    # one layer's adaLN modulation rows (N >= 4096)
]


@pytest.mark.parametrize("t", sorted(TYPES))
@pytest.mark.parametrize("rows,ne0,M", SHAPES)
@pytest.mark.parametrize("transposed", [0, 1])
def test_block_plane_gemm_equals_dequantised_product(t, rows, ne0, M, transposed):
    L = _lib()
    raw, w = _weight(t, rows, ne0, seed=rows * 7 + ne0 + t)
    K = rows if transposed else ne0
    N = ne0 if transposed else rows
    Bm = np.ascontiguousarray(w.T if transposed else w)       # B [N][K]
    A = np.random.default_rng(M + K).normal(size=(M, K)).astype(np.float32)
    buf = C.create_string_buffer(raw, len(raw))
    for ksplit in (0, 1):
        got = np.zeros((M, N), np.float32)
        want = np.zeros((M, N), np.float32)
        assert L.jepa_b200_gemm_quant(t, buf, rows, ne0, transposed, capi.fptr(A), M, capi.fptr(got), ksplit) == 0, \
            jlib.error_text()
        f = L.jepa_b200_gemm_ksplit if ksplit else L.jepa_b200_gemm
        assert f(capi.fptr(A), capi.fptr(Bm), M, N, K, capi.fptr(want)) == 0, jlib.error_text()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
            (TYPES[t], transposed, ksplit, float(np.abs(got - want).max()))
    ref = A.astype(np.float64) @ Bm.astype(np.float64).T
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err


def test_block_planes_refuse_partial_blocks():
    """A weight whose sides are not whole 32-value blocks is refused with a message, not read."""
    L = _lib()
    raw, _ = _weight(8, 40, 64, seed=1)
    A = np.zeros((4, 64), np.float32)
    out = np.zeros((4, 40), np.float32)
    buf = C.create_string_buffer(raw, len(raw))
    jlib.load().jepa_error_reset()
    assert L.jepa_b200_gemm_quant(8, buf, 40, 64, 0, capi.fptr(A), 4, capi.fptr(out), 0) == -1
    assert "block" in jlib.error_text()


@pytest.mark.parametrize("ftype", ["q8_0", "q4_0", "f16"])
@pytest.mark.parametrize("width,ffn,heads", [(384, 1536, 6), (768, 3072, 12)])
def test_planner_weight_layouts_give_the_same_bits(tmp_path, monkeypatch, ftype, width, ffn, heads):
    """The planner with its linears in hi / lo planes, in block planes everywhere, and in the default layout
    (planes unless they would crowd the device's memory) returns identical costs and action gradients."""
    from jepa_b200 import synth
    from jepa_b200.hjepa import Planner
    spec = synth.HJepaSpec(levels=[synth.Level(width, 2, heads, ffn, 2)], ftype=ftype, name="layouts")
    path = str(tmp_path / f"layouts-{ftype}-{width}.gguf")
    synth.write_hjepa(path, spec, seed=width + len(ftype))
    rng = np.random.default_rng(width)
    s0 = rng.normal(size=width).astype(np.float32)
    goal = rng.normal(size=(1, width)).astype(np.float32)
    acts = rng.uniform(-1, 1, (64, 3, 2)).astype(np.float32)
    out = {}
    for layout in ("planes", "blocks", "auto"):
        monkeypatch.setenv("JEPA_B200_WEIGHT_LAYOUT", layout)
        P = Planner(path, device=0)
        out[layout] = P.plan_cost(1, s0, goal, acts, goal_level=1, plan=dict(cost_last_n=1))
        P.close()
    for layout in ("blocks", "auto"):
        for a, b in zip(out[layout], out["planes"]):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (layout, float(np.abs(a - b).max()))
