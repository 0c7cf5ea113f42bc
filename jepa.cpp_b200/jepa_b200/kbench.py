"""Kernel microbenchmark: the planners' tcgen05 GEMMs at given shapes, through the C ABI.

    python -m jepa_b200.kbench M N K [reps] [--f16 | --blocks=q8_0|q4_0|f16 [--transposed]]
    python -m jepa_b200.kbench --attn n_cand n_frames rows heads hd [reps] [impl: 0 auto, 1 mma.sync, 2 tcgen05]
    python -m jepa_b200.kbench --ac samples cem_steps [model.gguf]
    python -m jepa_b200.kbench --hjepa config candidates [steps] [model.gguf]

Prints the mean device time per launch (CUDA events) and the algorithmic TFLOP/s (2 M N K per launch).
Without --f16 it times the H-JEPA planner's 3xTF32 GEMM, with --f16 the V-JEPA 2-AC predictor's f16 GEMM;
--blocks times the 3xTF32 GEMM with its weight operand in GGUF block planes dequantised in the mainloop (forward
B = W [N][K], or with --transposed the backward operand W^T of a weight [K][N]).
--attn times the AC predictor's attention (the last frame's rows over all frames' keys).
--ac runs one V-JEPA 2-AC CEM plan (horizon 2, two observed frames) on a model of the benchmark's size
(24 x 1024, 16 heads, MLP 4096, 16 x 16 patches of 1408-d latents, q8_0; written to the given path, or a
temporary file, when absent) with `samples` candidates: a small, self-contained case of the real kernels.
--hjepa solves level 1 of an H-JEPA benchmark configuration (1, 2, 3, 5: the bench's synthetic model) for
`steps` Adam iterations over `candidates` U[-1, 1] candidates -- every kernel of the level's iterations. Config
"w" is one level of config 5's width (768, 12 heads, MLP 3072, q8_0) with 2 layers and horizon 4: the same
per-launch shapes at a fraction of the memory, for profiler captures.
This module is part of the library's tooling: kernel timing in isolation, and a small, self-contained
target for ncu captures (the commands in profiles/ run it).
"""
from __future__ import annotations

import ctypes as C
import sys

from . import lib as jlib


def gemm(M: int, N: int, K: int, reps: int = 20, f16: bool = False) -> float:
    ms = C.c_double()
    L = jlib.load()
    fn = L.jepa_b200_gemm_f16_bench if f16 else L.jepa_b200_gemm_bench
    fn.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]
    if fn(M, N, K, reps, C.byref(ms)) != 0:
        raise RuntimeError(jlib.error_text())
    return ms.value


def gemm_blocks(M: int, N: int, K: int, ggml_type: int, transposed: bool, reps: int = 20) -> float:
    ms = C.c_double()
    L = jlib.load()
    L.jepa_b200_gemm_quant_bench.argtypes = [C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]
    if L.jepa_b200_gemm_quant_bench(ggml_type, M, N, K, int(transposed), reps, C.byref(ms)) != 0:
        raise RuntimeError(jlib.error_text())
    return ms.value


def attention(n_cand: int, n_frames: int, rows: int, heads: int, hd: int, reps: int = 20, impl: int = 0) -> float:
    ms = C.c_double()
    L = jlib.load()
    L.jepa_b200_attention_bench.argtypes = [C.c_int] * 7 + [C.POINTER(C.c_double)]
    if L.jepa_b200_attention_bench(n_cand, n_frames, rows, heads, hd, impl, reps, C.byref(ms)) != 0:
        raise RuntimeError(jlib.error_text())
    return ms.value


def ac_plan(samples: int, cem_steps: int, path: str = "") -> float:
    import os
    import tempfile

    import numpy as np

    from . import synth
    from .ac import ACWorldModel
    if not path:
        path = os.path.join(tempfile.gettempdir(), "kbench-ac.gguf")
    if not os.path.exists(path):
        synth.write_ac(path + ".tmp", synth.ACSpec(enc_dim=1408, pred_dim=1024, n_layer=24, n_head=16, ffn_dim=4096, grid=16,
                                                   n_frames=4, ftype="q8_0", name="kbench-ac"), seed=4)
        os.replace(path + ".tmp", path)
    rng = np.random.default_rng(4)
    wm = ACWorldModel(path)
    lat = rng.normal(size=(2 * wm.HW, 1408)).astype(np.float32)
    h = wm.context_new(lat, 2, rng.normal(0, 0.05, size=(1, 7)).astype(np.float32),
                       rng.normal(0, 0.3, size=(2, 7)).astype(np.float32))
    goal = rng.normal(size=(wm.HW, 1408)).astype(np.float32)
    params = wm.cem_params(samples=samples, topk=min(10, samples), cem_steps=cem_steps, horizon=2)
    noise = rng.standard_normal((cem_steps, 2, samples, 4)).astype(np.float32)
    wm.plan(h, goal, params, noise=noise)
    ms = wm.last_ms()
    wm.close()
    return ms


def hjepa_solve(cfg: str, S: int, steps: int = 2, path: str = "") -> float:
    import os
    import tempfile

    import numpy as np

    from . import synth
    from .hjepa import Planner
    if cfg == "w":
        spec = synth.HJepaSpec(levels=[synth.Level(768, 2, 12, 3072, 2)], ftype="q8_0", name="kbench-wide")
        plans = [dict(synth.hjepa_config(5)[1][0], horizon=4, cost_last_n=1)]
    else:
        spec, plans = synth.hjepa_config(int(cfg))
    seed = 99 if cfg == "w" else int(cfg)
    if not path:
        path = os.path.join(tempfile.gettempdir(), f"kbench-cfg{cfg}.gguf")
    if not os.path.exists(path):
        synth.write_hjepa(path + ".tmp", spec, seed=seed)
        os.replace(path + ".tmp", path)
    rng = np.random.default_rng(1)
    lv, p = spec.levels[0], plans[0]
    P = Planner(path, device=0)
    s0 = rng.normal(size=lv.embed_dim).astype(np.float32)
    acts = rng.uniform(-1, 1, (S, p["horizon"], lv.action_dim)).astype(np.float32)
    if len(spec.levels) > 1:
        goal = rng.normal(size=(p["cost_last_n"], spec.levels[1].embed_dim)).astype(np.float32)
        gl = 2
    else:
        goal = rng.normal(size=(1, lv.embed_dim)).astype(np.float32)
        gl = 0
    draws = rng.uniform(-1, 1, S * p["horizon"] * lv.action_dim).astype(np.float32)
    P.solve(1, s0, goal, dict(p, n_samples=S, n_steps=steps), noise=draws, goal_level=gl)
    ms = P.last_ms()
    P.close()
    return ms


if __name__ == "__main__":
    if "--hjepa" in sys.argv:
        a = [x for x in sys.argv[1:] if not x.startswith("--")]
        cfg, S = a[0], int(a[1])
        steps = int(a[2]) if len(a) > 2 else 2
        ms = hjepa_solve(cfg, S, steps, a[3] if len(a) > 3 else "")
        print(f"hjepa config {cfg} level-1 solve, {S} candidates, {steps} steps: {ms:.2f} ms")
        sys.exit(0)
    if "--ac" in sys.argv:
        a = [x for x in sys.argv[1:] if not x.startswith("--")]
        ms = ac_plan(int(a[0]), int(a[1]), a[2] if len(a) > 2 else "")
        print(f"ac plan samples={a[0]} cem_steps={a[1]}: {ms:.1f} ms")
        sys.exit(0)
    if "--attn" in sys.argv:
        a = [int(x) for x in sys.argv[1:] if not x.startswith("--")]
        nc, nf, rows, heads, hd = a[:5]
        reps = a[5] if len(a) > 5 else 20
        impl = a[6] if len(a) > 6 else 0
        t = attention(nc, nf, rows, heads, hd, reps, impl)
        fl = 4.0 * nc * heads * hd * rows * (nf * rows)
        print(f"attention[{impl}] cand={nc} frames={nf} rows={rows} heads={heads} hd={hd}: {t * 1e3:.2f} us/launch, "
              f"{fl / (t * 1e-3) / 1e12:.2f} TFLOP/s")
        sys.exit(0)
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    f16 = "--f16" in sys.argv
    M, N, K = (int(x) for x in args[:3])
    reps = int(args[3]) if len(args) > 3 else 20
    blk = [x.split("=", 1)[1] for x in sys.argv if x.startswith("--blocks=")]
    if blk:
        gt = {"q8_0": 8, "q4_0": 2, "f16": 1}[blk[0]]
        tr = "--transposed" in sys.argv
        t = gemm_blocks(M, N, K, gt, tr, reps)
        kind = f"3xtf32, B in {blk[0]} block planes{' (transposed)' if tr else ''}"
    else:
        t = gemm(M, N, K, reps, f16)
        kind = "f16" if f16 else "3xtf32"
    print(f"gemm[{kind}] M={M} N={N} K={K}: {t * 1e3:.2f} us/launch, {2.0 * M * N * K / (t * 1e-3) / 1e12:.2f} TFLOP/s")
