"""Benchmark of the two planners on B200: H-JEPA plan grad-steps/s (headline) and V-JEPA 2-AC CEM
candidates/s, and the reference arm.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 5|1|2|3|4]

Headline workload (N = 1 and the scaling runs): BASELINE configs[4] ("config 5"), the largest H-JEPA
configuration, which fits one GPU -- a 4-level hierarchy, q8_0 GGUF, seeded random init (weights
N(0, 0.02), biases 0, LayerNorm gamma 1), every level's predictor 12 layers x 768 wide, 12 heads, MLP 3072,
horizons 64 / 16 / 8 / 4 from the bottom up, 4096 candidates. Start and goal latents N(0, 1); candidates
initialised U[-1, 1] through the jepa_randn_fn hook (prior mean 0, std 1, candidate 0 at the mean), as the
measurement rule maps the configs' prose onto the reference's planner. Early stopping off, weight decay 0.

A step is one Adam iteration of every level over all 4096 candidates. The timed region is ONE
jepa_hjepa_plan call with n_steps = K on every level (the warm-up: one call with n_steps = W): K steps,
plus each level's closing no-gradient evaluation and argmin, which are timed but not counted. The metric
unit, a grad-step, is one Adam iteration of one level (4 per step). With N GPUs the 4096 candidates are
split over the N ranks (strong scaling; one NCCL exchange per level); value = 4 K / (max over ranks of the
device time).

`value` is device time (CUDA events on the planner's stream around the call, weights resident); `e2e` is
the same call timed on the host, with host buffers in and out through the C ABI. The working set (weights
as f32 planes, activations of 2048-row chains) is far above the 126 MB L2, so no flush is needed between
timed iterations.

The reference arm runs the reference's own planner source (src/hjepa-plan.cpp, compiled unmodified against
the ggml shim, oracle/) on the host cores: each step is one gradient evaluation of one level, the levels in
rotation, over 8 candidates per host thread (the reference evaluates candidates 8 per thread), scaled to
the config's candidates.

The default run also measures the metric's second half, V-JEPA 2-AC CEM candidates/s (BASELINE
configs[3]), as the `ac_cem` object of the same line.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
# NCCL's communicator log (its INIT lines name the rank count) goes to a per-process file that is copied to
# stderr at exit, so that stdout holds exactly one JSON line
os.environ.setdefault("NCCL_DEBUG", "INFO")
os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
NCCL_LOG = os.path.join(tempfile.gettempdir(), f"jepa-bench-nccl.{os.getpid()}.log")
os.environ.setdefault("NCCL_DEBUG_FILE", NCCL_LOG)


def copy_nccl_log() -> None:
    try:
        with open(NCCL_LOG) as f:
            sys.stderr.write(f.read())
        os.unlink(NCCL_LOG)
    except OSError:
        pass
sys.path.insert(0, os.path.join(ROOT, "jepa.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from jepa_b200 import capi, synth  # noqa: E402

METRIC = "H-JEPA plan grad-steps/s & V-JEPA2-AC CEM candidates/s at 1/2/4/8 B200"
UNIT = "grad-steps/s"
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
DEFAULT_CONFIG = 5
# DRAM read + write of one k_gemm_tf32x3_p launch at 2048 x 3072 x 768 (ncu, dram__bytes_read.sum +
# dram__bytes_write.sum, one capture of that kernel at that shape): 31.5 MB read (the A and B hi / lo
# planes, once) + 0.3 MB written (the 25.2 MB output is still in L2 when the kernel ends)
GEMM_WIDE_TRAFFIC = 31.8e6
GEMM_WIDE_SHAPE = (2048, 3072, 768)


def row_step_flops(lv: synth.Level) -> float:
    """Forward GEMM FLOPs of one predictor row-step (adaLN 12P^2, V and out 2PI each, up and down 2PF each
    per layer, plus the action Linear), the measurement rule's per-unit figure."""
    P, I, F = lv.P(), lv.n_head * lv.hd(), lv.ffn_dim
    return lv.n_layer * (12 * P * P + 4 * P * I + 4 * P * F) + 2 * lv.E() * P


def plan_flops(spec: synth.HJepaSpec, plans: list, S: int) -> float:
    """Algorithmic FLOPs of one jepa_hjepa_plan: per level n_steps x (forward + backward-to-inputs) of
    S x T row-steps plus the final forward, plus the goal-projection encoders of the level below."""
    total = 0.0
    for k, (lv, p) in enumerate(zip(spec.levels, plans)):
        rows = S * p["horizon"]
        f = row_step_flops(lv)
        enc = 0.0
        if k + 1 < len(spec.levels):   # this level's predictions are encoded by the level above's encoder
            up = spec.levels[k + 1]
            n_enc = p["horizon"] // up.stride
            h = up.enc_hidden or up.embed_dim
            enc = S * n_enc * (2 * lv.embed_dim * h + 2 * h * up.embed_dim)
        total += p["n_steps"] * (2 * rows * f + 2 * enc) + rows * f + enc
    return total


def chains_for(S: int, width: int) -> int:
    """The planner's automatic candidate-chain count (HPlanner::streams_for, csrc/hplan.cpp)."""
    n = (2 if S >= 512 else 1) if width >= 768 else min(4, S // 256)
    return max(1, min(n, S, 8))


def gemm_roofline(L, lv, S_rank: int, reps: int = 20):
    """The planner's dominant kernel at the lowest level's per-step shapes, M = the rows of one candidate chain:
    the composed value/output product (M x P x P), up (M x F x P), down (M x P x F), and the adaLN modulation
    of one step (M x 6PL x P) with its transposed backward (M x P x 6PL). Each is timed live with CUDA events on
    its launch stream over `reps` back-to-back launches (jepa_b200_gemm_bench). Returns (TFLOP/s over the set,
    [(M, N, K, us per launch)])."""
    P = lv.pred_dim or lv.embed_dim
    M = S_rank // chains_for(S_rank, P)
    fn = L.jepa_b200_gemm_bench
    fn.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]
    fl = ms_tot = 0.0
    shapes = []
    for (N, K) in ((P, P), (lv.ffn_dim, P), (P, lv.ffn_dim), (6 * P * lv.n_layer, P), (P, 6 * P * lv.n_layer)):
        ms = C.c_double()
        if fn(M, N, K, reps, C.byref(ms)) != 0:
            return None, []
        fl += 2.0 * M * N * K
        ms_tot += ms.value
        shapes.append((M, N, K, round(ms.value * 1e3, 2)))
    return fl / (ms_tot / 1e3) / 1e12, shapes


def peaks(sustained: bool = False):
    try:
        with open(PEAKS_PATH) as f:
            d = json.load(f)
        tf = float(d["bf16_tflops_sustained"] if sustained else d["bf16_tflops"])
        return tf, float(d["hbm_gbs"]), "measured"
    except Exception:
        return (1400.0 if sustained else 1590.0), 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, gpu: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={gpu}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def model_path(cfg: int, rank: int, dist) -> tuple[str, synth.HJepaSpec, list]:
    """The config's synthetic GGUF (written once per box by rank 0, seed = config index)."""
    spec, plans = synth.hjepa_config(cfg)
    workdir = os.environ.get("JEPA_BENCH_DIR", tempfile.gettempdir())
    path = os.path.join(workdir, f"bench-cfg{cfg}.gguf")
    if rank == 0 and not os.path.exists(path):
        synth.write_hjepa(path + ".tmp", spec, seed=cfg)
        os.replace(path + ".tmp", path)
    if dist:
        dist.barrier()
    return path, spec, plans


def inputs(spec: synth.HJepaSpec, seed: int = 1):
    rng = np.random.default_rng(seed)
    states = [rng.normal(size=l.embed_dim).astype(np.float32) for l in spec.levels]
    goals = [rng.normal(size=l.embed_dim).astype(np.float32) for l in spec.levels]
    return states, goals


def uniform_draws(spec, plans, S):
    """U[-1, 1] values standing in for the candidates' initial perturbation (prior mean 0, std 1)."""
    n = sum((S - 1) * p["horizon"] * l.action_dim for l, p in zip(spec.levels, plans))
    return np.random.default_rng(7).uniform(-1.0, 1.0, n).astype(np.float32)


def strong_scaling(cfg: int) -> bool:
    return cfg == 5


def total_candidates(cfg: int, plans, world: int) -> int:
    """configs[4] (config 5) splits its candidates over the GPUs; the others plan their candidates per GPU."""
    S = plans[0]["n_samples"]
    return S if strong_scaling(cfg) else S * world


def hjepa_config_dict(cfg: int, spec, plans, world: int) -> dict:
    """The `config` object of the H-JEPA line, the same in both arms."""
    S = total_candidates(cfg, plans, world)
    lv = spec.levels[0]
    hz = "/".join(str(p["horizon"]) for p in plans)
    return {"workload": f"hjepa-config{cfg}: {len(spec.levels)}-level {spec.ftype}, D{lv.embed_dim} L{lv.n_layer} "
                        f"F{lv.ffn_dim}, horizons {hz}, {S} candidates in all",
            "levels": len(spec.levels), "candidates_total": S,
            "step": "one Adam iteration of every level over all candidates",
            "parallelism": f"candidates split over {world} GPU(s) ({'strong' if strong_scaling(cfg) else 'weak'} scaling)",
            "l2": "no flush: the working set (f32 weight planes, 2048-row activations) is far above L2"}


# ---------------------------------------------------------------------------------------------
# the reference planner on the host (oracle/_ref)
# ---------------------------------------------------------------------------------------------
class RefLevels:
    """One gradient evaluation of one level of the reference planner per call, the levels in rotation,
    over S candidates (actions U[-1, 1], the level above's states as goals, the top level's goal)."""

    def __init__(self, path, spec, plans, S, threads):
        import ref
        self.ok = ref.available()
        if not self.ok:
            return
        self.P = ref.RefPlanner(path, n_threads=threads)
        states, goals = inputs(spec)
        rng = np.random.default_rng(3)
        self.levels = []
        for k, (lv, p) in enumerate(zip(spec.levels, plans)):
            level = k + 1
            T, A = p["horizon"], lv.action_dim
            acts = rng.uniform(-1, 1, (S, T, A)).astype(np.float32)
            if level < len(spec.levels):
                up = spec.levels[level]
                n_goal = p["cost_last_n"]
                goal = rng.normal(size=(n_goal, up.embed_dim)).astype(np.float32)
                g = capi.Goal(capi.fptr(goal), n_goal, level + 1, 0, capi.fptr(None))
            else:
                goal = goals[k].reshape(1, -1)
                g = capi.Goal(capi.fptr(goal), 1, 0, 0, capi.fptr(None))
            lp = capi.LevelPlan.of(**p)
            self.levels.append((level, states[k], acts, goal, g, lp, np.zeros(S, np.float32), np.zeros_like(acts)))
        self.S = S
        self.turn = len(self.levels) - 1   # the cheapest level (the top) first

    def step(self) -> float:
        """Seconds of one gradient evaluation of the next level in the rotation."""
        level, s0, acts, goal, g, lp, costs, grad = self.levels[self.turn]
        self.turn = (self.turn - 1) % len(self.levels)
        t0 = time.perf_counter()
        rc = self.P.lib.jepa_hjepa_plan_cost(self.P.ctx, level, capi.fptr(s0), C.byref(g), C.byref(lp), capi.fptr(acts),
                                             self.S, acts.shape[1], capi.fptr(costs), capi.fptr(grad))
        assert rc == 0
        return time.perf_counter() - t0

    def close(self):
        if self.ok:
            self.P.close()


def ref_sample_rows(S_total: int, threads: int) -> int:
    """Candidates per reference evaluation: 8 per host thread (the reference hands each thread chunks of 8),
    at most the config's."""
    return max(1, min(S_total, 8 * threads))


def reference_rate(path, spec, plans, S_total, threads, steps, warmup):
    """(grad-steps/s of the config's S_total candidates, seconds measured, sample description) of the
    reference planner: `warmup` + `steps` evaluations in the level rotation, the timed ones summed; each
    evaluation counts as S / S_total of a grad-step."""
    S = ref_sample_rows(S_total, threads)
    R = RefLevels(path, spec, plans, S, threads)
    if not R.ok:
        return None, 0.0, ""
    for _ in range(warmup):
        R.step()
    secs = sum(R.step() for _ in range(steps))
    R.close()
    grad_steps = steps * S / S_total
    sample = (f"{steps} gradient evaluation(s) of one level each, the {len(plans)} levels in rotation, {S} candidates "
              f"per evaluation ({threads} threads x 8), counted as {S}/{S_total} of a grad-step each, after {warmup} "
              f"warm-up evaluation(s); reference src/hjepa-plan.cpp via oracle/_ref")
    return grad_steps / secs, secs, sample


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    if args.config == 4:
        # the reference's AC path is ggml CPU graph code that cannot be built here; its numpy restatement stands in
        spec = ac_spec()
        with tempfile.TemporaryDirectory() as tmp:
            path = os.path.join(os.environ.get("JEPA_BENCH_DIR", tmp), "bench-cfg4.gguf")
            if not os.path.exists(path):
                synth.write_ac(path, spec, seed=4)
            for _ in range(args.warmup):
                ac_cpu_port(path, spec)
            sec = sum(ac_cpu_port(path, spec) for _ in range(args.steps)) / max(args.steps, 1)
        value = 1.0 / sec
        sample = ("one candidate-iteration per step (one candidate through both horizon steps, each re-evaluating the "
                  "whole context, plus its energy), numpy restatement oracle/ac_oracle.py, f32, BLAS threads")
        print(json.dumps({"metric": METRIC, "unit": AC_UNIT, "impl": "reference", "higher_is_better": True,
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "dtype": "f32",
                          "data": "synthetic", "scaling": "strong", "value": value, "ms_per_step": sec * 1e3,
                          "config": ac_config_dict(spec, world),
                          "cpu_baseline": {"value": value, "unit": AC_UNIT, "cores": threads, "kind": "port",
                                           "sample": sample},
                          "e2e": {"value": value, "unit": AC_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                          "vs_baseline": None}))
        return
    path, spec, plans = model_path(args.config, 0, None)
    S_total = total_candidates(args.config, plans, world)
    base = {"metric": METRIC, "unit": UNIT, "impl": "reference", "higher_is_better": True, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "dtype": "f32", "data": "synthetic",
            "scaling": "strong" if strong_scaling(args.config) else "weak",
            "config": hjepa_config_dict(args.config, spec, plans, world)}
    value, secs, sample = reference_rate(path, spec, plans, S_total, threads, args.steps, args.warmup)
    if value is None:
        base["unavailable"] = "oracle/_ref/libhjepa_ref.so is not built (needs the reference tree at build time)"
        print(json.dumps(base))
        return
    # one bench step is one Adam iteration of every level: len(plans) grad-steps
    ms_per_step = len(plans) / value * 1e3
    base.update({"value": value, "ms_per_step": ms_per_step,
                 "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample},
                 "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                 "vs_baseline": None})
    print(json.dumps(base))


# ---------------------------------------------------------------------------------------------
# V-JEPA 2-AC CEM
# ---------------------------------------------------------------------------------------------
AC_UNIT = "CEM candidates/s"
AC_K, AC_H, AC_ITERS, AC_TOPK, AC_SEED_FRAMES = 800, 2, 10, 10, 2
# DRAM read + write per k_gemm_f16 launch at the benchmark's rows: ncu capture at M = 33,024 rows, scaled
# by rows to the 206,400 of the plan's passes (every operand but the weights grows with M)
AC_GEMM_TRAFFIC = 2.06e9


def ac_spec() -> synth.ACSpec:
    """24 layers x 1024, 16 heads, MLP 4096, 16 x 16 patches of 1408-d ViT-g latents, 7-d actions / poses,
    q8_0, weights N(0, 0.02), biases 0, LayerNorm gamma 1."""
    return synth.ACSpec(enc_dim=1408, pred_dim=1024, n_layer=24, n_head=16, ffn_dim=4096, grid=16, n_frames=4,
                        ftype="q8_0", name="bench-vjepa2-ac")


def ac_config_dict(spec, world: int) -> dict:
    return {"workload": f"vjepa2-ac-config4: CEM {AC_K} samples in all x {AC_ITERS} iterations, horizon {AC_H}, "
                        f"top-{AC_TOPK}, {AC_SEED_FRAMES} observed frames x 256 x 1408, predictor 24 x 1024 "
                        f"(16 heads, MLP 4096), q8_0",
            "candidates_total": AC_K,
            "parallelism": f"candidates split over {world} GPU(s) (strong scaling), one NCCL all-gather of energies "
                           f"per CEM iteration",
            "l2": "no flush: the working set (keys / values 40 GB, activations 4 GB at one GPU) is far above L2"}


def ac_inputs(spec: synth.ACSpec, K: int):
    rng = np.random.default_rng(4)
    HW = spec.grid * spec.grid
    latents = rng.normal(size=(AC_SEED_FRAMES * HW, spec.enc_dim)).astype(np.float32)
    seed_action = rng.normal(0, 0.05, size=(AC_SEED_FRAMES - 1, spec.action_dim)).astype(np.float32)
    states = rng.normal(0, 0.3, size=(AC_SEED_FRAMES, spec.state_dim)).astype(np.float32)
    goal = rng.normal(size=(HW, spec.enc_dim)).astype(np.float32)
    noise = np.random.default_rng(4).standard_normal((AC_ITERS, AC_H, K, 4)).astype(np.float32)
    return latents, seed_action, states, goal, noise


def ac_flops(spec: synth.ACSpec):
    """Per candidate-iteration: (algorithmic GFLOP as the reference evaluates it -- every step re-runs the
    whole context, block-causal attention, shared frames embedded once -- , GFLOP this engine executes --
    only each step's new frame, keys / values of earlier frames cached, the shared frame once per plan)."""
    D, F, L, HW, E = spec.pred_dim, spec.ffn_dim, spec.n_layer, spec.grid ** 2, spec.enc_dim
    R = HW + 2
    per_row = 2 * (4 * D * D + 2 * F * D) * L
    alg = ex = 0.0
    for s in range(AC_H):
        T = AC_SEED_FRAMES + s
        alg += T * R * per_row + 4 * D * R * R * T * (T + 1) / 2 * L + 2 * HW * E * D * s + 2 * HW * D * E
        ex += R * per_row + 4 * D * R * (T * R) * L + (2 * HW * E * D if s > 0 else 0) + 2 * HW * D * E
    return alg / 1e9, ex / 1e9


def ac_cpu_port(path, spec):
    """The numpy restatement (oracle/ac_oracle.py) of the reference's rollout, the way the reference runs
    it: one candidate carried through both horizon steps, each step re-evaluating the whole context
    (predict_all over T = 2 then 3 frames), then its L1 energy. Returns seconds per candidate-iteration."""
    import ac_oracle
    m = ac_oracle.ACModel(path)
    latents, seed_action, states, goal, _ = ac_inputs(spec, 1)
    acts = np.random.default_rng(5).normal(0, 0.02, size=(1, AC_H, spec.action_dim)).astype(np.float32)
    t0 = time.perf_counter()
    roll = ac_oracle.rollout(m, latents, AC_SEED_FRAMES, seed_action, states, acts)
    ac_oracle.energy(roll[:, -1], goal)
    return time.perf_counter() - t0


def kernel_profile(L, call, last_ms):
    """Run `call` once with the library's per-kernel event timing on; returns ({kind: {n, ms, flops, bytes}},
    the call's device ms)."""
    L.jepa_b200_kprof_begin.restype = None
    L.jepa_b200_kprof_end.argtypes = [C.c_char_p, C.c_size_t]
    L.jepa_b200_kprof_end.restype = C.c_int
    L.jepa_b200_kprof_begin()
    call()
    total = last_ms()
    buf = C.create_string_buffer(1 << 16)
    L.jepa_b200_kprof_end(buf, len(buf))
    kinds = {}
    for line in buf.value.decode().splitlines():
        k, n, ms, fl, by = line.split()
        kinds[k] = {"n": int(n), "ms": float(ms), "flops": float(fl), "bytes": float(by)}
    return kinds, total


def nccl_id(rank, dist):
    from jepa_b200 import lib as jlib
    uid = C.create_string_buffer(128)
    if rank == 0:
        assert jlib.load().jepa_b200_nccl_unique_id(uid) == 0
    obj = [bytes(uid.raw)] if rank == 0 else [None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def run_ac(args, rank, world, local, dist, primary: bool):
    from jepa_b200.ac import ACWorldModel
    from jepa_b200 import lib as jlib
    import torch
    spec = ac_spec()
    workdir = os.environ.get("JEPA_BENCH_DIR", tempfile.gettempdir())
    path = os.path.join(workdir, "bench-cfg4.gguf")
    if rank == 0 and not os.path.exists(path):
        synth.write_ac(path + ".tmp", spec, seed=4)
        os.replace(path + ".tmp", path)
    if dist:
        dist.barrier()
    K = AC_K                       # in all: each rank rolls out ceil(K / world) of them
    latents, seed_action, states, goal, noise = ac_inputs(spec, K)
    wm = ACWorldModel(path, device=local)
    if world > 1:
        wm.set_shard(rank, world, nccl_id(rank, dist))
    h = wm.context_new(latents, AC_SEED_FRAMES, seed_action, states)
    params = wm.cem_params(samples=K, topk=AC_TOPK, cem_steps=AC_ITERS, horizon=AC_H)
    L = jlib.load()
    for _ in range(max(3, args.warmup)):
        wm.plan(h, goal, params, noise=noise)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local)
    dev_ms, wall, launches = 0.0, 0.0, 0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        out, energy = wm.plan(h, goal, params, noise=noise)
        wall += time.perf_counter() - t0
        dev_ms += wm.last_ms()
        launches += L.jepa_b200_last_plan_launches(C.c_void_p(wm.ctx))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = clk.stop()
    # per-kernel device times: one more plan with every instrumented launch bracketed by CUDA events
    kinds, plan_ms_prof = kernel_profile(L, lambda: wm.plan(h, goal, params, noise=noise), wm.last_ms)
    t = torch.tensor([dev_ms, wall], dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, wall = float(t[0]), float(t[1])
    cands = K * AC_ITERS * args.steps
    value, e2e = cands / (dev_ms / 1e3), cands / wall
    alg, ex = ac_flops(spec)
    peak_tf, _, peak_kind = peaks(sustained=True)
    g = {"n": 0, "ms": 0.0, "flops": 0.0}
    for k, v in kinds.items():
        if k.startswith("gemm_f16"):
            g = {"n": g["n"] + v["n"], "ms": g["ms"] + v["ms"], "flops": g["flops"] + v["flops"]}
    gemm_tf = g["flops"] / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else None
    Kr = -(-K // world)
    n_seq = AC_SEED_FRAMES + AC_H - 1
    h2d = goal.nbytes + noise.nbytes + AC_ITERS * Kr * n_seq * (spec.action_dim + spec.state_dim) * 4
    d2h = AC_H * spec.action_dim * 4 + AC_ITERS * 4
    res = {
        "metric": METRIC, "value": value, "unit": AC_UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dev_ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (seeded random-init q8_0 GGUF, N(0,1) context / goal latents, N(0,1) CEM noise)",
        "config": ac_config_dict(spec, world),
        "arith": "f16 operands, f32 accumulate (tcgen05 kind::f16), f32 residual stream",
        "gflop_per_candidate_iteration": {"algorithmic": round(alg, 1), "executed": round(ex, 1)},
        "e2e": {"value": e2e, "unit": AC_UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "achieved": gemm_tf, "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": (gemm_tf / peak_tf) if gemm_tf else None, "traffic": AC_GEMM_TRAFFIC,
                     "traffic_note": "DRAM bytes per GEMM launch (mean of a layer's four), ncu at M = 33,024 rows scaled "
                                     "by rows to M = 206,400; algorithmic 2.34 GB",
                     "kernel": "k_gemm_f16 (tcgen05 kind::f16)",
                     "scope": f"2 M N K per launch / CUDA-event duration per launch, summed over the {g['n']} GEMM "
                              f"launches of one plan ({g['ms']:.1f} of {plan_ms_prof:.1f} ms)",
                     "peak_kind": f"bf16/f16 dense sustained, {peak_kind}",
                     "whole_plan_executed_tflops": ex * 1e9 * Kr * AC_ITERS / (plan_ms_prof / 1e3) / 1e12},
        "clocks": clocks,
        "kernels": {k: {"launches": v["n"], "ms": round(v["ms"], 3), "share": round(v["ms"] / plan_ms_prof, 4),
                        **({"tflops": round(v["flops"] / v["ms"] / 1e9, 1)} if v["flops"] else {}),
                        **({"gbs": round(v["bytes"] / v["ms"] / 1e6, 1)} if v["bytes"] else {})}
                    for k, v in sorted(kinds.items(), key=lambda kv: -kv[1]["ms"])},
    }
    if world == 1 and not args.no_cpu_baseline and rank == 0:
        try:
            ac_cpu_port(path, spec)                  # warm-up, as the reference arm takes
            sec = ac_cpu_port(path, spec)
            res["cpu_baseline"] = {"value": 1.0 / sec, "unit": AC_UNIT, "cores": os.cpu_count() or 1, "kind": "port",
                                   "sample": "one candidate-iteration (one candidate through both horizon steps, each "
                                             "re-evaluating the whole context as the reference does, plus its energy) "
                                             "with the numpy restatement oracle/ac_oracle.py (f32, BLAS threads), after "
                                             "one warm-up"}
        except Exception as e:
            res["cpu_baseline_error"] = str(e)
    wm.close()
    if rank == 0 and primary:
        print(json.dumps(res))
    return res


# ---------------------------------------------------------------------------------------------
# H-JEPA (headline)
# ---------------------------------------------------------------------------------------------
def run_hjepa(args, rank, world, local, dist):
    import torch
    from jepa_b200.hjepa import Planner
    from jepa_b200 import lib as jlib
    cfg = args.config
    path, spec, plans = model_path(cfg, rank, dist)
    S = total_candidates(cfg, plans, world)
    if S % world:
        raise SystemExit(f"{S} candidates do not split evenly over {world} GPUs")
    S_rank = S // world
    P = Planner(path, device=local)
    if world > 1:
        P.set_shard(rank, world, nccl_id(rank, dist))
    states, goals = inputs(spec)
    draws = uniform_draws(spec, plans, S)
    K, W = args.steps, max(3, args.warmup)

    def plan(n_steps):
        p = [dict(q, n_samples=S, n_steps=n_steps) for q in plans]
        t0 = time.perf_counter()
        P.plan(states, goals, p, noise=draws)
        return P.last_ms(), P.last_launches(), time.perf_counter() - t0

    plan(W)                                   # warm-up: W steps, workspaces built and graphs captured
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local)
    dev_ms, launches, wall = plan(K)          # the timed region: K steps in one call
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = clk.stop()
    t = torch.tensor([dev_ms, wall], dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, wall = float(t[0]), float(t[1])
    res = None
    if rank == 0:
        gemm_tf, shapes = gemm_roofline(jlib.load(), spec.levels[0], S_rank)
        grad_steps = len(plans) * K
        value = grad_steps / (dev_ms / 1e3)
        peak_tf, _, peak_kind = peaks()
        flops = plan_flops(spec, [dict(p, n_steps=K) for p in plans], S)
        achieved_tf = flops / (dev_ms / 1e3) / 1e12
        draws_bytes = draws.nbytes
        h2d = sum(l.embed_dim * 4 * 2 for l in spec.levels) + draws_bytes
        d2h = plans[0]["horizon"] * spec.levels[0].action_dim * 4 + \
            sum((p["horizon"] + 1) * l.embed_dim * 4 + p["horizon"] * l.action_dim * 4 + 8 for l, p in zip(spec.levels, plans))
        Mw, Nw, Kw = GEMM_WIDE_SHAPE
        res = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": dev_ms / K, "higher_is_better": True,
            "scaling": "strong" if strong_scaling(cfg) else "weak", "vs_baseline": None,
            "dtype": "f32", "data": f"synthetic (seeded random-init {spec.ftype} GGUF, N(0,1) latents, U[-1,1] candidates)",
            "config": hjepa_config_dict(cfg, spec, plans, world),
            "arith": "3xTF32 tensor-core GEMMs (tcgen05 kind::tf32, f32 accuracy), f32 element-wise",
            "e2e": {"value": grad_steps / wall, "unit": UNIT, "h2d_bytes_per_step": int(h2d / K),
                    "d2h_bytes_per_step": int(d2h / K)},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "achieved": gemm_tf, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": (gemm_tf / peak_tf) if gemm_tf else None,
                         "traffic": GEMM_WIDE_TRAFFIC * (shapes[1][0] / Mw) if shapes else None,
                         "traffic_note": f"DRAM read + write of one launch at {Mw} x {Nw} x {Kw} from an ncu capture of the "
                                         f"same kernel, scaled by rows to M = {shapes[1][0] if shapes else '?'} (the up "
                                         f"product); algorithmic {(4 * 2 * (Mw * Kw + Nw * Kw) + 4 * Mw * Nw) / 1e6:.1f} MB "
                                         f"at {Mw} rows",
                         "kernel": "k_gemm_tf32x3_p (tcgen05 kind::tf32, 3xTF32, persistent)",
                         "scope": "2 M N K / CUDA-event duration per launch at the lowest level's per-step shapes "
                                  "(M, N, K, us per launch): " + ", ".join(f"{m}x{n}x{k} {u}" for m, n, k, u in shapes),
                         "peak_kind": f"bf16 dense, {peak_kind}; the kernel runs tf32 (half the bf16 rate) three products "
                                      f"per output (hi x hi, hi x lo, lo x hi), so its own ceiling is 1/6 of this peak",
                         "whole_plan_tflops": achieved_tf, "whole_plan_frac": achieved_tf / (peak_tf * world),
                         "whole_plan_note": f"algorithmic FLOPs of the plan over all {world} GPU(s) / device time, "
                                            f"against {world} x the bf16 peak"},
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                threads = os.cpu_count() or 1
                # the reference arm's warm-up count, then one evaluation per level
                rate, secs, sample = reference_rate(path, spec, plans, S, threads, len(plans), max(1, args.warmup))
                if rate is not None:
                    res["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": threads, "kind": "reference",
                                           "sample": sample}
            except Exception as e:   # the baseline is reported, never required
                res["cpu_baseline_error"] = str(e)
    P.close()
    return res


def run_ours(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    torch.cuda.set_device(local)
    if args.config == 4:
        run_ac(args, rank, world, local, dist, primary=True)
    else:
        res = run_hjepa(args, rank, world, local, dist)
        if not args.no_ac:
            # the metric's second half: V-JEPA 2-AC CEM candidates/s on the same GPUs
            ac = run_ac(args, rank, world, local, dist, primary=False)
            if rank == 0:
                res["ac_cem"] = {k: ac[k] for k in ("value", "unit", "ms_per_step", "scaling", "dtype", "config", "e2e",
                                                     "gpu_launches", "roofline", "clocks", "cpu_baseline",
                                                     "cpu_baseline_error") if k in ac}
        if rank == 0:
            print(json.dumps(res))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=DEFAULT_CONFIG, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ac", action="store_true", help="skip the V-JEPA 2-AC CEM leg of an H-JEPA run")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)
        copy_nccl_log()


if __name__ == "__main__":
    main()
