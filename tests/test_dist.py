"""The candidate-sharding protocol of the planners on CPU: two gloo ranks, the oracle standing in for
each rank's GPU slice.

The engine gives rank r of W the candidates [r S / W, (r + 1) S / W) of every level (hplan_api.cpp),
evaluates them locally and exchanges only (min cost, global index) pairs; the lowest cost wins, the lowest
global index on ties (std::min_element over the whole batch, reference: src/hjepa-plan.cpp:952). This
test runs that exchange over torch.distributed (gloo, world size 2) and checks it picks exactly the
candidate the unsharded evaluation picks, including on a planted tie.
"""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _slice(S, rank, world):
    return S * rank // world, S * (rank + 1) // world


def _pick(pairs):
    best = None
    for c, i in pairs:
        if best is None or c < best[0] or (c == best[0] and i < best[1]):
            best = (c, i)
    return best


def _worker(rank, world, port, path, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "oracle"))
    sys.path.insert(0, os.path.join(root, "jepa.cpp_b200"))
    import hjepa_oracle as O
    m = O.Model(path)
    rng = np.random.default_rng(0)
    S, T = 10, 3
    acts = rng.uniform(-1, 1, (S, T, 2)).astype(np.float32)
    acts[7] = acts[2]                                    # a planted tie across the two ranks
    s0 = rng.normal(size=64).astype(np.float32)
    goal = rng.normal(size=(1, 64)).astype(np.float32)
    cs = O.CostSpec(level=1, horizon=T, s0=s0, goal=goal)
    r0, r1 = _slice(S, rank, world)
    costs, _, _ = O.batch_cost(m, cs, acts[r0:r1], want_grad=False)
    i = int(np.argmin(costs))
    mine = torch.tensor([float(costs[i]), float(r0 + i)], dtype=torch.float64)
    allp = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(allp, mine)
    got = _pick([(float(p[0]), int(p[1])) for p in allp])
    full, _, _ = O.batch_cost(m, cs, acts, want_grad=False)
    # the tie: make candidate 2 and 7 the joint best by construction of the check
    full_pick = int(np.argmin(full))
    if rank == 0:
        out.put((got[1], full_pick, float(full[2]), float(full[7])))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_argmin_matches_unsharded(tmp_path):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "jepa.cpp_b200"))
    from jepa_b200 import synth
    path = str(tmp_path / "dist.gguf")
    synth.write_hjepa(path, synth.HJepaSpec(levels=[synth.Level(64, 2, 2, 128, 2)], rand_all=True, cond_std=0.3, w_std=0.1), seed=3)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=300)
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    got, full_pick, c2, c7 = res
    assert c2 == c7                       # identical candidates cost the same bits
    assert got == full_pick               # the sharded exchange picks what the whole batch picks


def test_partition_covers_every_candidate():
    for S in (1, 7, 256, 4096, 1000):
        for W in (1, 2, 3, 4, 8):
            parts = [_slice(S, r, W) for r in range(W)]
            assert parts[0][0] == 0 and parts[-1][1] == S
            assert all(parts[i][1] == parts[i + 1][0] for i in range(W - 1))


# ---------------------------------------------------------------------------------------------
# V-JEPA 2-AC CEM: each rank scores a contiguous slice of the K candidates; one all-gather of the
# energies (slices padded to ceil(K / W)) gives every rank the same sorted elites and the same refit
# (ac_engine.cpp, jepa_ac_plan). The energies here come from a fixed nonlinear map of the actions.
# ---------------------------------------------------------------------------------------------
def _cem_params(K):
    return dict(samples=K, topk=5, cem_steps=4, horizon=2, maxnorm=0.05, gripper_clamp=0.75, momentum_mean=0.25,
                momentum_std=0.95, momentum_mean_gripper=0.15, momentum_std_gripper=0.15, round_gripper=0.25)


def _cem_energy(acts):
    w = np.linspace(-1.0, 1.0, acts.shape[1] * acts.shape[2]).astype(np.float32)
    flat = acts.reshape(acts.shape[0], -1)
    return np.abs(np.sin(7.0 * flat) + flat * w).sum(1).astype(np.float32)


def _cem_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import ac_oracle as O
    K = 23                                              # not a multiple of the world size
    Kr = (K + world - 1) // world
    lo, hi = min(K, rank * Kr), min(K, rank * Kr + Kr)

    def sharded(acts):
        local = np.full(Kr, np.inf, np.float32)
        local[:hi - lo] = _cem_energy(acts[lo:hi])
        parts = [torch.zeros(Kr, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(local))
        e = np.zeros(K, np.float32)
        for r in range(world):
            rl, rh = min(K, r * Kr), min(K, r * Kr + Kr)
            e[rl:rh] = parts[r].numpy()[:rh - rl]
        return e

    p = _cem_params(K)
    noise = np.random.default_rng(3).normal(size=(p["cem_steps"], p["horizon"], K, 4)).astype(np.float32)
    plan, best, elites = O.cem(None, None, 1, None, None, None, p, noise, A=7, energy_fn=sharded)
    ref, ref_best, ref_elites = O.cem(None, None, 1, None, None, None, p, noise, A=7, energy_fn=_cem_energy)
    out.put((rank, plan.tobytes() == ref.tobytes(), best.tobytes() == ref_best.tobytes(),
             all(np.array_equal(a, b) for a, b in zip(elites, ref_elites))))
    dist.barrier()
    dist.destroy_process_group()


def test_cem_energy_allgather_protocol():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 97
    procs = [ctx.Process(target=_cem_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same_plan, same_best, same_elites in res:
        assert same_plan and same_best and same_elites, rank
