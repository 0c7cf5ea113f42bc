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
