"""Candidate sharding across GPUs (needs >= 2 CUDA devices; skipped otherwise): a 2-level plan whose
candidates are split over two processes / GPUs with the NCCL exchange per level returns exactly (bit for
bit) the plan of one GPU holding every candidate, because a candidate's arithmetic does not depend on the
batch it is in."""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _n_gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _plans():
    base = dict(pre_decay_horizon=0, lr=0.1, weight_decay=0.01, var_scale=1.0, action_noise=0.0, action_clip_sigma=0.0,
                min_its=3, early_stop_patience=2, early_stop_rel_delta=1e-2, intermediate_cost_weight=1.0,
                action_cost_weight=0.0, horizon_one_goal_upper=0)
    return [dict(base, horizon=4, n_samples=40, n_steps=8, cost_last_n=2, num_subgoals=1),
            dict(base, horizon=3, n_samples=40, n_steps=8, cost_last_n=1, num_subgoals=2)]


def _inputs():
    rng = np.random.default_rng(5)
    return ([rng.normal(size=64).astype(np.float32) for _ in range(2)], [rng.normal(size=64).astype(np.float32) for _ in range(2)],
            rng.normal(size=50000).astype(np.float32))


def _worker(rank, world, port, path, q):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "jepa.cpp_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from jepa_b200 import lib as jlib
    from jepa_b200.hjepa import Planner
    P = Planner(path, device=rank)
    uid = C.create_string_buffer(128)
    if rank == 0:
        assert jlib.load().jepa_b200_nccl_unique_id(uid) == 0
    obj = [bytes(uid.raw)] if rank == 0 else [None]
    dist.broadcast_object_list(obj, src=0)
    P.set_shard(rank, world, obj[0])
    states, goals, draws = _inputs()
    out, info, _ = P.plan(states, goals, _plans(), noise=draws)
    q.put((rank, out.tobytes(), list(info.iters)[:2], list(info.cost)[:2]))
    P.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
def test_sharded_plan_is_bit_identical(tmp_path):
    import sys
    import torch.multiprocessing as mp
    sys.path.insert(0, os.path.join(ROOT, "jepa.cpp_b200"))
    from jepa_b200 import synth
    from jepa_b200.hjepa import Planner
    path = str(tmp_path / "shard.gguf")
    L1 = synth.Level(64, 2, 2, 128, 2)
    L2 = synth.Level(64, 2, 2, 128, 4, stride=2, enc_kind="latent_mlp", act_enc_kind="mlp")
    synth.write_hjepa(path, synth.HJepaSpec(levels=[L1, L2], ftype="q8_0", rand_all=True, cond_std=0.3, w_std=0.1), seed=9)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 100
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r[0], r[1:]) for r in (q.get(timeout=600), q.get(timeout=600)))
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    states, goals, draws = _inputs()
    whole = Planner(path, device=0)
    out, info, _ = whole.plan(states, goals, _plans(), noise=draws)
    for r in (0, 1):
        assert res[r][0] == out.tobytes()
        assert res[r][1] == list(info.iters)[:2]


# ---------------------------------------------------------------------------------------------
# V-JEPA 2-AC CEM over two GPUs: each rank rolls out half the candidates, one NCCL all-gather of the
# energies per iteration; the plan and the per-iteration best energies equal the one-GPU plan bit for bit.
# ---------------------------------------------------------------------------------------------
def _ac_setup():
    rng = np.random.default_rng(8)
    HW, E = 16, 96
    lat = rng.normal(size=(2 * HW, E)).astype(np.float32)
    sa = rng.normal(0, 0.05, size=(1, 7)).astype(np.float32)
    ss = rng.normal(0, 0.3, size=(2, 7)).astype(np.float32)
    goal = rng.normal(size=(HW, E)).astype(np.float32)
    p = dict(samples=26, topk=5, cem_steps=3, horizon=2)
    noise = rng.normal(size=(p["cem_steps"], p["horizon"], p["samples"], 4)).astype(np.float32)
    return lat, sa, ss, goal, p, noise


def _ac_worker(rank, world, port, path, q):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "jepa.cpp_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from jepa_b200 import lib as jlib
    from jepa_b200.ac import ACWorldModel
    wm = ACWorldModel(path, device=rank)
    uid = C.create_string_buffer(128)
    if rank == 0:
        assert jlib.load().jepa_b200_nccl_unique_id(uid) == 0
    obj = [bytes(uid.raw)] if rank == 0 else [None]
    dist.broadcast_object_list(obj, src=0)
    wm.set_shard(rank, world, obj[0])
    lat, sa, ss, goal, p, noise = _ac_setup()
    h = wm.context_new(lat, 2, sa, ss)
    plan, best = wm.plan(h, goal, wm.cem_params(**p), noise=noise)
    q.put((rank, plan.tobytes(), best.tobytes()))
    wm.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_n_gpus() < 2, reason="needs 2 GPUs")
def test_sharded_cem_is_bit_identical(tmp_path):
    import sys
    import torch.multiprocessing as mp
    sys.path.insert(0, os.path.join(ROOT, "jepa.cpp_b200"))
    from jepa_b200 import synth
    from jepa_b200.ac import ACWorldModel
    path = str(tmp_path / "ac_shard.gguf")
    synth.write_ac(path, synth.ACSpec(enc_dim=96, pred_dim=64, n_layer=2, n_head=4, ffn_dim=128, grid=4, n_frames=4,
                                      ftype="q8_0", rand_all=True, w_std=0.1, name="ac-shard"), seed=12)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + os.getpid() % 90
    procs = [ctx.Process(target=_ac_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r[0], r[1:]) for r in (q.get(timeout=600), q.get(timeout=600)))
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    lat, sa, ss, goal, p, noise = _ac_setup()
    whole = ACWorldModel(path, device=0)
    h = whole.context_new(lat, 2, sa, ss)
    plan, best = whole.plan(h, goal, whole.cem_params(**p), noise=noise)
    for r in (0, 1):
        assert res[r][0] == plan.tobytes()
        assert res[r][1] == best.tobytes()
