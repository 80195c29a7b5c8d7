"""The N>1 path's semantics on CPU with world_size-2 gloo ranks.

The multi-GPU trainer (csrc/comm.cpp, csrc/ppo_host.cpp) shards environments by
rank with global env ids, allreduces the fp64 advantage sums for a global
normalisation (ppo.hpp:128-140), and forms global minibatch k from every rank's
chunk k with the loss scaled by 1/B_global (ppo.hpp:159). Here each gloo rank
runs a shard of the CPU oracle and the results are checked against one process
holding every environment:
  * rollouts of a shard equal the matching slice of the single-process rollout
    bit for bit (global env ids drive seeds and clean-env parity);
  * normalised advantages from allreduced fp64 statistics equal the
    single-process ones bit for bit;
  * the allreduced per-rank gradients of chunk k equal the gradient of the union
    of those rows within fp32 summation tolerance (1e-5 relative).
A rank that fails before a collective makes the job end with that rank's error
instead of hanging (process-group timeout).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_oracle_module, load_package

N_TOTAL, T, MB = 48, 8, 64


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))


def _shard_worker(rank, world, port):
    _init(rank, world, port)
    pkg, om = load_package(), load_oracle_module()
    L = pkg.layouts
    raptor = L.load_raptor_file(os.path.join(os.path.dirname(__file__), "golden", "raptor.bin"))
    n = N_TOTAL // world
    cfg = L.default_config(n=n, family=12, speed=1.0, distance=3.0, seed=7, sensor_delay=1, wind=0.3)
    shard = om.OracleSim(L, cfg, T, raptor, env_base=rank * n)
    full = om.OracleSim(L, L.default_config(n=N_TOTAL, family=12, speed=1.0, distance=3.0, seed=7, sensor_delay=1,
                                            wind=0.3), T, raptor)
    for t in range(T):
        shard.step(t)
        full.step(t)
    # 1) rollouts: shard == slice of the full rollout, bit for bit
    for name, width in (("obs", 184), ("rewards", 1), ("terminated", 1), ("next_values", 1)):
        mine = shard.buf(name).reshape(T, n, width)
        ref = full.buf(name).reshape(T, N_TOTAL, width)[:, rank * n:(rank + 1) * n]
        assert np.array_equal(mine, ref), (rank, name)
    # 2) global advantage normalisation from allreduced fp64 sums
    shard.gae(normalize=False)
    full.gae(normalize=True)
    adv = shard.buf("advantages")
    count = float(N_TOTAL * T)
    total = torch.tensor([np.sum(adv.astype(np.float64))], dtype=torch.float64)
    dist.all_reduce(total)
    mean = np.float32(total.item() / count)
    sq = torch.tensor([np.sum(((adv - mean).astype(np.float64)) ** 2)], dtype=torch.float64)
    dist.all_reduce(sq)
    inv = np.float32(1.0) / np.sqrt(np.float32(sq.item() / count) + np.float32(1e-8))
    normed = (adv - mean) * inv
    ref = full.buf("advantages").reshape(T, N_TOTAL)[:, rank * n:(rank + 1) * n].ravel()
    assert np.array_equal(normed.astype(np.float32), ref), rank
    # 3) global minibatch = union of the ranks' chunk k, loss scale 1/B_global
    shard.buf("advantages")[:] = normed
    begin = 64
    local_rows = np.arange(begin, begin + MB, dtype=np.uint32)
    grad = torch.from_numpy(shard.rows_grad(local_rows, MB * world).copy())
    dist.all_reduce(grad)
    if rank == 0:
        union = []
        for r in range(world):
            t_idx, i_idx = np.divmod(local_rows.astype(np.int64), n)
            union.append(t_idx * N_TOTAL + r * n + i_idx)
        g_full = full.rows_grad(np.concatenate(union), MB * world)
        g = grad.numpy()
        scale = np.abs(g_full).max()
        assert np.allclose(g, g_full, rtol=1e-5, atol=1e-6 * scale), float(np.abs(g - g_full).max() / scale)
    dist.barrier()
    dist.destroy_process_group()


def _failing_worker(rank, world, port):
    _init(rank, world, port)
    if rank == 1:
        raise RuntimeError("rank 1 fails before the collective")
    t = torch.ones(1)
    dist.all_reduce(t)  # never completes: rank 1 is gone


def test_two_gloo_ranks_match_one_process():
    mp.spawn(_shard_worker, args=(2, _free_port()), nprocs=2, join=True)


def test_failed_rank_ends_the_job():
    with pytest.raises(Exception) as info:
        mp.spawn(_failing_worker, args=(2, _free_port()), nprocs=2, join=True)
    assert "rank 1 fails" in str(info.value) or "ProcessRaisedException" in type(info.value).__name__ \
        or "process" in str(info.value).lower()


def _bank_worker(rank, world, port):
    """Challenge-bank sampler state stays identical on every rank when each
    rank contributes its environments' rollout evidence through
    gather_rollout_evidence (equal to one process observing all of it)."""
    _init(rank, world, port)
    import json
    pkg = load_package()
    bank = os.path.join(os.path.dirname(__file__), "golden", "challenge_bank_small.jsonl")
    h = json.loads(open(bank).readline())["world_source_sha256"]
    n_total, horizon = 12, 5
    n = n_total // world
    mine = pkg.ChallengeSampler(bank, h, environment_count=n_total, horizon=horizon, selection=1,
                                rehearsal_environments=2)
    solo = pkg.ChallengeSampler(bank, h, environment_count=n_total, horizon=horizon, selection=1,
                                rehearsal_environments=2)
    sched = mine.initial_schedule()
    assert np.array_equal(sched, solo.initial_schedule())
    active = sched[:, 0].copy()
    rng = np.random.default_rng(5)  # the same full evidence on every rank; each rank sends its slice
    for rollout in range(3):
        if rollout:
            sched = mine.next_schedule(active, rollout)
            assert np.array_equal(sched, solo.next_schedule(active, rollout))
        ids = np.zeros((horizon, n_total), np.uint32)
        term = np.zeros((horizon, n_total), np.uint8)
        for t in range(horizon):
            for e in range(n_total):
                ids[t, e] = active[e]
                if rng.random() < 0.4:
                    term[t, e] = 1
                    active[e] = sched[e, t + 1]
        gae = rng.normal(0, 1, (horizon, n_total)).astype(np.float32)
        trunc = np.zeros_like(term)
        cols = slice(rank * n, (rank + 1) * n)
        full = pkg.gather_rollout_evidence(gae[:, cols], term[:, cols], trunc[:, cols], ids[:, cols])
        assert all(np.array_equal(a, b) for a, b in zip(full, (gae, term, trunc, ids)))
        mine.observe_raw_gae(*full, rollout)
        solo.observe_raw_gae(gae, term, trunc, ids, rollout)
        for lvl in range(len(mine.bank)):
            assert mine.level_stats(lvl) == solo.level_stats(lvl)
    dist.destroy_process_group()


def test_bank_sampler_across_ranks():
    mp.spawn(_bank_worker, args=(2, _free_port()), nprocs=2, join=True)
