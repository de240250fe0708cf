"""Host-side logic of the data-parallel update, on CPU.

* pl_muon_shard_plan: which rank orthogonalises which matrix (every rank must derive the same plan).
* The decomposition the library implements with NCCL, run here as gloo ranks on the oracle (2 and 3
  ranks, uneven shares): each rank takes rows [n*r/R, n*(r+1)/R) of the one minibatch (the
  strong-scaling split), the advantage (sum, sum of squares, count) and the summed gradients are
  all-reduced, and the result equals the single-process minibatch of all rows.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import pufferlean_b200 as plb
from oracle import cpu_port


def shard_plan(rows, cols, world):
    L = plb.lib()
    n = len(rows)
    r = (C.c_size_t * n)(*rows)
    c = (C.c_size_t * n)(*cols)
    o = (C.c_int * n)()
    L.pl_muon_shard_plan.argtypes = [C.POINTER(C.c_size_t), C.POINTER(C.c_size_t), C.c_size_t, C.c_int,
                                     C.POINTER(C.c_int)]
    assert L.pl_muon_shard_plan(r, c, n, world, o) == 0
    return list(o)


C5_SHAPES = ([2048, 2048, 2048, 2048, 2048, 65], [1024, 2048, 2048, 2048, 2048, 2048])


def _cost(r, c):
    m, n = min(r, c), max(r, c)
    return 4 * m * m * n + 2 * m ** 3


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_plan_covers_every_matrix_and_balances(world):
    rows, cols = C5_SHAPES
    own = shard_plan(rows, cols, world)
    assert own == shard_plan(rows, cols, world)  # deterministic
    assert all(0 <= o < world for o in own)
    if world == 1:
        assert own == [0] * len(rows)
    load = [0] * world
    for o, r, c in zip(own, rows, cols):
        load[o] += _cost(r, c)
    used = [l for l in load if l > 0]
    biggest = max(_cost(r, c) for r, c in zip(rows, cols))
    assert max(used) - min(used) <= biggest  # LPT bound


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        D, H, A, L, act = 12, 32, 5, 2, 1
        g = np.random.default_rng(0)  # same data on every rank: the global minibatch
        n = 96
        lay, P = cpu_port.layers_of(D, H, A, L)
        params = g.uniform(-0.2, 0.2, P)
        obs = g.standard_normal((n, D))
        acts = g.integers(0, A, n).astype(float)
        adv = g.standard_normal(n) * 2 + 0.3
        ret = g.standard_normal(n)
        olp = np.log(np.full(n, 1 / A)) + 0.1 * g.standard_normal(n)
        mine = slice(rank * n // world, (rank + 1) * n // world)
        # global advantage statistics from the local (sum, sum of squares, count)
        sums = torch.tensor([adv[mine].sum(), (adv[mine] ** 2).sum(), float(adv[mine].size)], dtype=torch.float64)
        dist.all_reduce(sums)
        mean = sums[0].item() / sums[2].item()
        std = np.sqrt(max(sums[1].item() / sums[2].item() - mean * mean, 0.0))
        advn = (adv[mine] - mean) / (std + 1e-8)
        gl = cpu_port.ppo_grad(params, obs[mine], acts[mine], advn, ret[mine], olp[mine], D, H, A, L, act, ov=ret[mine],
                               vfclip=0.2)
        gt = torch.tensor(gl)
        dist.all_reduce(gt)
        plan = shard_plan([ly[2] for ly in lay], [ly[3] for ly in lay], world)
        plans = [None] * world
        dist.all_gather_object(plans, plan)
        if rank == 0:
            full_n = (adv - adv.mean()) / (adv.std() + 1e-8)
            ref = cpu_port.ppo_grad(params, obs, acts, full_n, ret, olp, D, H, A, L, act, ov=ret, vfclip=0.2)
            q.put((float(np.abs(gt.numpy() - ref).max()), float(np.abs(ref).max()), plans))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_data_parallel_decomposition_equals_full_minibatch_gloo(world):
    port = 29500 + os.getpid() % 1000 + 7 * world
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    err, scale, plans = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert err < 1e-10 * max(1.0, scale)
    assert plans[0] == plans[1]


# ---------------------------------------------------------------------------------------- MinGRU
def _mg_rank(rank, world, port, q):
    """One rank of the MinGRU decomposition on the oracle: its own rollout and sample, the advantage
    sum and squared-deviation sum all-reduced (two passes, as pl_mg_grad does), its own sequences'
    summed gradient all-reduced."""
    from oracle import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, T, D, H, L, A = 8, 5, 4, 8, 1, 3
        g = np.random.default_rng(90 + rank)
        adv = g.standard_normal(N * T)
        val, logp = g.standard_normal(N * T), g.uniform(-2, -0.5, N * T)
        act, term = g.integers(0, A, N * T).astype(float), (g.random(N * T) < 0.2) * 1.0
        obs = g.uniform(0, 1, N * T * D)
        seg = np.array([1.0, 6.0, 1.0]) if rank == 0 else np.array([0.0, 3.0, 7.0])
        mbp = np.array([1.0, 0.5, 1.5]) if rank == 0 else np.array([0.9, 1.1, 1.2])
        params, _ = O.init_mingru(D, H, L, A, 0x5151)
        Bmb = seg.size
        a_s = np.array([adv[int(e) * T + t] for e in seg for t in range(T)])
        tot = torch.tensor([a_s.sum()], dtype=torch.float64)
        dist.all_reduce(tot)
        mean = float(tot[0]) / (Bmb * T * world)
        sq = torch.tensor([((a_s - mean) ** 2).sum()], dtype=torch.float64)
        dist.all_reduce(sq)
        std = np.sqrt(float(sq[0]) / (Bmb * T * world))
        sc = O.gather_seq_minibatch(act, logp, term, adv, val, seg, mbp, T, Bmb)
        nb = T * Bmb
        for b in range(Bmb):  # re-normalise the advantage rows with the all-rank statistics
            e = int(seg[b])
            for t in range(T):
                sc[nb + t * Bmb + b] = mbp[b] * (adv[e * T + t] - mean) / (std + 1e-8)
        obsTB = np.zeros(nb * D)
        for t in range(T):
            for b in range(Bmb):
                e = int(seg[b])
                obsTB[(t * Bmb + b) * D:(t * Bmb + b + 1) * D] = obs[(e * T + t) * D:(e * T + t + 1) * D]
        P = params.size
        gr = torch.tensor(O.mingru_grad_batch(params, obsTB, sc, Bmb, T, H, D, L, A)[:P])
        dist.all_reduce(gr)
        parts = [None] * world
        dist.all_gather_object(parts, (adv, val, logp, act, term, obs, seg, mbp))
        if rank == 0:
            # single process: both rollouts side by side, rank 1's segments offset by N
            cat = [np.concatenate([p[i] for p in parts]) for i in range(6)]
            segu = np.concatenate([parts[0][6], parts[1][6] + N])
            mbpu = np.concatenate([parts[0][7], parts[1][7]])
            Bu = segu.size
            scu = O.gather_seq_minibatch(cat[3], cat[2], cat[4], cat[0], cat[1], segu, mbpu, T, Bu)
            obsu = np.zeros(T * Bu * D)
            for t in range(T):
                for b in range(Bu):
                    e = int(segu[b])
                    obsu[(t * Bu + b) * D:(t * Bu + b + 1) * D] = cat[5][(e * T + t) * D:(e * T + t + 1) * D]
            ref = O.mingru_grad_batch(params, obsu, scu, Bu, T, H, D, L, A)[:P]
            q.put(float(np.max(np.abs(gr.numpy() - ref) / (np.abs(ref) + 1e-9))))
    finally:
        dist.destroy_process_group()


def test_mingru_dp_decomposition_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + os.getpid() % 300
    procs = [ctx.Process(target=_mg_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rel = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert rel < 1e-9, rel
