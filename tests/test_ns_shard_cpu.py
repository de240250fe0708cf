"""Host side of the sharded batched Newton-Schulz (pl_ns_batched_bf16_dev_sharded), on CPU.

* pl_ns_shard_chunks: the plan every rank derives alone (matrices per rank and chunk, chunks used).
* The decomposition the library runs with NCCL, here as gloo ranks on the oracle's f64 Newton-Schulz
  (2 and 3 ranks, batches that leave a remainder and batches smaller than the world): in chunk c rank r
  orthogonalises its slice in place, the chunk is all-gathered in place, the remainder runs on every
  rank, and every rank ends with the single-process result.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import pufferlean_b200 as plb
from oracle import oracle as O

ROWS, COLS = 8, 16


def plan(batch, world, chunks):
    L = plb.lib()
    L.pl_ns_shard_chunks.argtypes = [C.c_size_t, C.c_size_t, C.c_size_t, C.POINTER(C.c_size_t),
                                     C.POINTER(C.c_size_t)]
    cs, used = C.c_size_t(), C.c_size_t()
    assert L.pl_ns_shard_chunks(batch, world, chunks, C.byref(cs), C.byref(used)) == 0
    return cs.value, used.value


@pytest.mark.parametrize("batch,world,chunks,want", [
    (64, 8, 2, (4, 2)), (64, 2, 2, (16, 2)), (64, 1, 2, (32, 2)), (7, 2, 2, (1, 2)), (5, 2, 4, (1, 2)),
    (3, 2, 2, (1, 1)), (1, 2, 2, (0, 0)), (64, 8, 64, (1, 8)), (100, 3, 0, (33, 1)),
])
def test_shard_chunks(batch, world, chunks, want):
    # (64, 8, 64): clamped to 16 chunks, then lowered to 8, one matrix per rank and chunk
    got = plan(batch, world, chunks)
    assert got == want
    cs, used = got
    assert used * world * cs <= batch
    if used:
        assert cs >= 1 and used <= 16


def _ns_all(X, n):
    return np.stack([O.newton_schulz(X[i].ravel(), ROWS, COLS, 1e-7).reshape(ROWS, COLS) for i in range(n)])


def _rank(rank, world, port, batch, chunks, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = np.random.default_rng(1234 + batch)
        X = g.standard_normal((batch, ROWS, COLS))  # every rank holds the same inputs
        cs, used = plan(batch, world, chunks)
        span = world * cs
        for c in range(used):
            lo = c * span + rank * cs
            X[lo:lo + cs] = _ns_all(X[lo:lo + cs], cs)
            parts = [torch.empty(cs, ROWS, COLS, dtype=torch.float64) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(X[lo:lo + cs].copy()))
            X[c * span:(c + 1) * span] = torch.cat(parts).numpy()
        done = used * span
        X[done:] = _ns_all(X[done:], batch - done)
        q.put((rank, X.tobytes()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,batch,chunks", [(2, 9, 2), (3, 7, 2), (2, 1, 2), (3, 12, 3)])
def test_sharded_decomposition_equals_one_process(world, batch, chunks):
    port = 29600 + (os.getpid() + 7 * world + batch) % 300
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, batch, chunks, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    g = np.random.default_rng(1234 + batch)
    X = g.standard_normal((batch, ROWS, COLS))
    ref = _ns_all(X, batch)
    for r in range(world):
        assert np.array_equal(np.frombuffer(outs[r]).reshape(batch, ROWS, COLS), ref), r


def test_groups_entry_rejects_bad_tables_before_any_work():
    """pl_ns_groups_bf16_dev checks every group before it runs any: these fail with PL_ERR_INVALID
    without a device (a call that reached the GPU would fail with PL_ERR_NO_DEVICE here instead)."""
    L = plb.lib()
    fn = L.pl_ns_groups_bf16_dev
    fn.argtypes = [C.c_size_t, C.POINTER(C.c_void_p)] + [C.POINTER(C.c_size_t)] * 3 + [
        C.c_double, C.POINTER(C.c_double), C.c_size_t, C.c_void_p]
    co = np.ascontiguousarray(np.array([[3.4445, -4.7750, 2.0315]] * 5))
    cp = co.ctypes.data_as(C.POINTER(C.c_double))

    def call(n, shapes, ptrs=None, coeffs=cp, iters=5, table=True):
        if not table:
            return fn(n, None, None, None, None, 1e-7, coeffs, iters, None)
        k = max(len(shapes), 1)
        X = (C.c_void_p * k)(*(ptrs if ptrs is not None else [0x1000] * k))
        b, r, c = [(C.c_size_t * k)(*[s[i] for s in shapes] or [0]) for i in range(3)]
        return fn(n, X, b, r, c, 1e-7, coeffs, iters, None)

    assert call(0, []) == 0  # nothing to do
    assert call(17, [(1, 8, 8)] * 17) == -1  # more than 16 groups
    assert call(1, [], table=False) == -1  # no group table
    assert call(1, [(1, 512, 512)], coeffs=None) == -1  # no coefficients
    assert call(1, [(1, 512, 512)], iters=0) == -1
    # the bad group is the last: the first two (one chain group, one fused) must not have run
    assert call(3, [(2, 512, 512), (2, 64, 64), (1, 512, 100)]) == -1
    assert "multiples of 8" in plb.lib().pl_last_error().decode()
    assert call(2, [(2, 512, 512), (1, 256, 256)], ptrs=[0x1000, 0]) == -1  # NULL matrices
