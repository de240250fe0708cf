"""Sharded batched Newton-Schulz on 2 GPUs (skipped with fewer): one process per GPU, the library's
own NCCL communicator. Every rank passes the same batch; each must end with every matrix bit-identical
to pl_ns_batched_bf16_dev of the whole batch on one GPU: wide and tall shapes, the chain (m > 128) and
the small fused kernel (n <= 128), a batch that leaves a remainder for every rank, and one smaller than
the world (nothing sharded)."""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

WORLD = 2
SHAPES = [(12, 512, 2048, 2), (7, 384, 768, 2), (5, 1024, 512, 2), (16, 128, 128, 4), (1, 256, 256, 2)]
QUINTIC = [(4.0848, -6.8946, 2.9270), (3.9505, -6.3029, 2.6377), (3.7418, -5.5913, 2.3037), (2.8769, -3.1427, 1.2046),
           (2.8366, -3.0525, 1.2012)]


def _inputs(batch, rows, cols):
    g = torch.Generator().manual_seed(batch * 7 + rows + cols)
    return torch.randn(batch, rows, cols, generator=g).to(torch.bfloat16)


def _run_shapes(L, comm):
    co = np.ascontiguousarray(np.array(QUINTIC, dtype=np.float64))
    dp = C.POINTER(C.c_double)
    L.pl_ns_batched_bf16_dev_sharded.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_double, dp,
                                                 C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p]
    L.pl_ns_batched_bf16_dev.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_double, dp, C.c_size_t,
                                         C.c_void_p]
    res = []
    for batch, rows, cols, chunks in SHAPES:
        X = _inputs(batch, rows, cols).cuda()
        ref = X.clone()
        for rep in range(2):  # the second call reuses the streams, events and workspace
            Xs = X.clone()
            rc = L.pl_ns_batched_bf16_dev_sharded(Xs.data_ptr(), batch, rows, cols, 1e-7, co.ctypes.data_as(dp), 5,
                                                  comm, chunks, None)
            assert rc == 0, L.pl_last_error()
        assert L.pl_ns_batched_bf16_dev(ref.data_ptr(), batch, rows, cols, 1e-7, co.ctypes.data_as(dp), 5, None) == 0
        torch.cuda.synchronize()
        res.append((batch, rows, cols, bool(torch.equal(Xs, ref)), bool(torch.equal(Xs, X))))
    return res


def _rank(rank, port, q):
    import torch.distributed as dist

    import pufferlean_b200 as plb

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    L = plb.lib()
    L.pl_set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    comm = C.c_void_p()
    try:
        ident = (C.c_uint8 * 128)()
        if rank == 0:
            assert L.pl_comm_unique_id(ident) == 0
        box = [bytes(ident)]
        dist.broadcast_object_list(box, src=0)
        ident = (C.c_uint8 * 128)(*box[0])
        L.pl_comm_create.argtypes = [C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]
        assert L.pl_comm_create(rank, WORLD, ident, C.byref(comm)) == 0, L.pl_last_error()
        res = _run_shapes(L, comm)
        q.put((rank, res))
    finally:
        if comm.value:
            L.pl_comm_destroy.argtypes = [C.c_void_p]
            L.pl_comm_destroy(comm)
        dist.destroy_process_group()


def test_sharded_equals_one_gpu_bit_for_bit():
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    for r in range(WORLD):
        for batch, rows, cols, same, unchanged in outs[r]:
            assert same and not unchanged, (r, batch, rows, cols)


def test_sharded_one_rank_takes_the_chunked_path_and_equals_plain():
    """A one-rank communicator runs the same chunks, events and (single-rank, in-place) all-gathers."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import pufferlean_b200 as plb

    L = plb.lib()
    torch.cuda.set_device(0)
    ident = (C.c_uint8 * 128)()
    assert L.pl_comm_unique_id(ident) == 0
    comm = C.c_void_p()
    L.pl_comm_create.argtypes = [C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]
    assert L.pl_comm_create(0, 1, ident, C.byref(comm)) == 0, L.pl_last_error()
    try:
        for batch, rows, cols, same, unchanged in _run_shapes(L, comm):
            assert same and not unchanged, (batch, rows, cols)
    finally:
        L.pl_comm_destroy.argtypes = [C.c_void_p]
        assert L.pl_comm_destroy(comm) == 0
