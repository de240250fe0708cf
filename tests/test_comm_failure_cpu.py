"""Failure handling of the data-parallel communicator, on the host only (no GPU is faulted, trapped or
hung): the NCCL entry points and the stream query are replaced by fakes (pl_test_comm_fake), and a rank
that leaves between updates is a real process that exits.

* a peer that never joins: creation fails with PL_ERR_COMM at the deadline and the half-made
  communicator is aborted;
* a peer that fails once the communicator is up: the watchdog (pl_comm_wait) reports it, aborts, and
  every later call fails at once;
* enqueued work that never completes: the watchdog's deadline aborts;
* a rank that exits between updates: its peer learns it from the host-side store (RankWatch) before
  the next launch and aborts the communicator.
"""
import ctypes as C
import os
import time

import pytest
import torch.multiprocessing as mp

import pufferlean_b200 as plb

def _lib():
    L = plb.lib()
    L.pl_test_comm_fake.argtypes = [C.c_int]
    L.pl_comm_set_timeout.argtypes = [C.c_double]
    L.pl_comm_create.argtypes = [C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]
    L.pl_comm_wait.argtypes = [C.c_void_p, C.c_void_p]
    L.pl_comm_abort.argtypes = [C.c_void_p]
    L.pl_comm_aborted.argtypes = [C.c_void_p]
    L.pl_comm_destroy.argtypes = [C.c_void_p]
    return L


def _err_comm():
    return -7  # PL_ERR_COMM (include/pufferlean_b200.h)


@pytest.fixture()
def fake():
    L = _lib()
    prev_timeout = 600.0
    yield L
    L.pl_test_comm_fake(0)
    L.pl_comm_set_timeout(prev_timeout)


def _create(L, rank=0, world=2):
    ident = (C.c_uint8 * 128)()
    assert L.pl_comm_unique_id(ident) == 0
    comm = C.c_void_p()
    rc = L.pl_comm_create(rank, world, ident, C.byref(comm))
    return rc, comm


def test_peer_that_never_joins_fails_creation_at_the_deadline(fake):
    L = fake
    L.pl_test_comm_fake(1)
    L.pl_comm_set_timeout(0.3)
    a0 = L.pl_test_comm_fake_aborts()
    t0 = time.monotonic()
    rc, comm = _create(L)
    dt = time.monotonic() - t0
    assert rc == _err_comm()
    assert "did not complete" in L.pl_last_error().decode()
    assert not comm.value
    assert L.pl_test_comm_fake_aborts() == a0 + 1
    assert 0.25 < dt < 5.0


def test_failed_peer_is_reported_by_the_watchdog_and_aborts(fake):
    L = fake
    L.pl_test_comm_fake(2)
    L.pl_comm_set_timeout(5.0)
    rc, comm = _create(L)
    assert rc == 0, L.pl_last_error()
    assert L.pl_comm_aborted(comm) == 0
    a0 = L.pl_test_comm_fake_aborts()
    assert L.pl_comm_wait(comm, None) == _err_comm()
    assert "remote process exited" in L.pl_last_error().decode()
    assert L.pl_comm_aborted(comm) == 1
    assert L.pl_test_comm_fake_aborts() == a0 + 1
    # every later call fails at once, and the abort is not repeated
    t0 = time.monotonic()
    assert L.pl_comm_wait(comm, None) == _err_comm()
    assert "aborted" in L.pl_last_error().decode()
    assert time.monotonic() - t0 < 0.5
    assert L.pl_comm_abort(comm) == 0
    assert L.pl_test_comm_fake_aborts() == a0 + 1
    assert L.pl_comm_destroy(comm) == 0


def test_work_that_never_completes_is_aborted_at_the_deadline(fake):
    L = fake
    L.pl_test_comm_fake(3)
    L.pl_comm_set_timeout(0.3)
    rc, comm = _create(L)
    assert rc == 0, L.pl_last_error()
    t0 = time.monotonic()
    assert L.pl_comm_wait(comm, None) == _err_comm()
    assert 0.25 < time.monotonic() - t0 < 5.0
    assert "did not complete" in L.pl_last_error().decode()
    assert L.pl_comm_aborted(comm) == 1
    assert L.pl_comm_destroy(comm) == 0


def test_healthy_communicator_waits_and_destroys(fake):
    L = fake
    L.pl_test_comm_fake(4)
    rc, comm = _create(L)
    assert rc == 0
    assert L.pl_comm_wait(comm, None) == 0
    assert L.pl_comm_aborted(comm) == 0
    assert L.pl_comm_aborted(None) == -1
    assert L.pl_comm_destroy(comm) == 0


def _rank(rank, world, port, steps_before_exit, q):
    import torch.distributed as dist

    from pufferlean_b200.watch import PeerLost, RankWatch

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, wait_for_workers=True)
    L = _lib()
    L.pl_test_comm_fake(4)
    rc, comm = _create(L, rank, world)
    assert rc == 0
    w = RankWatch(store, rank, world)
    for step in range(4):
        try:
            w.ready(step, timeout_s=2.0)
        except PeerLost as e:
            L.pl_comm_abort(comm)
            q.put((rank, step, e.missing, L.pl_comm_aborted(comm)))
            return
        # ... the update's kernels and collectives would be enqueued here, then pl_comm_wait ...
        assert L.pl_comm_wait(comm, None) == 0
        if rank == 1 and step + 1 == steps_before_exit:
            os._exit(0)  # leaves between two updates, with nothing in flight
    q.put((rank, None, [], L.pl_comm_aborted(comm)))


def test_rank_that_exits_between_updates_is_found_before_the_next_launch():
    """Rank 1 finishes updates 0 and 1 and exits; rank 0 finds it missing at update 2, before launching."""
    world, port = 2, 29400 + os.getpid() % 500
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, 2, q)) for r in range(world)]
    for p in procs:
        p.start()
    rank, step, missing, aborted = q.get(timeout=60)
    for p in procs:
        p.join(timeout=30)
    assert rank == 0 and step == 2 and missing == [1] and aborted == 1
    assert all(p.exitcode == 0 for p in procs)
