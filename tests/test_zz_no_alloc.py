"""The allocation-free Newton-Schulz entry point (pl_ns_batched_bf16_dev_noalloc).

It exists for callers that cannot call cudaMalloc: a host whose device memory belongs to its own
allocator or to a budget fixed at start-up, or a loop that must stay off the driver's allocator. It
runs the same kernels as the allocating entry point, so it must give the same bits, call after call,
although every call reuses (and finds the previous call's leftovers in) the same fixed workspace. This file is named to
be collected last, so a run that stops at the first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402

pytestmark = pytest.mark.gpu

QUINTIC = np.ascontiguousarray(np.array([[3.4445, -4.7750, 2.0315]] * 5, dtype=np.float64))
DP = C.POINTER(C.c_double)


def _fn(name):
    f = getattr(plb.lib(), name)
    f.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_double, DP, C.c_size_t, C.c_void_p]
    f.restype = C.c_int
    return f


def _run(name, X, batch, rows, cols):
    rc = _fn(name)(X.data_ptr(), batch, rows, cols, 1e-7, QUINTIC.ctypes.data_as(DP), 5, None)
    assert rc == 0, plb.lib().pl_last_error().decode()


def _rel(a, b):
    return float((a - b).norm() / b.norm())


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


# fused small-matrix kernel (both sides <= 128), wide persistent chain with the normalisation folded
# into the first step (m > 128), tall matrices through the transpose (m > 128), then the small case
# again on what the larger calls left behind
SHAPES = [(4, 128, 256), (2, 256, 1024), (3, 768, 512), (3, 96, 64)]


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    # consecutive calls with different shapes and data: each later call runs on the leftover
    # workspace (counters, partial sums, iterates) of the one before; both entry points run the same
    # kernels, so the results must be bit-identical
    for rep in range(2):
        for seed, (batch, rows, cols) in enumerate(SHAPES):
            torch.manual_seed(100 + 10 * rep + seed)
            X = torch.randn(batch, rows, cols, device="cuda").to(torch.bfloat16)
            ref = X.clone()
            _run("pl_ns_batched_bf16_dev", ref, batch, rows, cols)
            got = X.clone()
            _run("pl_ns_batched_bf16_dev_noalloc", got, batch, rows, cols)
            torch.cuda.synchronize()
            assert torch.isfinite(got.float()).all()
            assert torch.equal(got, ref), (batch, rows, cols, _rel(got.float(), ref.float()))


def test_noalloc_rejects_requests_above_its_fixed_workspace():
    X = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    rc = _fn("pl_ns_batched_bf16_dev_noalloc")(X.data_ptr(), 64, 2048, 2048, 1e-7, QUINTIC.ctypes.data_as(DP), 5,
                                                 None)
    assert rc == -1
    assert "limit" in plb.lib().pl_last_error().decode()
