"""The allocation-free Newton-Schulz entry point (pl_ns_batched_bf16_dev_noalloc).

It exists for callers that cannot call cudaMalloc (graph capture, a host that owns device memory
through its own allocator or a fixed budget). It must give the same result as the allocating entry
point, call after call, although every call reuses the same fixed workspace. This file is named to
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


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    # two calls in a row (different shapes and data, so the second one runs on the first one's
    # leftover workspace); each must agree with the allocating entry point
    for seed, (batch, rows, cols) in enumerate([(4, 128, 256), (3, 256, 128)]):
        torch.manual_seed(100 + seed)
        X = torch.randn(batch, rows, cols, device="cuda").to(torch.bfloat16)
        ref = X.clone()
        _run("pl_ns_batched_bf16_dev", ref, batch, rows, cols)
        got = X.clone()
        _run("pl_ns_batched_bf16_dev_noalloc", got, batch, rows, cols)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        # the tolerance of the Newton-Schulz tests (2e-2 relative Frobenius); the kernels are the same
        assert _rel(got.float(), ref.float()) < 2e-2


def test_noalloc_rejects_requests_above_its_fixed_workspace():
    X = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    rc = _fn("pl_ns_batched_bf16_dev_noalloc")(X.data_ptr(), 64, 2048, 2048, 1e-7, QUINTIC.ctypes.data_as(DP), 5,
                                                 None)
    assert rc == -1
    assert "limit" in plb.lib().pl_last_error().decode()
