"""The persistent Newton-Schulz chain (every step of a batch in one cooperative launch, with per-matrix
tile counters as the only synchronisation) against the per-step GEMM launches on the same inputs -- bit
for bit, since both run the same 128 x 256 tiles through the same epilogue -- and against the f64 oracle:
square, wide, tall (transposed on the way in and out), sides that are not multiples of the tile, even and
odd step counts, repeated calls, the allocation-free entry point, and the fp32-output form inside a bf16
MLP update."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu
DP = C.POINTER(C.c_double)


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def _chain(mode):
    L = plb.lib()
    L.pl_test_ns_chain_mode.argtypes = [C.c_int]
    return L.pl_test_ns_chain_mode(mode)


def _ns(X, batch, rows, cols, co, entry="pl_ns_batched_bf16_dev"):
    L = plb.lib()
    fn = getattr(L, entry)
    fn.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_double, DP, C.c_size_t, C.c_void_p]
    rc = fn(X.data_ptr(), batch, rows, cols, 1e-7, co.ctypes.data_as(DP), co.shape[0], None)
    assert rc == 0, L.pl_last_error()
    torch.cuda.synchronize()
    code = C.c_uint(0)
    assert L.pl_test_device_error(C.byref(code)) == 0 and code.value == 0, hex(code.value)


def _both(X0, batch, rows, cols, co, entry="pl_ns_batched_bf16_dev"):
    prev = _chain(1)
    try:
        Xc = X0.clone()
        _ns(Xc, batch, rows, cols, co, entry)
        _chain(0)
        Xs = X0.clone()
        _ns(Xs, batch, rows, cols, co, entry)
    finally:
        _chain(prev)
    return Xc, Xs


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("batch,rows,cols", [(8, 512, 512), (5, 384, 768), (3, 256, 1024), (4, 1024, 512),
                                             (2, 200, 328), (16, 512, 2048), (1, 136, 2048), (1, 72, 2048),
                                             (2, 128, 1024), (3, 64, 640), (1, 2048, 72)])
@pytest.mark.parametrize("steps", [5, 4])
def test_chain_is_bit_identical_to_per_step_launches(batch, rows, cols, steps):
    torch.manual_seed(rows + 3 * cols + steps)
    X0 = torch.randn(batch, rows, cols, device="cuda").to(torch.bfloat16)
    co = np.ascontiguousarray(O.QUINTIC_COEFFS[:steps])
    Xc, Xs = _both(X0, batch, rows, cols, co)
    assert torch.equal(Xc, Xs)
    assert not torch.equal(Xc, X0)


def test_chain_vs_oracle_and_repeatable():
    batch, rows, cols = 3, 200, 328
    torch.manual_seed(5)
    X0 = torch.randn(batch, rows, cols, device="cuda").to(torch.bfloat16)
    co = np.ascontiguousarray(O.QUINTIC_COEFFS)
    prev = _chain(1)
    try:
        a = X0.clone()
        _ns(a, batch, rows, cols, co)
        b = X0.clone()
        _ns(b, batch, rows, cols, co)
    finally:
        _chain(prev)
    assert torch.equal(a, b)
    Xin, got = X0.double().cpu().numpy(), a.double().cpu().numpy()
    for i in range(batch):
        ref = O.newton_schulz(Xin[i].ravel(), rows, cols, 1e-7, co).reshape(rows, cols)
        assert rel(got[i], ref) < 2e-2, (i, rel(got[i], ref))


def test_chain_noalloc_entry():
    batch, rows, cols = 6, 512, 768
    torch.manual_seed(9)
    X0 = torch.randn(batch, rows, cols, device="cuda").to(torch.bfloat16)
    co = np.ascontiguousarray(O.QUINTIC_COEFFS)
    Xc, Xs = _both(X0, batch, rows, cols, co, "pl_ns_batched_bf16_dev_noalloc")
    assert torch.equal(Xc, Xs)
    Xr = X0.clone()
    _ns(Xr, batch, rows, cols, co)  # the allocating entry: same kernels, same result
    assert torch.equal(Xc, Xr)


def test_chain_fp32_output_in_deep_update():
    """bf16-tier deep MLP update whose two hidden 192 x 192 matrices take the chain (batched, fp32 output
    for the finalise): the same parameters bit for bit as with per-step launches."""
    from tests.test_gpu_update import _problem, _run_resident
    NT, D, H, A, L, E, MB = 2048, 20, 192, 7, 3, 1, 2
    P, pm, obs, acts, adv, ret, olp, ov = _problem(NT, D, H, A, L, 41, 1)
    perm = O.shuffle_perm(NT, E, 79)
    prev = _chain(1)
    try:
        got_c, _ = _run_resident(pm, P, (L, 1), obs, acts, adv, ret, olp, ov, perm, NT, D, H, A, E, MB, 0.02, 0.2, 0.5, 1)
        _chain(0)
        got_s, _ = _run_resident(pm, P, (L, 1), obs, acts, adv, ret, olp, ov, perm, NT, D, H, A, E, MB, 0.02, 0.2, 0.5, 1)
    finally:
        _chain(prev)
    assert np.array_equal(got_c, got_s)


@pytest.mark.parametrize("batch,rows,cols,steps", [(3, 200, 328, 5), (2, 512, 1024, 2), (4, 256, 256, 3)])
def test_folded_normalisation_vs_oracle(batch, rows, cols, steps):
    """Wide batches with m > 128 start from the caller's unnormalised X: the first step's G and X'
    epilogues apply 1/||X||^2 and 1/||X|| per matrix (no scaled copy), and the result, written back
    over X, meets the 2e-2 bar against the f64 oracle, chain or per-step launches alike."""
    torch.manual_seed(batch * rows + steps)
    X0 = (3.0 * torch.randn(batch, rows, cols, device="cuda")).to(torch.bfloat16)
    co = np.ascontiguousarray(O.QUINTIC_COEFFS[:steps])
    Xc, Xs = _both(X0, batch, rows, cols, co)
    assert torch.equal(Xc, Xs)
    Xin, got = X0.double().cpu().numpy(), Xc.double().cpu().numpy()
    for i in range(batch):
        ref = O.newton_schulz(Xin[i].ravel(), rows, cols, 1e-7, co).reshape(rows, cols)
        assert rel(got[i], ref) < 2e-2, (i, rel(got[i], ref))


@pytest.mark.parametrize("batch,rows,cols", [(2, 512, 1024), (1, 1024, 512)])
def test_chain_recorded_in_a_graph_equals_eager(batch, rows, cols):
    """The persistent chain recorded into a CUDA graph (a cooperative kernel node) and replayed gives the
    eager launch's bits, twice in a row (the graph's counter resets run with it)."""
    L = plb.lib()
    L.pl_test_ns_chain_capture.argtypes = [C.c_int]
    co = np.ascontiguousarray(O.QUINTIC_COEFFS)
    torch.manual_seed(rows + cols + batch)
    X0 = torch.randn(batch, rows, cols, device="cuda").to(torch.bfloat16)
    prev_c, prev_g = _chain(1), L.pl_test_ns_chain_capture(1)
    try:
        Xe = X0.clone()
        _ns(Xe, batch, rows, cols, co)
        Xg = X0.clone()
        st = torch.cuda.Stream()
        fn = L.pl_ns_batched_bf16_dev
        fn.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_double, DP, C.c_size_t, C.c_void_p]
        with torch.cuda.stream(st):  # warm-up: the workspace is allocated outside the capture
            assert fn(Xg.data_ptr(), batch, rows, cols, 1e-7, co.ctypes.data_as(DP), co.shape[0], st.cuda_stream) == 0
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            rc = fn(Xg.data_ptr(), batch, rows, cols, 1e-7, co.ctypes.data_as(DP), co.shape[0],
                    torch.cuda.current_stream().cuda_stream)
        assert rc == 0, L.pl_last_error()
        for _ in range(2):
            Xg.copy_(X0)
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(Xg, Xe)
        code = C.c_uint(0)
        assert L.pl_test_device_error(C.byref(code)) == 0 and code.value == 0, hex(code.value)
        del g
    finally:
        _chain(prev_c)
        L.pl_test_ns_chain_capture(prev_g)


@pytest.mark.parametrize("batch,rows,cols", [(2, 512, 1024), (2, 64, 256), (1, 1024, 512)])
@pytest.mark.parametrize("eps", [1e-7, 1e-12])
def test_zero_matrices_stay_zero(batch, rows, cols, eps):
    """A zero input (the normalisation's scale then 1 / eps) orthogonalises to zero, with no NaN: the
    trace-scaled first step, the fused kernel's in-kernel normalisation and the transposed path."""
    X = torch.zeros(batch, rows, cols, device="cuda", dtype=torch.bfloat16)
    X[-1, 0, 0] = 1.0  # one non-zero matrix beside the zero ones
    co = np.ascontiguousarray(O.QUINTIC_COEFFS)
    rc = plb.lib().pl_ns_batched_bf16_dev(X.data_ptr(), batch, rows, cols, eps, co.ctypes.data_as(DP), co.shape[0],
                                          None)
    assert rc == 0, plb.lib().pl_last_error()
    torch.cuda.synchronize()
    assert bool(torch.isfinite(X.float()).all())
    if batch > 1:
        assert bool((X[:-1] == 0).all())
    assert float(X[-1].float().abs().max()) > 0.5


def _groups(Xs, shapes, co):
    L = plb.lib()
    L.pl_ns_groups_bf16_dev.argtypes = [C.c_size_t, C.POINTER(C.c_void_p)] + [C.POINTER(C.c_size_t)] * 3 + [
        C.c_double, DP, C.c_size_t, C.c_void_p]
    n = len(shapes)
    ptrs = (C.c_void_p * n)(*[X.data_ptr() for X in Xs])
    b, r, c = [(C.c_size_t * n)(*[s[i] for s in shapes]) for i in range(3)]
    rc = L.pl_ns_groups_bf16_dev(n, ptrs, b, r, c, 1e-7, co.ctypes.data_as(DP), co.shape[0], None)
    assert rc == 0, L.pl_last_error()
    torch.cuda.synchronize()
    code = C.c_uint(0)
    assert L.pl_test_device_error(C.byref(code)) == 0 and code.value == 0, hex(code.value)


@pytest.mark.parametrize("shapes", [
    [(8, 128, 128), (8, 512, 512), (8, 512, 2048)],  # configs[2]'s three shapes, fewer matrices each
    [(2, 256, 1024), (3, 192, 640), (1, 2048, 512), (4, 64, 320), (1, 384, 384)],  # tall, short, ragged tiles
    [(1, 136, 2048), (2, 200, 264), (1, 512, 512), (2, 256, 256), (1, 1024, 2048)],  # five chain groups: two launches
])
def test_groups_entry_matches_one_call_per_shape(shapes):
    """pl_ns_groups_bf16_dev gives every group the bits pl_ns_batched_bf16_dev gives it alone: the wide
    groups with a short side above 128 share persistent launches (at most four per launch), the others
    take the single-shape paths."""
    g = torch.Generator(device="cuda").manual_seed(0x6E5)
    co = np.ascontiguousarray(O.QUINTIC_COEFFS)
    X0 = [torch.randn(b, r, c, device="cuda", generator=g).to(torch.bfloat16) for b, r, c in shapes]
    Xg = [x.clone() for x in X0]
    _groups(Xg, shapes, co)
    for x, xg, (b, r, c) in zip(X0, Xg, shapes):
        xs = x.clone()
        _ns(xs, b, r, c, co)
        assert torch.equal(xg, xs), (b, r, c)
        assert not torch.equal(xg, x)
