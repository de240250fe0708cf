"""The CTA-pair (cta_group::2) tcgen05 GEMM against a plain fp32 torch reference of the same bf16 inputs
and against the single-CTA kernel on the same inputs: every pair instance (fp32 / bf16+axpby / forward /
data-gradient epilogues, each operand layout the update uses), on shapes whose edges the pair tiling
meets — M not a multiple of 256 (including an odd CTA whose 128 rows all lie past M), N leaving half of a
pair's B rows empty, K not a multiple of 64, split-K slices and stacked matrices."""
import ctypes as C
import math

import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402

from . import gemm_util as G  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def _mode(m):
    L = plb.lib()
    L.pl_test_gemm_pair_mode.argtypes = [C.c_int]
    return L.pl_test_gemm_pair_mode(m)


def _both(run):
    """run() under single-CTA tiles and under CTA pairs; returns (single, pair) outputs."""
    prev = _mode(0)
    try:
        a = run()
        torch.cuda.synchronize()
        _mode(1)
        b = run()
        torch.cuda.synchronize()
    finally:
        _mode(prev)
    assert G.device_error() == 0
    return a, b


def _bf(x):
    return x.to(torch.bfloat16)


def _rel(x, y):
    return (x.float() - y.float()).norm().item() / max(y.float().norm().item(), 1e-30)


def _pad8(t):
    c = (t.shape[1] + 7) // 8 * 8
    out = torch.zeros(t.shape[0], c, dtype=t.dtype, device=t.device)
    out[:, :t.shape[1]] = t
    return out


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,N,K", [(512, 512, 1024), (260, 384, 100), (300, 256, 640), (1024, 768, 64)])
def test_pair_f32_layouts(a_mn, b_mn, M, N, K):
    torch.manual_seed(M + N + K + 2 * a_mn + b_mn)
    A = _pad8(_bf(torch.randn(K, M, device="cuda"))) if a_mn else _pad8(_bf(torch.randn(M, K, device="cuda")))
    B = _pad8(_bf(torch.randn(K, N, device="cuda"))) if b_mn else _pad8(_bf(torch.randn(N, K, device="cuda")))

    def run():
        out = torch.full((M, N), float("nan"), device="cuda")
        G.gemm(A, B, M, N, K, a_mn, b_mn, 256, G.EPI_F32, out=out)
        return out

    single, pair = _both(run)
    A32 = (A.float().t() if a_mn else A.float())[:M, :K]
    B32 = (B.float().t() if b_mn else B.float())[:N, :K]
    ref = A32 @ B32.t()
    assert _rel(pair, ref) < 1e-5, _rel(pair, ref)
    assert _rel(pair, single) < 1e-6, _rel(pair, single)


def test_pair_split_k():
    torch.manual_seed(5)
    M, N, K = 512, 768, 8192
    A = _bf(torch.randn(K, M, device="cuda"))
    B = _bf(torch.randn(K, N, device="cuda"))

    def run():
        part = torch.zeros(4, M, N, device="cuda")
        G.gemm(A, B, M, N, K, True, True, 256, G.EPI_F32, out=part[0], out_bstride=M * N, k_splits=4)
        return part

    single, pair = _both(run)
    ref = A.float().t() @ B.float()
    assert _rel(pair.sum(0), ref) < 1e-5
    assert _rel(pair, single) < 1e-6


@pytest.mark.parametrize("b_mn", [False, True])
def test_pair_bf16_batched_axpby(b_mn):
    """The Newton-Schulz shapes: stacked matrices, bf16 output alpha*acc + beta*aux."""
    torch.manual_seed(11 + b_mn)
    nb, m, n = 5, 512, 640
    X = _bf(torch.randn(nb, m, n, device="cuda") / math.sqrt(n))
    Y = _bf(torch.randn(nb, n, m, device="cuda") / math.sqrt(n)) if b_mn else X
    aux = _bf(torch.randn(nb, m, m, device="cuda"))

    def run():
        out = torch.empty(nb, m, m, dtype=torch.bfloat16, device="cuda")
        g = G.GemmArgs()
        g.a, g.a_rows, g.a_cols, g.a_ld, g.a_bstride, g.a_mn = X.data_ptr(), m, n, n, m * n, 0
        if b_mn:
            g.b, g.b_rows, g.b_cols, g.b_ld, g.b_bstride, g.b_mn = Y.data_ptr(), n, m, m, n * m, 1
        else:
            g.b, g.b_rows, g.b_cols, g.b_ld, g.b_bstride, g.b_mn = X.data_ptr(), m, n, n, m * n, 0
        g.M, g.N, g.K, g.bn, g.epi, g.batch, g.k_splits = m, m, n, 256, G.EPI_BF16, nb, 1
        g.out, g.ldo, g.out_bstride, g.out_rows, g.out_cols = out.data_ptr(), m, m * m, m, m
        g.alpha, g.beta = 0.75, -0.5
        g.aux, g.ld_aux, g.aux_bstride = aux.data_ptr(), m, m * m
        G.run(g)
        return out

    single, pair = _both(run)
    Bm = Y.float() if b_mn else X.float().transpose(1, 2)
    ref = 0.75 * (X.float() @ Bm) - 0.5 * aux.float()
    assert _rel(pair, ref) < 1e-2, _rel(pair, ref)
    assert _rel(pair, single) < 1e-3, _rel(pair, single)


@pytest.mark.parametrize("act", [0, 1])
def test_pair_forward_and_dgrad(act):
    torch.manual_seed(20 + act)
    M, H, D = 300, 512, 128
    X = _bf(torch.randn(M, D, device="cuda"))
    W = _bf(torch.randn(H, D, device="cuda") / math.sqrt(D))
    b = torch.randn(H, device="cuda")

    def fwd():
        Hout = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
        Z = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
        G.gemm(X, W, M, H, D, False, False, 256, G.EPI_FWD, out=Hout, bias=b, out2=Z, ldo2=H, act=act)
        return torch.cat([Hout, Z], 1)

    single, pair = _both(fwd)
    z = X.float() @ W.float().t() + b
    h = torch.relu(z) if act == 0 else torch.nn.functional.gelu(z, approximate="tanh")
    assert _rel(pair[:, :H], h) < 1e-2 and _rel(pair[:, H:], z) < 1e-2
    assert _rel(pair, single) < 1e-3
    Z = pair[:, H:].contiguous()
    Hh = pair[:, :H].contiguous()
    # data gradient with column partials; M = 260 leaves the odd CTA of the second pair tile past M
    M2, N2 = 260, 192
    dY = _bf(torch.randn(M2, N2, device="cuda"))
    W2 = _bf(torch.randn(N2, H, device="cuda"))
    aux = (Z if act == 1 else Hh)[:M2].contiguous()
    mt = (M2 + 127) // 128

    def dgrad():
        dZ = torch.empty(M2, H, dtype=torch.bfloat16, device="cuda")
        cs = torch.full((mt + 1, H), 7.0, device="cuda")  # one guard row past the ceil(M / 128) partials
        G.gemm(dY, W2, M2, H, N2, False, True, 256, G.EPI_DGRAD, out=dZ, aux=aux, ld_aux=H, act=act, colsum=cs,
               ld_colsum=H)
        return dZ, cs

    (dz1, cs1), (dz2, cs2) = _both(dgrad)
    dh = dY.float() @ W2.float()
    zz = aux.float()
    if act == 0:
        dz = dh * (zz > 0).float()
    else:
        u = 0.7978845608028654 * (zz + 0.044715 * zz ** 3)
        t = torch.tanh(u)
        dz = dh * (0.5 * (1 + t) + 0.5 * zz * (1 - t * t) * 0.7978845608028654 * (1 + 3 * 0.044715 * zz * zz))
    assert _rel(dz2, dz) < 1e-2
    assert _rel(dz2, dz1) < 1e-3
    assert _rel(cs2[:mt].sum(0), dz.sum(0)) < 1e-4
    assert bool(torch.all(cs2[mt] == 7.0)), "a column partial was written past ceil(M / 128) rows"


def test_pair_mode_hook_round_trip():
    prev = _mode(-1)
    assert _mode(0) == prev
    assert _mode(-1) == 0
    _mode(prev)
    assert _mode(-1) == prev

