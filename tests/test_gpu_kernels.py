"""GPU parity of the first kernels: V-trace (exact f64 and fast fp32), the f64 Muon step, and the
tcgen05 GEMM with each operand layout and epilogue.

Exact tiers are compared bit-for-bit with the reference's outputs (tests/golden, produced by the
reference's compiled C) and with the pinned oracle; the fp32 scan against the f64 oracle at 1e-5
relative; GEMMs against a plain fp32 torch reference of the same bf16 inputs.
"""
import math
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import oracle as O  # noqa: E402

from . import gemm_util as G  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


# ------------------------------------------------------------------------------------------------ V-trace
def test_vtrace_kat_bit_exact():
    f = load("vtrace")
    B, T, g, l, rho, c = f["meta"]
    out = plb.cuda_vtrace(f["rew"], f["val"], f["term"], f["imp"], int(B), int(T), g, l, rho, c)
    assert np.array_equal(out, f["adv"])


def test_vtrace_mingru_kat_bit_exact():
    f = load("vtrace_mingru")
    B, T, g, l, rho, c = f["meta"]
    out = plb.cuda_vtrace_mingru(f["rew"], f["val"], f["term"], f["imp"], f["bootv"], int(B), int(T), g, l, rho, c)
    assert np.array_equal(out, f["adv"])


def _rollout(B, T, seed, done_p=0.05):
    g = np.random.default_rng(seed)
    rew = g.uniform(-1.5, 1.5, B * T)
    val = g.standard_normal(B * T)
    term = (g.random(B * T) < done_p).astype(np.float64)
    imp = np.exp(g.normal(0, 0.3, B * T))
    boot = g.standard_normal(B)
    return rew, val, term, imp, boot


@pytest.mark.parametrize("B,T", [(1, 1), (3, 2), (64, 64), (257, 33), (100, 256), (8192, 64), (45, 17)])
def test_vtrace_f64_dev_bit_exact_vs_oracle(B, T):
    rew, val, term, imp, boot = _rollout(B, T, B * 1000 + T)
    for mingru in (False, True):
        ref = (O.vtrace_mingru(rew, val, term, imp, boot, B, T, 0.995, 0.9, 1.0, 1.0) if mingru else
               O.vtrace(rew, val, term, imp, B, T, 0.995, 0.9, 1.0, 1.0))
        d = {k: torch.tensor(v, device="cuda") for k, v in dict(rew=rew, val=val, term=term, imp=imp, boot=boot).items()}
        adv = torch.empty(B * T, dtype=torch.float64, device="cuda")
        l1 = torch.empty(B, dtype=torch.float64, device="cuda")
        rc = plb.lib().pl_vtrace_f64_dev(d["rew"].data_ptr(), d["val"].data_ptr(), d["term"].data_ptr(),
                                         d["imp"].data_ptr(), d["boot"].data_ptr() if mingru else None, B, T, 0.995,
                                         0.9, 1.0, 1.0, adv.data_ptr(), l1.data_ptr(), None)
        assert rc == 0, plb.lib().pl_last_error()
        torch.cuda.synchronize()
        assert np.array_equal(adv.cpu().numpy(), ref)
        assert np.array_equal(l1.cpu().numpy(), O.adv_l1(ref, B, T))


@pytest.mark.parametrize("B,T", [(1, 1), (5, 7), (64, 12), (4096, 64), (300, 100), (33, 256), (17, 200)])
def test_vtrace_f32_fast_matches_oracle(B, T):
    rew, val, term, imp, boot = _rollout(B, T, B * 7 + T, done_p=0.01)
    f32 = {k: v.astype(np.float32) for k, v in dict(rew=rew, val=val, term=term, imp=imp, boot=boot).items()}
    for mingru in (False, True):
        # the oracle sees exactly the fp32 inputs, widened
        ref = (O.vtrace_mingru(f32["rew"], f32["val"], f32["term"], f32["imp"], f32["boot"], B, T, 0.995, 0.9, 1.0, 1.0)
               if mingru else O.vtrace(f32["rew"], f32["val"], f32["term"], f32["imp"], B, T, 0.995, 0.9, 1.0, 1.0))
        d = {k: torch.tensor(v, device="cuda") for k, v in f32.items()}
        adv = torch.full((B * T,), float("nan"), dtype=torch.float32, device="cuda")
        l1 = torch.empty(B, dtype=torch.float32, device="cuda")
        rc = plb.lib().pl_vtrace_f32_dev(d["rew"].data_ptr(), d["val"].data_ptr(), d["term"].data_ptr(),
                                         d["imp"].data_ptr(), d["boot"].data_ptr() if mingru else None, B, T, 0.995,
                                         0.9, 1.0, 1.0, adv.data_ptr(), l1.data_ptr(), None)
        assert rc == 0, plb.lib().pl_last_error()
        got = adv.cpu().numpy().astype(np.float64)
        # tolerance stated by the spec: 1e-5 relative for fp32 advantages (relative to the scale of the row)
        scale = np.maximum(np.abs(ref), 1.0)
        assert np.max(np.abs(got - ref) / scale) < 1e-5
        np.testing.assert_allclose(l1.cpu().numpy(), O.adv_l1(ref, B, T), rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("B,T", [(1, 1), (5, 7), (64, 12), (8192, 64), (300, 100), (33, 256), (17, 200), (9, 33)])
def test_vtrace_f64_scan_matches_oracle(B, T):
    """The warp-parallel f64 scan (the recurrent update's bf16 tier) against the sequential oracle:
    a different summation order, so rounding-level agreement (1e-13 relative to the row scale)."""
    rew, val, term, imp, boot = _rollout(B, T, B * 11 + T, done_p=0.02)
    L = plb.lib()
    L.pl_vtrace_f64_scan_dev.argtypes = L.pl_vtrace_f64_dev.argtypes
    for mingru in (False, True):
        ref = (O.vtrace_mingru(rew, val, term, imp, boot, B, T, 0.995, 0.9, 1.0, 1.0) if mingru else
               O.vtrace(rew, val, term, imp, B, T, 0.995, 0.9, 1.0, 1.0))
        d = {k: torch.tensor(v, device="cuda") for k, v in dict(rew=rew, val=val, term=term, imp=imp, boot=boot).items()}
        adv = torch.full((B * T,), float("nan"), dtype=torch.float64, device="cuda")
        l1 = torch.empty(B, dtype=torch.float64, device="cuda")
        rc = L.pl_vtrace_f64_scan_dev(d["rew"].data_ptr(), d["val"].data_ptr(), d["term"].data_ptr(),
                                      d["imp"].data_ptr(), d["boot"].data_ptr() if mingru else None, B, T, 0.995, 0.9,
                                      1.0, 1.0, adv.data_ptr(), l1.data_ptr(), None)
        assert rc == 0, L.pl_last_error()
        got = adv.cpu().numpy()
        scale = np.maximum(np.abs(ref), 1.0)
        assert np.max(np.abs(got - ref) / scale) < 1e-13
        np.testing.assert_allclose(l1.cpu().numpy(), O.adv_l1(ref, B, T), rtol=1e-13, atol=1e-12)


# ------------------------------------------------------------------------------------------------ Muon f64
def test_muon_stepmat_kat_bit_exact():
    f = load("muon_stepmat")
    lr, wd, mu, eps = f["meta"]
    for i in range(3):
        rows, cols = (int(x) for x in f[f"shape{i}"])
        out = plb.cuda_muon_stepmat(f[f"W{i}"], f[f"G{i}"], f[f"M{i}"], rows, cols, lr, wd, mu, eps)
        assert np.array_equal(out, f[f"out{i}"]), (rows, cols)


@pytest.mark.parametrize("rows,cols", [(128, 4), (3, 128), (33, 17)])
def test_muon_stepmat_bit_exact_vs_oracle(rows, cols):
    g = np.random.default_rng(rows * cols)
    W, Gr, M = (g.uniform(-0.5, 0.5, rows * cols) for _ in range(3))
    out = plb.cuda_muon_stepmat(W, Gr, M, rows, cols, 0.02, 0.01, 0.95, 1e-7)
    nW, nM = O.muon_stepmat(W, Gr, M, rows, cols, 0.02, 0.01, 0.95, 1e-7)
    assert np.array_equal(out[:rows * cols], nW) and np.array_equal(out[rows * cols:], nM)


# ------------------------------------------------------------------------------------------------ GEMM
def _bf(x):
    return x.to(torch.bfloat16)


def _ref(A, B, a_mn, b_mn):
    A32 = A.float() if not a_mn else A.float().t()
    B32 = B.float() if not b_mn else B.float().t()
    return A32 @ B32.t()


def _rel(x, y):
    return (x - y).norm().item() / max(y.norm().item(), 1e-30)


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K,bn", [(128, 128, 64, 128), (256, 384, 320, 128), (200, 130, 100, 128),
                                      (512, 512, 1024, 256), (64, 64, 64, 128)])
def test_gemm_layouts(a_mn, b_mn, M, N, K, bn):
    if bn == 256 and a_mn != b_mn:
        pytest.skip("instance not built")
    torch.manual_seed(M + N + K)
    Kp = (K + 63) // 64 * 64
    A = _bf(torch.randn(K, M, device="cuda")) if a_mn else _bf(torch.randn(M, K, device="cuda"))
    B = _bf(torch.randn(K, N, device="cuda")) if b_mn else _bf(torch.randn(N, K, device="cuda"))
    # storage inner dims must be multiples of 8
    def pad(t):
        c = (t.shape[1] + 7) // 8 * 8
        out = torch.zeros(t.shape[0], c, dtype=t.dtype, device=t.device)
        out[:, :t.shape[1]] = t
        return out
    Ap, Bp = pad(A), pad(B)
    out = torch.full((M, N), float("nan"), device="cuda")
    G.gemm(Ap, Bp, M, N, K, a_mn, b_mn, bn, G.EPI_F32, out=out)
    torch.cuda.synchronize()
    assert G.device_error() == 0
    ref = _ref(A, B, a_mn, b_mn)
    assert _rel(out, ref) < 1e-5, _rel(out, ref)
    assert Kp >= K


def test_gemm_split_k_and_bf16_axpby():
    torch.manual_seed(0)
    M, N, K = 256, 256, 4096
    A = _bf(torch.randn(K, M, device="cuda"))
    B = _bf(torch.randn(K, N, device="cuda"))
    part = torch.zeros(4, M, N, device="cuda")
    G.gemm(A, B, M, N, K, True, True, 128, G.EPI_F32, out=part[0], out_bstride=M * N, k_splits=4)
    torch.cuda.synchronize()
    ref = _ref(A, B, True, True)
    assert _rel(part.sum(0), ref) < 1e-5
    # bf16 output with fused alpha*acc + beta*aux
    A2 = _bf(torch.randn(M, K, device="cuda"))
    B2 = _bf(torch.randn(N, K, device="cuda"))
    aux = _bf(torch.randn(M, N, device="cuda"))
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    G.gemm(A2, B2, M, N, K, False, False, 128, G.EPI_BF16, out=out, alpha=0.5, beta=-2.0, aux=aux, ld_aux=N)
    torch.cuda.synchronize()
    ref2 = 0.5 * (A2.float() @ B2.float().t()) - 2.0 * aux.float()
    assert _rel(out.float(), ref2) < 1e-2


@pytest.mark.parametrize("act", [0, 1])
def test_gemm_forward_and_dgrad_epilogues(act):
    torch.manual_seed(act)
    M, H, D = 300, 192, 128
    X = _bf(torch.randn(M, D, device="cuda"))
    W = _bf(torch.randn(H, D, device="cuda") / math.sqrt(D))
    b = torch.randn(H, device="cuda")
    Hout = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
    Z = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
    G.gemm(X, W, M, H, D, False, False, 64, G.EPI_FWD, out=Hout, bias=b, out2=Z, ldo2=H, act=act)
    torch.cuda.synchronize()
    z = X.float() @ W.float().t() + b
    h = torch.relu(z) if act == 0 else torch.nn.functional.gelu(z, approximate="tanh")
    assert _rel(Hout.float(), h) < 1e-2 and _rel(Z.float(), z) < 1e-2
    # data gradient: dZ = (dY W2) * act'(z), with bias-grad column partials
    N2 = 64
    dY = _bf(torch.randn(M, N2, device="cuda"))
    W2 = _bf(torch.randn(N2, H, device="cuda"))
    dZ = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
    mt = (M + 127) // 128
    cs = torch.full((mt, H), float("nan"), device="cuda")
    aux = Z if act == 1 else Hout
    G.gemm(dY, W2, M, H, N2, False, True, 128, G.EPI_DGRAD, out=dZ, aux=aux, ld_aux=H, act=act, colsum=cs, ld_colsum=H)
    torch.cuda.synchronize()
    dh = dY.float() @ W2.float()
    zz = aux.float()
    if act == 0:
        dz = dh * (zz > 0).float()
    else:
        u = 0.7978845608028654 * (zz + 0.044715 * zz ** 3)
        t = torch.tanh(u)
        dz = dh * (0.5 * (1 + t) + 0.5 * zz * (1 - t * t) * 0.7978845608028654 * (1 + 3 * 0.044715 * zz * zz))
    assert _rel(dZ.float(), dz) < 1e-2
    assert _rel(cs.sum(0), dz.sum(0)) < 1e-4


@pytest.mark.parametrize("M,H,K", [(1000, 2048, 65), (333, 200, 8), (257, 520, 128)])
def test_gemm_dgrad_short_k_aux_through_tma(M, H, K):
    """The data gradient of a short-K product (the head's, K <= 128) runs 128-wide tiles whose aux (the
    pre-activation) comes through TMA into shared memory: same values as the reference, ragged rows and
    columns included; the operand A is stored 128 wide with K live columns, as the update stores dOut."""
    torch.manual_seed(M + H + K)
    dY = torch.zeros(M, 128, device="cuda")
    dY[:, :K] = torch.randn(M, K, device="cuda")
    dY = _bf(dY)
    W2 = torch.zeros(128, (H + 7) // 8 * 8, device="cuda")
    W2[:K, :H] = torch.randn(K, H, device="cuda") / math.sqrt(K)
    W2 = _bf(W2)
    Z = _bf(torch.randn(M, (H + 7) // 8 * 8, device="cuda"))
    dZ = torch.full((M, Z.shape[1]), float("nan"), dtype=torch.bfloat16, device="cuda")
    mt = (M + 127) // 128
    cs = torch.full((mt, Z.shape[1]), float("nan"), device="cuda")
    G.gemm(dY, W2, M, H, K, False, True, 256, G.EPI_DGRAD, out=dZ, ldo=Z.shape[1], out_cols=H, aux=Z,
           ld_aux=Z.shape[1], act=1, colsum=cs, ld_colsum=Z.shape[1])
    torch.cuda.synchronize()
    assert G.device_error() == 0
    dh = dY.float()[:, :K] @ W2.float()[:K, :H]
    zz = Z.float()[:, :H]
    u = 0.7978845608028654 * (zz + 0.044715 * zz ** 3)
    t = torch.tanh(u)
    dz = dh * (0.5 * (1 + t) + 0.5 * zz * (1 - t * t) * 0.7978845608028654 * (1 + 3 * 0.044715 * zz * zz))
    assert _rel(dZ.float()[:, :H], dz) < 1e-2
    assert _rel(cs[:, :H].sum(0), dz.sum(0)) < 1e-4


@pytest.mark.parametrize("A,Op", [(5, 64), (64, 128), (79, 128), (100, 128)])
def test_gemm_ppo_head_epilogue(A, Op):
    """A + 1 <= 80 with a 128-wide tile takes the register-resident epilogue, the others the general one."""
    torch.manual_seed(3 + A)
    M, H = 333, 128
    Hid = _bf(torch.randn(M, H, device="cuda"))
    Wo = torch.zeros(Op, H, device="cuda")
    Wo[:A + 1] = torch.randn(A + 1, H, device="cuda") / math.sqrt(H)
    Wo = _bf(Wo)
    bias = torch.zeros(Op, device="cuda")
    bias[:A + 1] = torch.randn(A + 1, device="cuda") * 0.1
    act = torch.randint(0, A, (M,), device="cuda", dtype=torch.int32)
    adv = torch.randn(M, device="cuda")
    ret = torch.randn(M, device="cuda")
    olp = -torch.rand(M, device="cuda") * 1.5 - 0.2
    ov = torch.randn(M, device="cuda")
    dOut = torch.full((M, Op), float("nan"), dtype=torch.bfloat16, device="cuda")
    mt = (M + 127) // 128
    cs = torch.zeros(mt, Op, device="cuda")
    nlp = torch.empty(M, device="cuda")
    nv = torch.empty(M, device="cuda")
    G.gemm(Hid, Wo, M, A + 1, H, False, False, Op, G.EPI_PPO, out=dOut, ldo=Op, out_cols=A + 1, bias=bias,
           colsum=cs, ld_colsum=Op, act_idx=act, adv=adv, ret=ret, olp=olp, ov=ov, A=A, vf=0.5, ent=0.01, clip=0.2,
           vfclip=0.2, newlp=nlp, newval=nv)
    torch.cuda.synchronize()
    # f64 reference through the oracle's per-row formula (one hidden layer with identity act is not needed:
    # feed the logits directly by evaluating the head in f64)
    out = (Hid.double() @ Wo.double().t() + bias.double())[:, :A + 1].cpu().numpy()
    a = act.cpu().numpy()
    lse = np.log(np.exp(out[:, :A]).sum(1))
    p = np.exp(out[:, :A] - lse[:, None])
    pout = (p * out[:, :A]).sum(1)
    logpA = out[np.arange(M), a] - lse
    ratio = np.exp(logpA - olp.double().cpu().numpy())
    advn = adv.double().cpu().numpy()
    lo, hi = 0.8, 1.2
    rc = np.clip(ratio, lo, hi)
    dPol = np.where(advn * ratio <= advn * rc, advn * ratio, advn * ((lo < ratio) & (ratio < hi)) * ratio)
    onehot = np.eye(A)[a]
    d = dPol[:, None] * (onehot - p) + 0.01 * p * (pout[:, None] - out[:, :A])
    vnew = out[:, A]
    retn, ovn = ret.double().cpu().numpy(), ov.double().cpu().numpy()
    dd = vnew - ovn
    vc = ovn + np.clip(dd, -0.2, 0.2)
    dv = np.where(((vnew - retn) ** 2 >= (vc - retn) ** 2) | ((dd > -0.2) & (dd < 0.2)), vnew - retn, 0.0)
    ref = np.concatenate([d, (-0.5 * dv)[:, None]], 1)
    got = dOut.float().cpu().numpy()
    assert np.abs(got[:, :A + 1] - ref).max() < 2e-2 * max(1.0, np.abs(ref).max())
    assert np.all(got[:, A + 1:] == 0)
    np.testing.assert_allclose(nlp.cpu().numpy(), logpA, rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(nv.cpu().numpy(), vnew, rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(cs.sum(0).cpu().numpy()[:A + 1], ref.sum(0), rtol=1e-3, atol=1e-3)


def test_gemm_batched_bf16():
    torch.manual_seed(9)
    nb, m, n = 3, 128, 256
    X = _bf(torch.randn(nb, m, n, device="cuda"))
    out = torch.empty(nb, m, m, dtype=torch.bfloat16, device="cuda")
    g = G.GemmArgs()
    g.a, g.a_rows, g.a_cols, g.a_ld, g.a_bstride, g.a_mn = X.data_ptr(), m, n, n, m * n, 0
    g.b, g.b_rows, g.b_cols, g.b_ld, g.b_bstride, g.b_mn = X.data_ptr(), m, n, n, m * n, 0
    g.M, g.N, g.K, g.bn, g.epi, g.batch, g.k_splits = m, m, n, 128, G.EPI_BF16, nb, 1
    g.out, g.ldo, g.out_bstride, g.out_rows, g.out_cols = out.data_ptr(), m, m * m, m, m
    g.alpha, g.beta = 1.0, 0.0
    G.run(g)
    torch.cuda.synchronize()
    ref = X.float() @ X.float().transpose(1, 2)
    assert _rel(out.float(), ref) < 1e-2
