"""Multi-discrete heads on the MinGRU path (k_mg_ppo_b_md, ffi/puffercuda.cu:4940-4980) on the GPU against
the f64 oracle: the host-mode gradient (both tiers), a session gradient from a host sample with a repeated
segment, the whole update (device V-trace, sampling, gather of W-wide actions, BPTT, Muon), and the Lean
symbols (prep with a K-wide action column, host-mode gradient with head sizes).

Bars as for the categorical MinGRU head: tight tier 2e-3 relative (1e-4 floor) on the gradient and 1e-5 on
new log-probs and values; bf16 the reference's mixed bar on the small session batch and relative Frobenius
(2e-2 whole, 5e-2 per block) on the wider host batch; whole update 1e-3 (fp32) / 0.15 with cosine > 0.99
(bf16) on the parameter deltas."""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import kat  # noqa: E402
from oracle import oracle as O  # noqa: E402
from oracle.oracle import FA  # noqa: E402

pytestmark = pytest.mark.gpu
HS = [3, 2, 4]
A = sum(HS)
W = len(HS)


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def rel_floor(a, ref, floor=1e-4):
    return float(np.max(np.abs(a - ref) / (np.abs(ref) + floor)))


def mixed(a, ref):
    return float(np.max(np.abs(a - ref) / (2e-2 + 5e-2 * np.abs(ref))))


def _batch(D, H, L, T, B, K, seed):
    g = np.random.default_rng(seed)
    params, _ = O.init_mingru(D, H, L, A, 0x2000 + seed, K)
    R = T * B
    obs = g.uniform(-1, 1, R * D)
    acts = np.stack([g.integers(0, s, R) for s in HS], axis=1).astype(float).ravel()
    olp = sum(np.log(np.full(R, 1.0 / s)) for s in HS) + 0.2 * g.standard_normal(R)
    scal = np.concatenate([acts, g.uniform(-1.5, 1.5, R), g.uniform(-1, 2, R), olp, (g.random(R) < 0.1).astype(float),
                           g.uniform(-0.5, 0.5, R)])
    return params, obs, scal


@pytest.mark.parametrize("K", [3, 2])
def test_md_host_grad_tight(K):
    D, H, L, T, B = 12, 64, 2, 16, 24
    params, obs, scal = _batch(D, H, L, T, B, K, 5 + K)
    ref = O.mingru_grad_batch(params, obs, scal, B, T, H, D, L, A, K, hs=HS)
    out = plb.cuda_mingru_ppo_grad(params, obs, scal, B, T, H, D, L, A, 0.5, 0.01, 0.2, 0.2, bf16=0, K=K, hs=HS)
    P = params.size
    assert rel_floor(out[:P], ref[:P], 1e-3) < 2e-3, rel_floor(out[:P], ref[:P], 1e-3)
    np.testing.assert_allclose(out[P:], ref[P:], rtol=1e-5, atol=1e-5)


def frob(a, ref):
    return float(np.linalg.norm(a - ref) / max(np.linalg.norm(ref), 1e-30))


def test_md_host_grad_bf16():
    """The bf16 tier as the categorical head's wide test measures it: 2e-2 relative Frobenius on the whole
    gradient, 5e-2 per parameter block. Old log-probs sit within 0.1 of the new ones: with bf16 logits a
    three-head joint log-prob moves by ~1e-2, which switches any row whose ratio lies on a clip edge
    between its gradient and zero (that is the edge, not the arithmetic)."""
    D, H, L, T, B, K = 24, 128, 1, 16, 32, 3
    params, obs, scal = _batch(D, H, L, T, B, K, 9)
    P, R = params.size, T * B
    nl = O.mingru_grad_batch(params, obs, scal, B, T, H, D, L, A, K, hs=HS)[P:P + R]
    scal[(W + 2) * R:(W + 3) * R] = nl + np.random.default_rng(10).uniform(-0.1, 0.1, R)
    ref = O.mingru_grad_batch(params, obs, scal, B, T, H, D, L, A, K, hs=HS)
    out = plb.cuda_mingru_ppo_grad(params, obs, scal, B, T, H, D, L, A, 0.5, 0.01, 0.2, 0.2, bf16=1, K=K, hs=HS)
    assert frob(out[:P], ref[:P]) < 2e-2, frob(out[:P], ref[:P])
    sizes = [H * D, H] + [K * H * H] * L + [A * H, A, H, 1]
    off = 0
    for n in sizes:
        assert frob(out[off:off + n], ref[off:off + n]) < 5e-2, (off, n, frob(out[off:off + n], ref[off:off + n]))
        off += n
    np.testing.assert_allclose(out[P:], ref[P:], rtol=3e-2, atol=3e-2)


def _md_update_inputs():
    k = kat.kat_mingru_update()
    g = np.random.default_rng(0x3D)
    NT = k["N"] * k["T"]
    k["A"] = A
    k["act"] = np.stack([g.integers(0, s, NT) for s in HS], axis=1).astype(float).ravel()
    k["logp"] = sum(np.log(np.full(NT, 1.0 / s)) for s in HS) + 0.1 * g.standard_normal(NT)
    params, _ = O.init_mingru(k["D"], k["H"], k["L"], A, 0x6A5E, k["K"])
    k["pm0"] = np.concatenate([params, np.zeros(params.size)])
    return k


def _session(k):
    s = plb.MgSession(k["N"], k["T"])
    s.set_heads(W, HS)
    s.set_columns(k["rew"], k["term"], k["act"], k["logp"], k["val0"], k["boot"])
    s.set_obs(k["obs"], k["D"])
    return s


@pytest.mark.parametrize("bf16", [0, 1])
def test_md_session_grad_host_sample(bf16):
    k = _md_update_inputs()
    s = _session(k)
    try:
        T, D, H, L = k["T"], k["D"], k["H"], k["L"]
        net = plb.mg_net(D, H, L, A)
        params = k["pm0"][:O.mg_param_count(D, H, L, A)]
        s.vtrace(k["gamma"], k["lam"], k["rho"], k["c"])
        _, _, adv = s.state()
        seg = np.array([5.0, 2.0, 5.0, 9.0])
        mbp = np.array([1.0, 0.7, 1.3, 0.9])
        Bmb = seg.size
        s.grad(net, params=params, seg=seg, mbp=mbp, Bmb=Bmb, bf16=bf16)
        P = params.size
        g, nl, _ = s.grad_download(P, T * Bmb)
        sc = O.gather_seq_minibatch(k["act"], k["logp"], k["term"], adv, k["val0"], seg, mbp, T, Bmb, W=W)
        obsTB = np.zeros(T * Bmb * D)
        for t in range(T):
            for b in range(Bmb):
                e = int(seg[b])
                obsTB[(t * Bmb + b) * D:(t * Bmb + b + 1) * D] = k["obs"][(e * T + t) * D:(e * T + t + 1) * D]
        ref = O.mingru_grad_batch(params, obsTB, sc, Bmb, T, H, D, L, A, hs=HS)
        if bf16:
            assert mixed(g, ref[:P]) < 1.0
        else:
            assert rel_floor(g, ref[:P]) < 2e-3, rel_floor(g, ref[:P])
        tol = 3e-2 if bf16 else 1e-5
        np.testing.assert_allclose(nl, ref[P:P + T * Bmb], rtol=tol, atol=tol)
    finally:
        s.close()


@pytest.mark.parametrize("bf16,tol", [(0, 1e-3), (1, 0.15)])
def test_md_whole_update_vs_oracle(bf16, tol):
    k = _md_update_inputs()
    s = _session(k)
    try:
        D, H, L = k["D"], k["H"], k["L"]
        net = plb.mg_net(D, H, L, A)
        P = O.mg_param_count(D, H, L, A)
        hy = plb.MgHyper(gamma=k["gamma"], lam=k["lam"], rhoClip=k["rho"], cClip=k["c"], prioAlpha=k["alpha"],
                         annealBeta=k["beta"], wd=k["wd"], mu=k["mu"], eps=k["eps"], vfCoef=k["vf"], entCoef=k["ent"],
                         clipEps=k["clip"], vfClip=k["vfClip"], maxGradNorm=k["maxGradNorm"], ns_coeffs=None,
                         ns_iters=0, bf16=bf16)
        h = plb.policy_load(k["pm0"], P)
        try:
            rng = s.update(net, h, hy, k["numMB"], k["mbSegs"], k["rng"], k["lr"])
            out = plb.policy_download(h, P)
        finally:
            plb.policy_free(h)
        ref, rref = O.mingru_update(k["pm0"], k["obs"], k["rew"], k["term"], k["act"], k["logp"], k["val0"], k["boot"],
                                    k["N"], k["T"], D, H, L, A, k["numMB"], k["mbSegs"], k["rng"], k["lr"], hs=HS)
        assert rng == rref
        d_ref, d_out = ref[:P] - k["pm0"][:P], out[:P] - k["pm0"][:P]
        rel = np.linalg.norm(d_out - d_ref) / np.linalg.norm(d_ref)
        assert rel < tol, rel
        assert float(d_out @ d_ref / (np.linalg.norm(d_out) * np.linalg.norm(d_ref))) > 0.99
    finally:
        s.close()


def test_md_lean_symbols(monkeypatch):
    """lean_cuda_mg_prep with a K-wide action column, then lean_cuda_mingru_ppo_grad in host mode with
    K = 3 head sizes (fp32 tier), against the oracle."""
    monkeypatch.setenv("PUFFER_MG_BF16", "0")
    plb.lib()
    L = C.CDLL(os.path.join(os.path.dirname(plb.LIB_PATH), "libpufferlean_lean.so"))
    VP = C.c_void_p
    k = _md_update_inputs()
    r = O.ref_call(L, "lean_cuda_mg_prep", VP, FA(k["rew"]), FA(k["term"]), FA(k["act"]), FA(k["logp"]),
                   FA(k["val0"]), FA(k["boot"]), k["N"], k["T"], W, ("obj", 1))
    assert O.ctor_tag(r) == 0
    D, H, Lh, T, B = 12, 64, 2, 8, 6
    params, obs, scal = _batch(D, H, Lh, T, B, 3, 21)
    ref = O.mingru_grad_batch(params, obs, scal, B, T, H, D, Lh, A, 3, hs=HS)
    r = O.ref_call(L, "lean_cuda_mingru_ppo_grad", VP, FA(params), FA(obs), FA(scal), B, T, H, D, Lh, A, W,
                   FA(np.array(HS, dtype=float)), 0.5, 0.01, 0.2, 0.2, FA(np.zeros(0)), FA(np.zeros(0)), ("obj", 1))
    assert O.ctor_tag(r) == 0
    out = O.read_float_array(O.ctor_field(r, 0))
    P = params.size
    assert rel_floor(out[:P], ref[:P], 1e-3) < 2e-3
    np.testing.assert_allclose(out[P:], ref[P:], rtol=1e-5, atol=1e-5)
