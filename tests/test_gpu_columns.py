"""The rollout-side column producer (the reference's device column stamping, ffi/puffercuda.cu:242-309,
and obs-trajectory scatter, :975-983): the generic scatters against the host layout, and a MinGRU session
whose columns are stamped step by step (envs in two chunks, one- and three-head action columns) against
the same session filled by the host upload — the whole update must agree bit for bit — plus the Lean
cols_ready handshake."""
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


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _d(a, dtype=torch.float64):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).cuda()


def test_generic_scatters():
    N, T, W = 7, 5, 3
    g = np.random.default_rng(1)
    col = torch.full((N * T * W,), -1.0, dtype=torch.float64, device="cuda")
    ref = np.full((N * T, W), -1.0)
    L = plb.lib()
    for s in range(T):
        for e0, ne in ((0, 3), (3, 4)):
            src = g.standard_normal((ne, W))
            d = _d(src)
            assert L.pl_stamp_rows_f64(col.data_ptr(), W, N, T, s, e0, ne, d.data_ptr(), None) == 0
            ref[[(e0 + i) * T + s for i in range(ne)]] = src
    assert np.array_equal(col.cpu().numpy().reshape(N * T, W), ref)
    obs = torch.zeros(N * T * 4, dtype=torch.float32, device="cuda")
    src = g.standard_normal((N, 4)).astype(np.float32)
    assert L.pl_stamp_rows_f32(obs.data_ptr(), 4, N, T, 2, 0, N, _d(src, torch.float32).data_ptr(), None) == 0
    o = obs.cpu().numpy().reshape(N * T, 4)
    assert np.array_equal(o[[e * T + 2 for e in range(N)]], src)
    plane = g.standard_normal((T, N))
    out = torch.zeros(N * T, dtype=torch.float64, device="cuda")
    assert L.pl_stamp_plane_f64(out.data_ptr(), N, T, _d(plane).data_ptr(), None) == 0
    assert np.array_equal(out.cpu().numpy().reshape(N, T), plane.T)
    # bounds are checked on the host
    assert L.pl_stamp_rows_f64(col.data_ptr(), W, N, T, T, 0, 1, _d(src).data_ptr(), None) != 0
    assert L.pl_stamp_rows_f64(col.data_ptr(), W, N, T, 0, 5, 3, _d(src).data_ptr(), None) != 0


def _inputs(hs):
    k = kat.kat_mingru_update()
    N, T = k["N"], k["T"]
    if hs:
        g = np.random.default_rng(8)
        k["A"] = sum(hs)
        k["act"] = np.stack([g.integers(0, s, N * T) for s in hs], axis=1).astype(float).ravel()
        params, _ = O.init_mingru(k["D"], k["H"], k["L"], k["A"], 0x6A5E, k["K"])
        k["pm0"] = np.concatenate([params, np.zeros(params.size)])
    return k


def _update(s, k, bf16):
    D, H, L, A = k["D"], k["H"], k["L"], k["A"]
    net = plb.mg_net(D, H, L, A)
    P = O.mg_param_count(D, H, L, A)
    hy = plb.MgHyper(gamma=k["gamma"], lam=k["lam"], rhoClip=k["rho"], cClip=k["c"], prioAlpha=k["alpha"],
                     annealBeta=k["beta"], wd=k["wd"], mu=k["mu"], eps=k["eps"], vfCoef=k["vf"], entCoef=k["ent"],
                     clipEps=k["clip"], vfClip=k["vfClip"], maxGradNorm=k["maxGradNorm"], ns_coeffs=None, ns_iters=0,
                     bf16=bf16)
    h = plb.policy_load(k["pm0"], P)
    try:
        s.update(net, h, hy, k["numMB"], k["mbSegs"], k["rng"], k["lr"])
        return plb.policy_download(h, P)
    finally:
        plb.policy_free(h)


@pytest.mark.parametrize("hs,bf16", [(None, 0), (None, 1), ([2, 3, 2], 1)])
def test_stamped_session_equals_uploaded(hs, bf16):
    k = _inputs(hs)
    N, T, D = k["N"], k["T"], k["D"]
    W = len(hs) if hs else 1
    up = plb.MgSession(N, T)
    st = plb.MgSession(N, T)
    try:
        if hs:
            up.set_heads(W, hs)
            st.set_heads(W, hs)
        up.set_columns(k["rew"], k["term"], k["act"], k["logp"], k["val0"], k["boot"])
        up.set_obs(k["obs"], D)
        assert not up.take_stamped()
        act = k["act"].reshape(N, T, W)
        obs = k["obs"].reshape(N, T, D).astype(np.float32)
        logp, val = k["logp"].reshape(N, T), k["val0"].reshape(N, T)
        keep = []
        for s in range(T):
            for e0, ne in ((0, 5), (5, N - 5)):
                arrs = [_d(act[e0:e0 + ne, s]), _d(logp[e0:e0 + ne, s]), _d(val[e0:e0 + ne, s]),
                        _d(obs[e0:e0 + ne, s], torch.float32)]
                keep += arrs
                st.stamp_step(s, e0, ne, *[a.data_ptr() for a in arrs[:3]], arrs[3].data_ptr(), D)
        rew_p, term_p = _d(k["rew"].reshape(N, T).T.copy()), _d(k["term"].reshape(N, T).T.copy())
        boot = _d(k["boot"])
        st.stamp_finish(rew_p.data_ptr(), term_p.data_ptr(), boot.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(np.concatenate(st.state()[:2]), np.concatenate(up.state()[:2]))
        a = _update(up, k, bf16)
        b = _update(st, k, bf16)
        assert np.array_equal(a, b)
        assert st.take_stamped() and not st.take_stamped()
    finally:
        up.close()
        st.close()


def test_lean_cols_ready_handshake():
    plb.lib()
    L = C.CDLL(os.path.join(os.path.dirname(plb.LIB_PATH), "libpufferlean_lean.so"))
    VP = C.c_void_p
    k = _inputs(None)
    N, T = k["N"], k["T"]
    r = O.ref_call(L, "lean_cuda_mg_prep", VP, FA(k["rew"]), FA(k["term"]), FA(k["act"]), FA(k["logp"]),
                   FA(k["val0"]), FA(k["boot"]), N, T, 1, ("obj", 1))
    assert O.ctor_tag(r) == 0

    def ready():
        rr = O.ref_call(L, "lean_cuda_mg_cols_ready", VP, N, T, ("obj", 1))
        return int(O.ctor_field(rr, 0)) >> 1  # a boxed scalar

    assert ready() == 0  # uploaded by prep, not stamped
    L.pl_lean_mg_session.restype = C.c_void_p
    sess = L.pl_lean_mg_session()
    lib = plb.lib()
    z = torch.zeros(N, dtype=torch.float64, device="cuda")
    for s in range(T):
        assert lib.pl_mg_stamp_step(sess, s, 0, N, z.data_ptr(), z.data_ptr(), z.data_ptr(), None, 0, None) == 0
    planes = torch.zeros(N * T, dtype=torch.float64, device="cuda")
    assert lib.pl_mg_stamp_finish(sess, planes.data_ptr(), planes.data_ptr(), z.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert ready() == 1
    assert ready() == 0  # read once
