"""Pins the C restatement (oracle/restate.c) to the reference's own outputs.

The golden fixtures were produced by the reference's compiled C on the seeded inputs of its
verify-* modes (tests/golden/gen_golden.py). Where the reference promises bit-exactness
(V-trace, Muon stepMat, shuffle, GAE, normalize) the restatement must match bit for bit.
"""
import os

import numpy as np
import pytest

from oracle import kat
from oracle import oracle as O

G = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(G, name + ".npz"))


def test_kat_inputs_regenerate_exactly():
    k = kat.kat_vtrace()
    f = load("vtrace")
    for x in ("rew", "val", "term", "imp"):
        assert np.array_equal(k[x], f[x])
    k = kat.kat_train_update()
    f = load("train_update")
    assert np.array_equal(k["pm0"], f["pm0"]) and np.array_equal(k["obs"], f["obs"])


def test_rng_matches_restatement():
    r = kat.Rng(0x5C1A)
    import ctypes as C

    s = C.c_uint64(0x5C1A)
    for _ in range(100):
        assert O.orc().orc_rng_next(C.byref(s)) == r.next()


def test_vtrace_bit_exact():
    f = load("vtrace")
    B, T, g, l, rho, c = f["meta"]
    out = O.vtrace(f["rew"], f["val"], f["term"], f["imp"], int(B), int(T), g, l, rho, c)
    assert np.array_equal(out, f["adv"])


def test_vtrace_mingru_bit_exact():
    f = load("vtrace_mingru")
    B, T, g, l, rho, c = f["meta"]
    out = O.vtrace_mingru(f["rew"], f["val"], f["term"], f["imp"], f["bootv"], int(B), int(T), g, l, rho, c)
    assert np.array_equal(out, f["adv"])


def test_muon_stepmat_bit_exact():
    f = load("muon_stepmat")
    lr, wd, mu, eps = f["meta"]
    for i in range(3):
        rows, cols = (int(x) for x in f[f"shape{i}"])
        nW, nM = O.muon_stepmat(f[f"W{i}"], f[f"G{i}"], f[f"M{i}"], rows, cols, lr, wd, mu, eps)
        n = rows * cols
        assert np.array_equal(nW, f[f"out{i}"][:n]), (rows, cols)
        assert np.array_equal(nM, f[f"out{i}"][n:]), (rows, cols)


def test_advnorm_bit_exact():
    f = load("advnorm")
    assert np.array_equal(O.normalize_adv(f["adv"]), f["out"])


def test_muon_whole_mlp_bit_exact():
    f = load("muon_cpu")
    H, D, Oo, gscale, lr, wd, mu, eps = f["meta"]
    H, D, Oo = int(H), int(D), int(Oo)
    P = f["params"].size
    g = f["grad"] * gscale  # muon_mat_cpu pre-scales G[i]*gscale (ffi/pufferblas.c:1376)
    pm = O.apply_muon(np.concatenate([f["params"], f["mom"]]), g, D, H, Oo - 1, 1, lr, wd, mu, eps)
    assert np.array_equal(pm[:P], f["out"][:P])
    assert np.array_equal(pm[P:], f["out"][P:])


def test_ppo_grad_matches_reference_blas():
    f = load("ppo_grad")
    N, D, H, A, vf, ent, clip, vfc = f["meta"]
    N, D, H, A = int(N), int(D), int(H), int(A)
    g, _, _ = O.mlp_ppo_grad(f["params"], f["obs"], f["acts"], f["advs"], f["rets"], f["olps"], N, D, H, A, 1, 0, vf,
                             ent, clip)
    np.testing.assert_allclose(g, f["g_blas"], rtol=1e-11, atol=1e-12)
    np.testing.assert_allclose(g, f["g_scalar"], rtol=1e-11, atol=1e-12)
    g2, nlp, nv = O.mlp_ppo_grad(f["params"], f["obs"], f["acts"], f["advs"], f["rets"], f["olps"], N, D, H, A, 1, 0,
                                 vf, ent, clip, ov=f["ov"], vfClip=vfc)
    P = g2.size
    np.testing.assert_allclose(g2, f["g_vclip"][:P], rtol=1e-11, atol=1e-12)
    np.testing.assert_allclose(nlp, f["g_vclip"][P:P + N], rtol=1e-13, atol=1e-14)
    np.testing.assert_allclose(nv, f["g_vclip"][P + N:], rtol=1e-13, atol=1e-14)


def test_train_step_matches_reference_composition():
    f = load("train_step")
    N, D, H, A, vf, ent, clip, lr, wd, mu, eps = f["meta"]
    N, D, H, A = int(N), int(D), int(H), int(A)
    advN = O.normalize_adv(f["adv"])
    assert np.array_equal(advN, f["advN"])
    g, _, _ = O.mlp_ppo_grad(f["params"], f["obs"], f["acts"], advN, f["rets"], f["olps"], N, D, H, A, 1, 0, vf, ent,
                             clip)
    np.testing.assert_allclose(g, f["grad"], rtol=1e-11, atol=1e-12)
    pm = O.apply_muon(np.concatenate([f["params"], f["mom"]]), O.grad_clip(g, 0.0, 1.0 / N), D, H, A, 1, lr, wd, mu,
                      eps)
    np.testing.assert_allclose(pm, f["out"], rtol=1e-9, atol=1e-10)


def test_train_update_matches_reference_composition():
    f = load("train_update")
    NT, D, H, A, E, MB, vf, ent, clip, lr, wd, mu, eps, seed = f["meta"]
    NT, D, H, A, E, MB = (int(x) for x in (NT, D, H, A, E, MB))
    perm = O.shuffle_perm(NT, E, int(seed))
    assert np.array_equal(perm, f["perm"])
    pm = O.train_update(f["pm0"], f["obs"], f["acts"], f["adv"], f["rets"], f["olps"], perm, NT, D, H, A, E, MB, lr,
                        wd, mu, eps, vf, ent, clip)
    np.testing.assert_allclose(pm, f["out"], rtol=1e-8, atol=1e-9)


def test_shuffle_bit_exact():
    f = load("shuffle")
    for i in range(3):
        NT, E, seed = (int(x) for x in f[f"args{i}"])
        assert np.array_equal(O.shuffle_perm(NT, E, seed), f[f"perm{i}"])


def test_gae_bit_exact():
    f = load("gae")
    N, T, g, l = f["meta"]
    out = O.gae_soa(f["vals"], f["rews"], f["terms"], int(N), int(T), g, l)
    assert np.array_equal(out, f["out"])
    # GAE is V-trace at rho = c = 1 (ffi/pufferffi.c:946 vs ffi/puffercuda.cu:69): same bits
    adv = O.vtrace(f["rews"], f["vals"], f["terms"], np.ones(int(N * T)), int(N), int(T), g, l, 1.0, 1.0)
    assert np.array_equal(adv, f["out"][:int(N * T)])


@pytest.mark.skipif(not O.ref_available(), reason="reference C not compiled on this host")
def test_reference_library_loads():
    lib = O.ref_cpu()
    assert hasattr(lib, "lean_ffi_mlp_ppo_grad_batch_blas")
