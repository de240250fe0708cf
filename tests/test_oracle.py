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


# ---------------------------------------------------------------------------------------------- MinGRU
def test_mingru_kat_inputs_regenerate_exactly():
    k = kat.kat_mingru_grad()
    f = load("mingru_grad")
    assert np.array_equal(k["params"], f["params"])
    assert np.array_equal(k["obsTB"], f["obsTB"]) and np.array_equal(k["scal"], f["scal"])


def test_mingru_grad_seq_bit_exact():
    """orc_mingru_grad_seq == the reference's lean_ffi_mingru_ppo_grad_seq (ffi/pufferffi.c:763-876) on the
    verify-mingru-grad-gpu inputs, gradient and new log-prob / value, every bit."""
    k = kat.kat_mingru_grad()
    f = load("mingru_grad")
    s = k["seqs"]
    P = O.mg_param_count(k["D"], k["H"], k["L"], k["A"])
    for b in range(k["B"]):
        g, nl, nv = O.mingru_grad_seq(k["params"], s["obs"][b], s["act"][b], s["adv"][b], s["ret"][b], s["old"][b],
                                      s["term"][b], s["ov"][b], k["T"], k["H"], k["D"], k["L"], k["A"])
        ref = f[f"seq{b}"]
        assert np.array_equal(g, ref[:P])
        assert np.array_equal(nl, ref[P:P + k["T"]]) and np.array_equal(nv, ref[P + k["T"]:])


def test_mingru_grad_batch_is_sum_of_sequences():
    k = kat.kat_mingru_grad()
    f = load("mingru_grad")
    P = O.mg_param_count(k["D"], k["H"], k["L"], k["A"])
    out = O.mingru_grad_batch(k["params"], k["obsTB"], k["scal"], k["B"], k["T"], k["H"], k["D"], k["L"], k["A"])
    assert np.array_equal(out[:P], 0.0 + f["seq0"][:P] + f["seq1"][:P])
    T, B = k["T"], k["B"]
    for b in range(B):
        assert np.array_equal(out[P + b:P + T * B:B], f[f"seq{b}"][P:P + T])


def test_mingru_variants_reduce_correctly():
    """K = 2 (no highway) and the GELU encoder have no reference counterpart; check them against a central
    finite difference of the primal objective they differentiate (the reference's own AD-vs-FD discipline,
    Puffer/RL/MinGRUTrain.lean:346-380). Tiny net, no terminal, no clipping active, ent = 0, so the
    objective is sum_t adv_t exp(logp_t - old_t) - (vf / 2) sum_t (v_t - ret_t)^2 with vf = 0.5."""
    rng = np.random.default_rng(5)
    D, H, L, A, T = 3, 4, 2, 3, 4
    for K, enc in ((2, 0), (3, 1), (2, 1)):
        params, _ = O.init_mingru(D, H, L, A, 0x77 + K + enc, K)
        obs = rng.uniform(-1, 1, T * D)
        acts = rng.integers(0, A, T).astype(float)
        adv = rng.uniform(-1, 1, T)
        ret = rng.uniform(0, 1, T)
        old = np.full(T, -1.1)
        term, ov = np.zeros(T), np.zeros(T)

        def run(p):
            return O.mingru_grad_seq(p, obs, acts, adv, ret, old, term, ov, T, H, D, L, A, K, enc, vf=0.5, ent=0.0,
                                     clip=10.0, vfClip=0.0)

        def objective(p):
            _, lp, v = run(p)
            return np.sum(adv * np.exp(lp - old)) - 0.25 * np.sum((v - ret) ** 2)

        g, _, _ = run(params)
        for i in rng.choice(params.size, 12, replace=False):
            h = 1e-6
            pp, pm_ = params.copy(), params.copy()
            pp[i] += h
            pm_[i] -= h
            fd = (objective(pp) - objective(pm_)) / (2 * h)
            assert abs(fd - g[i]) <= 1e-6 + 1e-5 * abs(fd), (K, enc, i, fd, g[i])


def test_gather_seq_minibatch_bit_exact():
    f = load("gather_seq")
    N, T, D, Bmb = (int(x) for x in f["meta"])
    out = O.gather_seq_minibatch(f["act"], f["logp"], f["term"], f["adv"], f["value"], f["seg"], f["mbPrio"], T, Bmb)
    assert np.array_equal(out, f["out"])


def test_prio_sample_bit_exact():
    f = load("prio")
    m = f["meta"]
    seg, mp = O.prio_sample(f["L1"], int(m[0]), int(m[2]), m[3], m[4], int(m[5]))
    assert np.array_equal(seg, f["idx"]) and np.array_equal(mp, f["mbPrio"])


def test_mingru_update_matches_reference_composition():
    """orc_mingru_update == the update composed from the reference's own C (V-trace, prioritised sampling,
    scalar gather, per-sequence BPTT, stepMat) and its Lean formulas (gradClipMG, stepVec, iterate)."""
    k = kat.kat_mingru_update()
    pm, r = O.mingru_update(k["pm0"], k["obs"], k["rew"], k["term"], k["act"], k["logp"], k["val0"], k["boot"],
                            k["N"], k["T"], k["D"], k["H"], k["L"], k["A"], k["numMB"], k["mbSegs"], k["rng"], k["lr"])
    f = load("mingru_update")
    assert np.array_equal(pm, f["out"]) and r == int(f["rng_out"][0])
