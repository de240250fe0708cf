"""Wide action heads on the CPU: the oracle's restatement against the reference's own C (golden fixtures),
the multi-discrete head against the pinned categorical gradient and against finite differences of the
PPO objective, and the host-side argument checks of the C-ABI entry points (no device work)."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_gauss_grad_oracle_matches_reference_c():
    """orc_mlp_ppo_grad_wide mode 2 is lean_ffi_gauss_ppo_grad_batch(_vclip) (ffi/pufferffi.c:311-360) bit for
    bit: the gradient without the value clip, and gradient, new log-probs and new values with it. Includes a raw log-std above
    the clamp's upper end (gradient cut)."""
    f = np.load(os.path.join(GOLD, "gauss_grad.npz"))
    N, D, H, W = (int(x) for x in f["meta"][:4])
    vf, ent, clip, vfc = f["meta"][4:]
    Og = 2 * W + 1
    P = H * D + H + Og * H + Og
    args = [f[x] for x in ("params", "obs", "acts", "advs", "rets", "olps")]
    g, nl, nv = O.mlp_ppo_grad_wide(*args, N, D, H, Og, W, 2, vf=vf, ent=ent, clip=clip, lsLo=-5.0)
    assert f["g_plain"].size == P and np.array_equal(g, f["g_plain"])  # the unclipped form returns g alone
    g, nl, nv = O.mlp_ppo_grad_wide(*args, N, D, H, Og, W, 2, ov=f["ov"], vf=vf, ent=ent, clip=clip, vfClip=vfc,
                                    lsLo=-5.0)
    assert np.array_equal(np.concatenate([g, nl, nv]), f["g_vclip"])
    # the upper clamp really is exercised: some rows' third raw log-std is above 2, others below
    pr = f["params"]
    Hh = np.maximum(f["obs"].reshape(N, D) @ pr[:H * D].reshape(H, D).T + pr[H * D:H * D + H], 0.0)
    raw = Hh @ pr[H * D + H:H * D + H + Og * H].reshape(Og, H)[W + 2] + pr[H * D + H + Og * H + W + 2]
    assert np.any(raw > 2.0) and np.any(raw < 2.0) and np.all(raw > -5.0)


def test_gauss_update_oracle_matches_reference_composition():
    """orc_train_update_wide mode 2 over 2 epochs x 4 minibatches (value clip on) equals the update composed
    from the reference's C: lean_cuda_adv_normalize, lean_ffi_gauss_ppo_grad_batch_vclip and
    lean_ffi_muon_step_mlp (the stepMat / stepVec of muonStepMlpBlasFFI) with gscale 1/n."""
    f = np.load(os.path.join(GOLD, "gauss_update.npz"))
    NT, D, H, W, E, MB = (int(x) for x in f["meta"])
    lr, wd, mu, eps, vf, ent, clip, vfc = f["hyp"]
    out = O.train_update_wide(f["pm0"], f["obs"], f["acts"], f["adv"], f["ret"], f["olp"], f["perm"], NT, D, H,
                              2 * W + 1, W, 2, E, MB, ov=f["ov"], lr=lr, wd=wd, mu=mu, eps=eps, vf=vf, ent=ent,
                              clip=clip, vfClip=vfc, maxGradNorm=0.0, lsLo=-5.0)
    assert np.array_equal(out, f["out"])


def _cat_inputs(seed, N, D, H, O_, W, hs=None):
    g = np.random.default_rng(seed)
    P = H * D + H + O_ * H + O_
    params = g.uniform(-0.4, 0.4, P)
    obs = g.uniform(-1, 1, N * D)
    if hs is None:
        acts = g.standard_normal(N * W)
    else:
        acts = np.stack([g.integers(0, s, N) for s in hs], axis=1).astype(float).ravel()
    return params, obs, acts, g.standard_normal(N), g.standard_normal(N), g.uniform(-4, -1, N), g.standard_normal(N)


@pytest.mark.parametrize("vfClip", [0.0, 0.2])
def test_md_single_head_is_the_categorical_gradient(vfClip):
    """One multi-discrete head of size A is the categorical head: the pinned orc_mlp_ppo_grad (which matches
    lean_ffi_mlp_ppo_grad_batch) to rounding (the two sum the forward in opposite orders)."""
    N, D, H, A = 19, 5, 12, 6
    params, obs, acts, adv, ret, olp, ov = _cat_inputs(4, N, D, H, A + 1, 1, hs=[A])
    gw, nlw, nvw = O.mlp_ppo_grad_wide(params, obs, acts, adv, ret, olp, N, D, H, A + 1, 1, 1, hs=[A],
                                       ov=ov if vfClip else None, vfClip=vfClip)
    gc, nlc, nvc = O.mlp_ppo_grad(params, obs, acts, adv, ret, olp, N, D, H, A, ov=ov if vfClip else None,
                                  vfClip=vfClip)
    np.testing.assert_allclose(gw, gc, rtol=1e-11, atol=1e-12)
    np.testing.assert_allclose(nlw, nlc, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(nvw, nvc, rtol=1e-12, atol=1e-12)


def _objective(params, obs, acts, adv, ret, olp, N, D, H, O_, W, mode, hs, vf, ent, clip, lsLo):
    """The PPO objective the wide heads ascend: sum over rows of min(adv r, adv clip(r)) + ent * entropy
    - vf/2 (v - ret)^2, entropy summed over heads (per-dim log-std for the Gaussian, up to a constant)."""
    W1 = params[:H * D].reshape(H, D)
    b1 = params[H * D:H * D + H]
    W2 = params[H * D + H:H * D + H + O_ * H].reshape(O_, H)
    b2 = params[H * D + H + O_ * H:]
    X = obs.reshape(N, D)
    Hh = np.maximum(X @ W1.T + b1, 0.0)
    out = Hh @ W2.T + b2
    a = acts.reshape(N, W)
    if mode == 1:
        logp, entr, off = np.zeros(N), np.zeros(N), 0
        for h, s in enumerate(hs):
            z = out[:, off:off + s]
            lse = np.log(np.exp(z).sum(1))
            logp += z[np.arange(N), a[:, h].astype(int)] - lse
            p = np.exp(z - lse[:, None])
            entr += -(p * (z - lse[:, None])).sum(1)
            off += s
    else:
        ls = np.clip(out[:, W:2 * W], lsLo, 2.0)
        zz = (a - out[:, :W]) * np.exp(-ls)
        logp = (-0.5 * zz * zz - ls - 0.5 * np.log(2 * np.pi)).sum(1)
        entr = ls.sum(1)
    r = np.exp(logp - olp)
    surr = np.minimum(adv * r, adv * np.clip(r, 1 - clip, 1 + clip))
    return float(np.sum(surr + ent * entr - vf * 0.5 * (out[:, -1] - ret) ** 2))


@pytest.mark.parametrize("mode", [1, 2])
def test_wide_gradient_is_the_objective_gradient(mode):
    """Central finite differences of the objective above against the oracle's analytic gradient, on rows
    whose ratio sits away from the clip edges."""
    N, D, H, W = 9, 4, 6, 3
    hs = [3, 4, 2] if mode == 1 else None
    O_ = (sum(hs) if mode == 1 else 2 * W) + 1
    params, obs, acts, adv, ret, olp, _ = _cat_inputs(11 + mode, N, D, H, O_, W, hs=hs)
    _, nl, _ = O.mlp_ppo_grad_wide(params, obs, acts, adv, ret, olp, N, D, H, O_, W, mode, hs=hs)
    olp = nl + np.random.default_rng(5).uniform(-0.1, 0.1, N)  # ratios in (0.9, 1.1): inside the clip band
    g, _, _ = O.mlp_ppo_grad_wide(params, obs, acts, adv, ret, olp, N, D, H, O_, W, mode, hs=hs)
    fd = np.zeros_like(params)
    h = 1e-6
    for i in range(params.size):
        p1, p0 = params.copy(), params.copy()
        p1[i] += h
        p0[i] -= h
        fd[i] = (_objective(p1, obs, acts, adv, ret, olp, N, D, H, O_, W, mode, hs, 0.5, 0.01, 0.2, -20.0)
                 - _objective(p0, obs, acts, adv, ret, olp, N, D, H, O_, W, mode, hs, 0.5, 0.01, 0.2, -20.0)) / (2 * h)
    np.testing.assert_allclose(g, fd, rtol=1e-5, atol=1e-6)


def test_wide_entry_points_reject_bad_modes_on_the_host():
    """Argument checks run before any device work: an unknown head mode and a NULL gradient buffer."""
    import pufferlean_b200 as plb
    L = plb.lib()
    one = np.zeros(8)
    p = one.ctypes.data_as(C.POINTER(C.c_double))
    rc = L.pl_train_update_wide_resident(1, p, p, p, p, p, None, 0, p, p, 4, 1, 1, 3, 1, 3, 1, 1, 0.1, 0.0, 0.9, 1e-7,
                                         0.5, 0.01, 0.2, 0.0, 0.0, 0, None)
    assert rc != 0 and b"mode" in L.pl_last_error()
    rc = L.pl_mlp_ppo_grad_wide(p, p, p, p, p, p, None, 1, 1, 1, 3, 1, 2, None, 0.5, 0.01, 0.2, 0.0, 0, None)
    assert rc != 0
