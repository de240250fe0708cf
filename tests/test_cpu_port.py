"""The numpy CPU port (oracle/cpu_port.py) does the reference's work: its PPO-objective gradient and
its Muon step agree with the reference's own compiled C (golden fixtures) and with the pinned C
restatement (oracle/restate.c) to 1e-11 relative, for the reference's one-hidden-layer ReLU network
and for the deep GELU networks of the bench configuration. The port is what the CPU baseline times
and what the full-width GPU parity tests compare against, so this pins both to the reference."""
import os

import numpy as np
import pytest

from oracle import cpu_port
from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def test_port_gradient_equals_reference_blas_gradient():
    """lean_ffi_mlp_ppo_grad_batch_blas and its value-clipped twin (ffi/pufferblas.c:699-747) on the
    verify-ppo-grad inputs."""
    f = np.load(os.path.join(GOLD, "ppo_grad.npz"))
    N, D, H, A, vf, ent, clip, vfclip = f["meta"]
    N, D, H, A = int(N), int(D), int(H), int(A)
    args = (f["params"], f["obs"].reshape(N, D), f["acts"], f["advs"], f["rets"], f["olps"], D, H, A, 1, 0)
    g = cpu_port.ppo_grad(*args, vf=vf, ent=ent, clip=clip)
    assert rel(g, f["g_blas"]) < 1e-11
    g = cpu_port.ppo_grad(*args, vf=vf, ent=ent, clip=clip, ov=f["ov"], vfclip=vfclip)
    assert rel(g, f["g_vclip"][:g.size]) < 1e-11  # the vclip form appends new log-probs and values


def test_port_muon_step_equals_reference_muon_step_mlp():
    """lean_ffi_muon_step_mlp (ffi/pufferblas.c:1411-1428, muon_mat_cpu per matrix) with its gradient
    scale and coefficient table."""
    f = np.load(os.path.join(GOLD, "muon_cpu.npz"))
    H, D, O_, gscale, lr, wd, mu, eps = f["meta"]
    H, D, A = int(H), int(D), int(O_) - 1
    pm = np.concatenate([f["params"], f["mom"]])
    got = cpu_port.muon_step(pm.copy(), f["grad"], D, H, A, 1, lr, wd, mu, eps, O.MUON_COEFFS, 0.0, gscale)
    P = f["params"].size
    assert rel(got[:P], f["out"][:P]) < 1e-11
    assert rel(got[P:], f["out"][P:]) < 1e-11


@pytest.mark.parametrize("L,act,vfclip", [(1, 0, 0.0), (1, 0, 0.2), (3, 1, 0.2), (5, 1, 0.0)])
def test_port_gradient_equals_restatement(L, act, vfclip):
    g = np.random.default_rng(40 + L)
    N, D, H, A = 300, 24, 40, 9
    P = O.param_count(D, H, A, L)
    params = g.uniform(-0.3, 0.3, P)
    obs = g.standard_normal(N * D)
    acts = g.integers(0, A, N).astype(float)
    adv, ret = g.standard_normal(N), g.standard_normal(N)
    olp = np.log(np.full(N, 1.0 / A)) + g.normal(0, 0.2, N)
    ov = ret + g.normal(0, 0.3, N)
    want, _, _ = O.mlp_ppo_grad(params, obs, acts, adv, ret, olp, N, D, H, A, L=L, act=act, ov=ov, vfClip=vfclip)
    got = cpu_port.ppo_grad(params, obs.reshape(N, D), acts, adv, ret, olp, D, H, A, L, act, ov=ov, vfclip=vfclip)
    assert rel(got, want) < 1e-11


@pytest.mark.parametrize("L,maxgn", [(1, 0.0), (3, 0.5)])
def test_port_muon_step_equals_restatement(L, maxgn):
    """The clipped mean gradient and the whole-network Muon step (grad_clip + apply_muon of the
    restatement) with BASELINE's quintic table, including a tall and a wide matrix."""
    g = np.random.default_rng(60 + L)
    D, H, A, N = 24, 40, 9, 300
    P = O.param_count(D, H, A, L)
    pm = np.concatenate([g.uniform(-0.3, 0.3, P), g.normal(0, 0.01, P)])
    grad = g.standard_normal(P)
    want = O.apply_muon(pm, O.grad_clip(grad, maxgn, 1.0 / N), D, H, A, L, 0.02, 0.01, 0.95, 1e-7,
                        O.QUINTIC_COEFFS)
    got = cpu_port.muon_step(pm.copy(), grad, D, H, A, L, 0.02, 0.01, 0.95, 1e-7, O.QUINTIC_COEFFS, maxgn, 1.0 / N)
    assert rel(got[:P], want[:P]) < 1e-11
    assert rel(got[P:], want[P:]) < 1e-11


@pytest.mark.parametrize("rows,cols", [(64, 256), (256, 64), (96, 96)])
def test_port_newton_schulz_equals_restatement(rows, cols):
    """The port's orthogonalisation (tall matrices through their transpose, (bA + cA^2)X) against the
    restatement's (the reference's A = X^T X form for tall matrices, a X + b(AX) + c A(AX))."""
    g = np.random.default_rng(rows * cols)
    X = g.standard_normal((rows, cols))
    want = O.newton_schulz(X.ravel(), rows, cols, 1e-7, O.QUINTIC_COEFFS).reshape(rows, cols)
    got = cpu_port.newton_schulz(X, O.QUINTIC_COEFFS, 1e-7)
    assert rel(got, want) < 1e-11


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("maxgn,NT,MB", [(0.0, 256, 4), (0.5, 301, 3)])
def test_reference_c_update_composition_equals_restatement(maxgn, NT, MB):
    """oracle/ref_update.py (the configs[0] CPU baseline: the reference's compiled C called in its CPU
    trainer's order) against the restatement's whole update with the same GAE and shuffle."""
    from oracle import ref_update as R

    g = np.random.default_rng(NT)
    T = 16 if NT % 16 == 0 else 7
    N = NT // T
    NT = N * T
    D, H, A, E = 4, 32, 2, 2
    P = O.param_count(D, H, A, 1)
    pm = np.concatenate([g.uniform(-0.3, 0.3, P), np.zeros(P)])
    obs, acts = g.standard_normal(NT * D), g.integers(0, A, NT).astype(float)
    olps = np.log(0.5) + 0.05 * g.standard_normal(NT)
    vals, rews, terms = g.standard_normal(NT), (g.random(NT) < 0.5).astype(float), (g.random(NT) < 0.05).astype(float)
    got = R.update(pm.copy(), obs, acts, olps, vals, rews, terms, N, T, D, H, A, E, MB, 77, eps=1e-12,
                   max_grad_norm=maxgn)
    ga = O.gae_soa(vals, rews, terms, N, T, 0.995, 0.90)
    perm = O.shuffle_perm(NT, E, 77)
    want = O.train_update(pm, obs, acts, ga[:NT], ga[NT:], olps, perm, NT, D, H, A, E, MB, 0.02, 0.0, 0.95, 1e-12,
                          0.5, 0.01, 0.2, maxGradNorm=maxgn)
    assert rel(got, want) < 1e-11
