"""Numerics at the headline configuration's own widths (configs[4]: observations of 1024, five
hidden GELU layers 1024 -> 2048 -> ... -> 2048, 64 actions + value, BASELINE's quintic Newton-Schulz),
on a reduced row count, against the CPU port (oracle/cpu_port.py, f64, pinned to the reference's C and
to the restatement by tests/test_cpu_port.py).

* One minibatch from zero momentum: the momentum after the step is the mean gradient, so each
  parameter block of the bf16 tier's gradient (K = 1024 and 2048 accumulations, the 64-action PPO head
  epilogue, five chained data-gradient GEMMs) is checked against f64 at the 2e-2 relative Frobenius bar.
* The same step's weight deltas (Newton-Schulz of 2048 x 2048, 2048 x 1024 and 65 x 2048 momenta).
* Newton-Schulz alone at the configs' matrix shapes (512 x 2048 of configs[2]; 2048 x 2048 and
  2048 x 1024 of configs[4]) against f64, at the 2e-2 bar.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import cpu_port  # noqa: E402
from oracle import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

D, H, A, L, ACT = 1024, 2048, 64, 5, 1
QUINTIC = np.ascontiguousarray(O.QUINTIC_COEFFS)


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


class _Arch(C.Structure):
    _fields_ = [("L", C.c_size_t), ("act", C.c_int), ("ns_coeffs", C.POINTER(C.c_double)), ("ns_iters", C.c_size_t)]


def _problem(NT, seed):
    g = np.random.default_rng(seed)
    lay, P = cpu_port.layers_of(D, H, A, L)
    pm = np.zeros(2 * P)
    for oW, ob, fout, fin in lay:  # Xavier-uniform weights (BASELINE's init), small biases
        lim = np.sqrt(6.0 / (fin + fout))
        pm[oW:oW + fout * fin] = g.uniform(-lim, lim, fout * fin)
        pm[ob:ob + fout] = g.uniform(-0.05, 0.05, fout)
    obs = g.standard_normal(NT * D)
    acts = g.integers(0, A, NT).astype(float)
    adv, ret = g.standard_normal(NT), g.standard_normal(NT)
    olp = np.log(np.full(NT, 1.0 / A)) + g.normal(0, 0.1, NT)
    ov = ret + g.normal(0, 0.3, NT)
    return lay, P, pm, obs, acts, adv, ret, olp, ov


def _device_update(pm, P, obs, acts, adv, ret, olp, ov, perm, NT, lr, vfclip, maxgn):
    h = plb.policy_load(pm, P)
    try:
        Lb = plb.lib()
        Lb.pl_train_update_resident_deep.argtypes = ([C.c_size_t, C.POINTER(_Arch)] + [C.POINTER(C.c_double)] * 6 +
                                                     [C.c_size_t, C.POINTER(C.c_double)] + [C.c_size_t] * 6 +
                                                     [C.c_double] * 9 + [C.c_uint8, C.POINTER(C.c_double)])
        arch = _Arch(L, ACT, QUINTIC.ctypes.data_as(C.POINTER(C.c_double)), 5)
        arrs = [np.ascontiguousarray(x, dtype=np.float64) for x in (obs, acts, adv, ret, olp, ov, perm)]
        p = [x.ctypes.data_as(C.POINTER(C.c_double)) for x in arrs]
        out0 = np.zeros(1)
        rc = Lb.pl_train_update_resident_deep(h, C.byref(arch), p[0], p[1], p[2], p[3], p[4], p[5], NT, p[6], NT, D, H,
                                              A, 1, 1, lr, 0.0, 0.95, 1e-7, 0.5, 0.01, 0.2, vfclip, maxgn, 1,
                                              out0.ctypes.data_as(C.POINTER(C.c_double)))
        assert rc == 0, Lb.pl_last_error()
        return plb.policy_download(h, P)
    finally:
        plb.policy_free(h)


def test_c5_widths_one_minibatch_gradient_and_step():
    NT = 2048
    lay, P, pm, obs, acts, adv, ret, olp, ov = _problem(NT, 0xC5)
    perm = O.shuffle_perm(NT, 1, 0xC5)
    got = _device_update(pm, P, obs, acts, adv, ret, olp, ov, perm, NT, 0.02, 0.2, 0.0)
    assert np.isfinite(got).all()
    # f64: the minibatch's rows in shuffle order, population-std advantage normalisation, the summed
    # gradient, the mean (no clip), then the Muon step from zero momentum
    idx = perm.astype(np.int64)
    X = obs.reshape(NT, D)[idx]
    a = adv[idx]
    advn = (a - a.mean()) / (a.std() + 1e-8)
    g = cpu_port.ppo_grad(pm[:P], X, acts[idx], advn, ret[idx], olp[idx], D, H, A, L, ACT, ov=ov[idx], vfclip=0.2)
    ref = cpu_port.muon_step(pm.copy(), g, D, H, A, L, 0.02, 0.0, 0.95, 1e-7, QUINTIC, 0.0, 1.0 / NT)
    mom, mom_ref = got[P:], ref[P:]
    worst = []
    for l, (oW, ob, fout, fin) in enumerate(lay):
        e_w, e_b = rel(mom[oW:ob], mom_ref[oW:ob]), rel(mom[ob:ob + fout], mom_ref[ob:ob + fout])
        worst.append((l, e_w, e_b))
    print("C5-width gradient blocks (layer, weight rel, bias rel):", worst)
    # every weight and bias gradient block within the 2e-2 bf16 bar
    assert all(e_w < 2e-2 and e_b < 2e-2 for _, e_w, e_b in worst), worst
    # weight deltas: the orthogonalised momentum of each matrix (see test_gpu_update for why the
    # whole-update bar on deltas is wider than the per-kernel one), and their direction
    for oW, ob, fout, fin in lay:
        dg, dr = got[oW:ob] - pm[oW:ob], ref[oW:ob] - pm[oW:ob]
        assert rel(dg, dr) < 0.15, (fout, fin, rel(dg, dr))
        assert float(dg @ dr / (np.linalg.norm(dg) * np.linalg.norm(dr))) > 0.99


def test_c5_one_chain_launch_for_all_groups_is_bit_identical():
    """The three Newton-Schulz groups of the C5 network (four 2048 x 2048 matrices, the 2048 x 1024
    encoder, the 65 x 2048 head) in one persistent launch give the same bits as one launch per group."""
    NT = 2048
    lay, P, pm, obs, acts, adv, ret, olp, ov = _problem(NT, 0xC6)
    perm = O.shuffle_perm(NT, 1, 0xC6)
    Lb = plb.lib()
    Lb.pl_test_ns_group_launch.argtypes = [C.c_int]
    prev = Lb.pl_test_ns_group_launch(1)
    try:
        one = _device_update(pm, P, obs, acts, adv, ret, olp, ov, perm, NT, 0.02, 0.2, 0.0)
        Lb.pl_test_ns_group_launch(0)
        per = _device_update(pm, P, obs, acts, adv, ret, olp, ov, perm, NT, 0.02, 0.2, 0.0)
    finally:
        Lb.pl_test_ns_group_launch(prev)
    assert np.isfinite(one).all() and not np.array_equal(one[:P], pm[:P])
    assert np.array_equal(one, per)


@pytest.mark.parametrize("batch,rows,cols", [(2, 512, 2048), (1, 2048, 2048), (1, 2048, 1024), (1, 1024, 2048)])
def test_newton_schulz_at_config_shapes_vs_f64(batch, rows, cols):
    torch.manual_seed(rows * 3 + cols)
    X = torch.randn(batch, rows, cols, device="cuda").to(torch.bfloat16)
    Xin = X.double().cpu().numpy()
    rc = plb.lib().pl_ns_batched_bf16_dev(X.data_ptr(), batch, rows, cols, 1e-7,
                                          QUINTIC.ctypes.data_as(C.POINTER(C.c_double)), 5, None)
    assert rc == 0, plb.lib().pl_last_error()
    torch.cuda.synchronize()
    got = X.double().cpu().numpy()
    for b in range(batch):
        ref = cpu_port.newton_schulz(Xin[b], QUINTIC, 1e-7)
        print(f"NS {rows}x{cols}[{b}] rel {rel(got[b], ref):.3e}")
        assert rel(got[b], ref) < 2e-2, (b, rel(got[b], ref))
