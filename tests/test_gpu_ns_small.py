"""The fused short-matrix Newton-Schulz (one CTA per matrix with a short side <= 128 and a long side
<= 512, every step chained in TMEM) against the f64 oracle and against the per-step tcgen05 GEMM chain on
the same inputs: square, wide, tall (transposed on the way in and out), ragged sides, long sides of 200
to 512 (the MinGRU encoder's 512 x 120 among them), the configs[2] 128 x 128 batch, and the fp32-output
form inside a CartPole-shaped bf16 update."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


def _small(mode):
    L = plb.lib()
    L.pl_test_ns_small_mode.argtypes = [C.c_int]
    return L.pl_test_ns_small_mode(mode)


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _ns(X, batch, rows, cols, co):
    rc = plb.lib().pl_ns_batched_bf16_dev(X.data_ptr(), batch, rows, cols, 1e-7,
                                          co.ctypes.data_as(C.POINTER(C.c_double)), co.shape[0], None)
    assert rc == 0, plb.lib().pl_last_error()
    torch.cuda.synchronize()


@pytest.mark.parametrize("batch,rows,cols", [(64, 128, 128), (3, 64, 128), (2, 128, 8), (5, 8, 128), (4, 40, 96),
                                             (1, 8, 8), (2, 120, 128), (2, 120, 512), (3, 512, 120), (2, 64, 320),
                                             (1, 128, 512), (2, 96, 200), (2, 8, 384), (4, 128, 256)])
def test_small_ns_fused_vs_oracle_and_chain(batch, rows, cols):
    torch.manual_seed(rows * 7 + cols)
    X0 = torch.randn(batch, rows, cols, device="cuda").to(torch.bfloat16)
    co = np.ascontiguousarray(O.QUINTIC_COEFFS)
    prev = _small(1)
    try:
        Xf = X0.clone()
        _ns(Xf, batch, rows, cols, co)
        _small(0)
        Xc = X0.clone()
        _ns(Xc, batch, rows, cols, co)
    finally:
        _small(prev)
    Xin = X0.double().cpu().numpy()
    f, c = Xf.double().cpu().numpy(), Xc.double().cpu().numpy()
    worst = []
    for b in range(batch):
        ref = O.newton_schulz(Xin[b].ravel(), rows, cols, 1e-7, co).reshape(rows, cols)
        worst.append((rel(f[b], ref), rel(c[b], ref), rel(f[b], c[b])))
    ef, ec, efc = (max(w[i] for w in worst) for i in range(3))
    # both forms round the same operands to bf16 at the same points, so the fused form has the chain's
    # own accuracy: the 2e-2 bar, except an 8 x 8 matrix, whose 64 bf16-rounded entries put both forms
    # near 5e-2 from f64
    bar = 2e-2 if rows * cols >= 1024 else 6e-2
    assert ef < bar and ec < bar, (ef, ec)
    assert efc < 5e-3, efc


def test_small_ns_fp32_output_in_cartpole_update():
    """The bf16-tier update of the CartPole-shaped policy (4 -> 128 -> 2 + 1): its Newton-Schulz matrices
    (128 x 4 and 3 x 128) run fused with fp32 output; the update agrees with the GEMM-chain run to bf16
    rounding and with the f64 oracle to the reference's 0.2 bar."""
    NT, D, H, A, E, MB = 2048, 4, 128, 2, 2, 4
    g = np.random.default_rng(3)
    P = H * D + H + (A + 1) * H + (A + 1)
    pm = np.concatenate([g.uniform(-0.3, 0.3, P), np.zeros(P)])
    obs, acts = g.standard_normal(NT * D), g.integers(0, A, NT).astype(float)
    adv, ret = g.standard_normal(NT), g.standard_normal(NT)
    olp = np.log(np.full(NT, 0.5)) + 0.05 * g.standard_normal(NT)
    perm = O.shuffle_perm(NT, E, 5)

    def run():
        h = plb.policy_load(pm, P)
        try:
            plb.cuda_train_update_resident(h, obs, acts, adv, ret, olp, None, perm, NT, D, H, A, E, MB, 0.02, 0.0, 0.95,
                                           1e-7, 0.5, 0.01, 0.2, 0.0, 0.0, 1)
            return plb.policy_download(h, P)
        finally:
            plb.policy_free(h)

    prev = _small(1)
    try:
        fused = run()
        _small(0)
        chain = run()
    finally:
        _small(prev)
    ref = O.train_update(pm, obs, acts, adv, ret, olp, perm, NT, D, H, A, E, MB, 0.02, 0.0, 0.95, 1e-7, 0.5, 0.01, 0.2)
    assert np.abs(fused - ref).max() < 0.2
    df, dc, dr = fused[:P] - pm[:P], chain[:P] - pm[:P], ref[:P] - pm[:P]
    assert rel(df, dc) < 0.1, rel(df, dc)
    assert float(df @ dr / (np.linalg.norm(df) * np.linalg.norm(dr))) > 0.99
