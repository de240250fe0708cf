"""The batched LSTM + PPO BPTT gradient on the GPU (pl_lstm_ppo_grad_batch) against the f64 oracle (pinned to
the reference's lean_ffi_lstm_ppo_grad_seq) and the reference's own outputs (golden): the f64 tier to 1e-11
relative, the f32 tier to the MinGRU tight-tier bar, the bf16 tier (products of bf16-rounded operands) to
2e-2 relative Frobenius; Wh in shared memory (H = 32) and read through L2
(H = 128); ragged B; detached non-zero initial states and terminals mid-sequence; new log-probs and values;
the input-reuse switch of the trainer's later epochs; determinism; the Lean symbols."""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import oracle as O  # noqa: E402
from oracle.oracle import FA  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "lstm.npz")


@pytest.fixture(scope="module", autouse=True)
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def frob(a, ref):
    return float(np.linalg.norm(a - ref) / max(np.linalg.norm(ref), 1e-30))


def rel_floor(a, ref, floor=1e-3):
    return float(np.max(np.abs(a - ref) / (np.abs(ref) + floor)))


def _inputs(B, T, H, D, A, seed):
    g = np.random.default_rng(seed)
    P = plb.lstm_param_count(D, H, A)
    params = g.uniform(-1, 1, P) / np.sqrt(max(D, H))
    R = T * B
    return dict(params=params, obs=g.standard_normal(R * D), acts=g.integers(0, A, R).astype(float),
                advs=g.standard_normal(R), rets=g.standard_normal(R), olps=g.uniform(-3, -0.3, R),
                terms=(g.random(R) < 0.1).astype(float), h0s=g.uniform(-0.5, 0.5, B * H),
                c0s=g.uniform(-0.5, 0.5, B * H))


def _args(k):
    return [k[x] for x in ("params", "obs", "acts", "advs", "rets", "olps", "terms", "h0s", "c0s")]


@pytest.mark.parametrize("B,T,H,D,A", [(13, 16, 32, 7, 5), (6, 8, 128, 9, 3), (40, 12, 64, 4, 2)])
def test_lstm_tiers_vs_oracle(B, T, H, D, A):
    k = _inputs(B, T, H, D, A, B + T + H)
    ref = O.lstm_grad_batch(*_args(k), B, T, H, D, A)
    P = plb.lstm_param_count(D, H, A)
    g64, nl, nv = plb.cuda_lstm_ppo_grad_batch(*_args(k), B, T, H, D, A, 0.5, 0.01, 0.2, tier=0, with_outputs=True)
    assert frob(g64, ref[:P]) < 1e-11, frob(g64, ref[:P])
    np.testing.assert_allclose(nl, ref[P:P + T * B], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(nv, ref[P + T * B:], rtol=1e-12, atol=1e-12)
    g32 = plb.cuda_lstm_ppo_grad_batch(*_args(k), B, T, H, D, A, 0.5, 0.01, 0.2, tier=1)
    assert frob(g32, ref[:P]) < 1e-4, frob(g32, ref[:P])
    assert rel_floor(g32, ref[:P]) < 2e-3, rel_floor(g32, ref[:P])
    # bf16 tier: every product's operands rounded to bf16, f32 accumulation and f32 gate arithmetic
    g16 = plb.cuda_lstm_ppo_grad_batch(*_args(k), B, T, H, D, A, 0.5, 0.01, 0.2, tier=2)
    assert frob(g16, ref[:P]) < 2e-2, frob(g16, ref[:P])
    assert not np.array_equal(g16, g32)
    assert np.array_equal(plb.cuda_lstm_ppo_grad_batch(*_args(k), B, T, H, D, A, 0.5, 0.01, 0.2, tier=2), g16)
    again = plb.cuda_lstm_ppo_grad_batch(*_args(k), B, T, H, D, A, 0.5, 0.01, 0.2, tier=1)
    assert np.array_equal(again, g32)


def test_lstm_against_reference_golden():
    f = np.load(GOLD)
    T, H, D, A, B = (int(x) for x in f["meta"])
    args = [f[x] for x in ("params", "obsB", "actB", "advB", "retB", "olpB", "termB", "h0s", "c0s")]
    g = plb.cuda_lstm_ppo_grad_batch(*args, B, T, H, D, A, 0.5, 0.01, 0.2, tier=0)
    ref = np.zeros_like(g)
    for b in range(B):
        ref = ref + f["seqs"][b]
    assert frob(g, ref) < 1e-11, frob(g, ref)


def test_lstm_reuse_inputs():
    B, T, H, D, A = 9, 10, 32, 6, 4
    k = _inputs(B, T, H, D, A, 3)
    p2 = k["params"] * 0.9 + 0.01
    L = plb.lib()
    plb.cuda_lstm_ppo_grad_batch(*_args(k), B, T, H, D, A, 0.5, 0.01, 0.2, tier=1)
    L.pl_lstm_reuse_inputs(1)
    try:
        junk = dict(k, obs=np.zeros_like(k["obs"]), advs=np.zeros_like(k["advs"]), params=p2)
        reused = plb.cuda_lstm_ppo_grad_batch(*_args(junk), B, T, H, D, A, 0.5, 0.01, 0.2, tier=1)
    finally:
        L.pl_lstm_reuse_inputs(0)
    fresh = plb.cuda_lstm_ppo_grad_batch(*_args(dict(k, params=p2)), B, T, H, D, A, 0.5, 0.01, 0.2, tier=1)
    assert np.array_equal(reused, fresh)


def test_lstm_lean_symbols():
    plb.lib()
    L = C.CDLL(os.path.join(os.path.dirname(plb.LIB_PATH), "libpufferlean_lean.so"))
    VP = C.c_void_p
    B, T, H, D, A = 7, 9, 16, 5, 3
    k = _inputs(B, T, H, D, A, 11)
    ref = O.lstm_grad_batch(*_args(k), B, T, H, D, A)
    P = plb.lstm_param_count(D, H, A)
    for name, bar in (("lean_ffi_lstm_ppo_grad_batch_blas", 1e-11), ("lean_ffi_lstm_ppo_grad_batch_blas_f32", 1e-4)):
        out = O.read_float_array(O.ref_call(L, name, VP, *[FA(x) for x in _args(k)], B, T, H, D, A, 0.5, 0.01, 0.2))
        assert out.size == P and frob(out, ref[:P]) < bar, (name, frob(out, ref[:P]))
    f = np.load(GOLD)
    N, Tg = int(f["gae_meta"][0]), int(f["gae_meta"][1])
    gae = O.read_float_array(O.ref_call(L, "lean_ffi_lstm_gae_boot_norm", VP, FA(f["vals"]), FA(f["rews"]),
                                        FA(f["terms"]), FA(f["boot"]), N, Tg, float(f["gae_meta"][2]),
                                        float(f["gae_meta"][3])))
    assert np.array_equal(gae, f["gae"])


@pytest.mark.parametrize("B,T,H,D,A", [(13, 16, 32, 7, 5), (300, 10, 64, 4, 2), (5, 7, 8, 3, 2)])
def test_lstm_four_threads_per_unit_vs_one(B, T, H, D, A):
    """The recurrences with four threads per unit (each gate's dot product one thread's, the reverse sum
    over gate blocks added by a butterfly) against one thread per unit: the forward is the same order of
    operations, the reverse only re-associates the dh sum, so the tiers agree to their own rounding."""
    k = _inputs(B, T, H, D, A, 7 * B + H)
    L = plb.lib()
    L.pl_test_lstm_quad.argtypes = [C.c_int]
    prev = L.pl_test_lstm_quad(1)
    try:
        quad = [plb.cuda_lstm_ppo_grad_batch(*_args(k), B, T, H, D, A, 0.5, 0.01, 0.2, tier=t) for t in (0, 1, 2)]
        L.pl_test_lstm_quad(0)
        one = [plb.cuda_lstm_ppo_grad_batch(*_args(k), B, T, H, D, A, 0.5, 0.01, 0.2, tier=t) for t in (0, 1, 2)]
    finally:
        L.pl_test_lstm_quad(prev)
    assert frob(quad[0], one[0]) < 1e-13, frob(quad[0], one[0])
    assert frob(quad[1], one[1]) < 1e-5, frob(quad[1], one[1])
    assert frob(quad[2], one[2]) < 1e-4, frob(quad[2], one[2])
