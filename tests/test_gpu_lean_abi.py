"""The reference's Lean symbols through libpufferlean_lean.so on the GPU, with Lean FloatArray
objects built the way the Lean runtime lays them out (include/lean_compat)."""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import pufferlean_b200 as plb  # noqa: E402
from oracle import oracle as O  # noqa: E402
from oracle.oracle import FA  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
VP = C.c_void_p


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    plb.lib()
    return C.CDLL(os.path.join(os.path.dirname(plb.LIB_PATH), "libpufferlean_lean.so"))


def test_lean_cuda_vtrace_kat(lib):
    f = np.load(os.path.join(GOLD, "vtrace.npz"))
    B, T, g, l, rho, c = f["meta"]
    out = O.ref_call(lib, "lean_cuda_vtrace", VP, FA(f["rew"]), FA(f["val"]), FA(f["term"]), FA(f["imp"]), int(B),
                     int(T), g, l, rho, c)
    assert np.array_equal(O.read_float_array(out), f["adv"])


def test_lean_cuda_train_update_kat(lib):
    f = np.load(os.path.join(GOLD, "train_update.npz"))
    NT, D, H, A, E, MB, vf, ent, clip, lr, wd, mu, eps, seed = f["meta"]
    NT, D, H, A, E, MB = (int(x) for x in (NT, D, H, A, E, MB))
    perm = O.read_float_array(O.ref_call(lib, "lean_ffi_shuffle_perm", VP, NT, E, ("u64", int(seed))))
    out = O.ref_call(lib, "lean_cuda_train_update", VP, FA(f["pm0"]), FA(f["obs"]), FA(f["acts"]), FA(f["adv"]),
                     FA(f["rets"]), FA(f["olps"]), FA(perm), NT, D, H, A, E, MB, lr, wd, mu, eps, vf, ent, clip,
                     ("u8", 0))
    assert np.abs(O.read_float_array(out) - f["out"]).max() < 1e-3


def test_lean_resident_policy_round_trip(lib):
    f = np.load(os.path.join(GOLD, "train_update.npz"))
    NT, D, H, A, E, MB, vf, ent, clip, lr, wd, mu, eps, seed = f["meta"]
    NT, D, H, A, E, MB = (int(x) for x in (NT, D, H, A, E, MB))
    P = f["pm0"].size // 2
    r = O.ref_call(lib, "lean_cuda_policy_load", VP, FA(f["pm0"]), P, ("obj", 1))
    assert O.ctor_tag(r) == 0
    hobj = O.ctor_field(r, 0)
    # USize boxed as a scalar constructor: the handle is its 8-byte payload
    handle = int.from_bytes(C.string_at(hobj + 8, 8), "little")
    perm = O.read_float_array(O.ref_call(lib, "lean_ffi_shuffle_perm", VP, NT, E, ("u64", int(seed))))
    r = O.ref_call(lib, "lean_cuda_train_update_resident", VP, handle, FA(f["obs"]), FA(f["acts"]), FA(f["adv"]),
                   FA(f["rets"]), FA(f["olps"]), FA(np.zeros(0)), FA(perm), NT, D, H, A, E, MB, lr, wd, mu, eps, vf,
                   ent, clip, 0.0, 0.0, ("u8", 0), ("obj", 1))
    assert O.ctor_tag(r) == 0
    p0 = O.read_float_array(O.ctor_field(r, 0))
    r = O.ref_call(lib, "lean_cuda_policy_download", VP, handle, P, ("obj", 1))
    pm = O.read_float_array(O.ctor_field(r, 0))
    assert p0[0] == pm[0]
    assert np.abs(pm - f["out"]).max() < 1e-3
    r = O.ref_call(lib, "lean_cuda_policy_free", VP, handle, ("obj", 1))
    assert O.ctor_tag(r) == 0


def _lean_handle(lib, pm, P):
    r = O.ref_call(lib, "lean_cuda_policy_load", VP, FA(pm), P, ("obj", 1))
    assert O.ctor_tag(r) == 0
    return int.from_bytes(C.string_at(O.ctor_field(r, 0) + 8, 8), "little")


def test_lean_wide_resident_gauss_golden(lib):
    """lean_cuda_train_update_wide_resident (mode 2) on the Gaussian golden update composed from the
    reference's C, then lean_cuda_muon_step_mlp_resident on the reference's muonStepMlpBlasFFI golden."""
    f = np.load(os.path.join(GOLD, "gauss_update.npz"))
    NT, D, H, W, E, MB = (int(x) for x in f["meta"])
    lr, wd, mu, eps, vf, ent, clip, vfc = f["hyp"]
    Oo = 2 * W + 1
    P = H * D + H + Oo * H + Oo
    handle = _lean_handle(lib, f["pm0"], P)
    r = O.ref_call(lib, "lean_cuda_train_update_wide_resident", VP, handle, FA(f["obs"]), FA(f["acts"]), FA(f["adv"]),
                   FA(f["ret"]), FA(f["olp"]), FA(f["ov"]), FA(f["perm"]), FA(np.zeros(0)), NT, D, H, Oo, W, ("u32", 2),
                   E, MB, lr, wd, mu, eps, vf, ent, clip, vfc, 0.0, ("u8", 0), ("obj", 1))
    assert O.ctor_tag(r) == 0
    p0 = O.read_float_array(O.ctor_field(r, 0))
    pm = O.read_float_array(O.ctor_field(O.ref_call(lib, "lean_cuda_policy_download", VP, handle, P, ("obj", 1)), 0))
    assert p0[0] == pm[0]
    assert np.abs(pm - f["out"]).max() < 1e-3
    O.ref_call(lib, "lean_cuda_policy_free", VP, handle, ("obj", 1))

    m = np.load(os.path.join(GOLD, "muon_cpu.npz"))
    H, D, Oo, gscale, lr, wd, mu, eps = m["meta"]
    H, D, Oo = int(H), int(D), int(Oo)
    P = m["params"].size
    handle = _lean_handle(lib, np.concatenate([m["params"], m["mom"]]), P)
    r = O.ref_call(lib, "lean_cuda_muon_step_mlp_resident", VP, handle, FA(m["grad"]), H, D, Oo, gscale, lr, wd, mu, eps,
                   ("obj", 1))
    assert O.ctor_tag(r) == 0
    assert np.array_equal(O.read_float_array(O.ctor_field(r, 0)), m["out"][:P])
    pm = O.read_float_array(O.ctor_field(O.ref_call(lib, "lean_cuda_policy_download", VP, handle, P, ("obj", 1)), 0))
    assert np.array_equal(pm, m["out"])
    O.ref_call(lib, "lean_cuda_policy_free", VP, handle, ("obj", 1))


def _mg_lean_inputs():
    from oracle import kat

    return kat.kat_mingru_update()


def test_lean_mingru_host_grad_against_reference_c(lib, monkeypatch):
    """lean_cuda_mingru_ppo_grad in host mode (obs and scal given) on the verify-mingru-grad-gpu inputs."""
    from oracle import kat

    monkeypatch.setenv("PUFFER_MG_BF16", "0")
    k = kat.kat_mingru_grad()
    g = np.load(os.path.join(GOLD, "mingru_grad.npz"))
    P = O.mg_param_count(k["D"], k["H"], k["L"], k["A"])
    r = O.ref_call(lib, "lean_cuda_mingru_ppo_grad", VP, FA(k["params"]), FA(k["obsTB"]), FA(k["scal"]), k["B"],
                   k["T"], k["H"], k["D"], k["L"], k["A"], 1, FA(np.zeros(0)), k["vf"], k["ent"], k["clip"],
                   k["vfClip"], FA(np.zeros(0)), FA(np.zeros(0)), ("obj", 1))
    assert O.ctor_tag(r) == 0
    out = O.read_float_array(O.ctor_field(r, 0))
    ref = 0.0 + g["seq0"][:P] + g["seq1"][:P]
    assert out.size == P + 2 * k["T"] * k["B"]
    assert np.max(np.abs(out[:P] - ref) / (np.abs(ref) + 1e-4)) < 2e-3


def test_lean_mingru_trainer_sequence_against_reference(lib, monkeypatch):
    """The reference trainer's per-minibatch calls (Puffer/RL/MinGRUTrain.lean:800-850) through the Lean
    symbols: mg_prep, then per minibatch mg_vtrace_prio, mingru_ppo_grad in device-column mode (params
    on the first call, empty after), mingru_muon_resident with an empty gClip; fp32 tier against the
    update composed from the reference's own C."""
    monkeypatch.setenv("PUFFER_MG_BF16", "0")
    k = _mg_lean_inputs()
    N, T, D, H, L, A = (k[x] for x in ("N", "T", "D", "H", "L", "A"))
    P = O.mg_param_count(D, H, L, A)
    hh = plb.policy_load(k["pm0"], P)
    try:
        r = O.ref_call(lib, "lean_cuda_mg_prep", VP, FA(k["rew"]), FA(k["term"]), FA(k["act"]), FA(k["logp"]),
                       FA(k["val0"]), FA(k["boot"]), N, T, 1, ("obj", 1))
        assert O.ctor_tag(r) == 0
        sess = lib.pl_lean_mg_session
        sess.restype = C.c_void_p
        s = sess()
        assert s
        obs = np.ascontiguousarray(k["obs"], dtype=np.float64)
        plb.lib().pl_mg_set_obs.argtypes = [C.c_void_p, C.POINTER(C.c_double), C.c_size_t]
        assert plb.lib().pl_mg_set_obs(s, obs.ctypes.data_as(C.POINTER(C.c_double)), D) == 0
        rng = k["rng"]
        Bmb = k["mbSegs"]
        for mb in range(k["numMB"]):
            r = O.ref_call(lib, "lean_cuda_mg_vtrace_prio", VP, N, T, k["gamma"], k["lam"], k["rho"], k["c"], Bmb,
                           k["alpha"], k["beta"], ("u64", rng), ("obj", 1))
            assert O.ctor_tag(r) == 0
            rng = (rng + Bmb * 0x9E3779B97F4A7C15) & ((1 << 64) - 1)
            pa = k["pm0"][:P] if mb == 0 else np.zeros(0)
            r = O.ref_call(lib, "lean_cuda_mingru_ppo_grad", VP, FA(pa), FA(np.zeros(0)), FA(np.zeros(0)), Bmb, T, H, D,
                           L, A, 1, FA(np.zeros(0)), k["vf"], k["ent"], k["clip"], k["vfClip"], FA(np.zeros(0)),
                           FA(np.zeros(0)), ("obj", 1))
            assert O.ctor_tag(r) == 0, "grad"
            assert O.read_float_array(O.ctor_field(r, 0)).size == 0
            r = O.ref_call(lib, "lean_cuda_mingru_muon_resident", VP, hh, FA(np.zeros(0)), H, D, L, A, k["lr"],
                           k["wd"], k["mu"], k["eps"], k["maxGradNorm"], 1.0 / (Bmb * T), ("obj", 1))
            assert O.ctor_tag(r) == 0, "muon"
        out = plb.policy_download(hh, P)
    finally:
        plb.policy_free(hh)
    ref = np.load(os.path.join(GOLD, "mingru_update.npz"))["out"]
    d_ref, d_out = ref[:P] - k["pm0"][:P], out[:P] - k["pm0"][:P]
    assert np.linalg.norm(d_out - d_ref) / np.linalg.norm(d_ref) < 1e-3


@pytest.mark.parametrize("bf16", [0, 1])
def test_lean_wide_gradients_md_and_cont(lib, bf16):
    """lean_cuda_mlp_ppo_grad_md / _cont (the verify modes' wide-head gradients) against the plain ABI
    (same kernels: bit-identical) and, in the tight tier, the oracle."""
    g = np.random.default_rng(31 + bf16)
    N, D, H = 700, 12, 64
    for mode in (1, 2):
        hs = np.array([3.0, 5.0, 2.0]) if mode == 1 else None
        W = 3 if mode == 1 else 4
        O_ = int(hs.sum()) + 1 if mode == 1 else 2 * W + 1
        P = H * D + H + O_ * H + O_
        params = g.uniform(-0.2, 0.2, P)
        obs = g.standard_normal(N * D)
        if mode == 1:
            acts = np.stack([g.integers(0, int(h), N) for h in hs], 1).astype(float).ravel()
        else:
            acts = g.standard_normal(N * W)
        adv, ret = g.standard_normal(N), g.standard_normal(N)
        olp = g.normal(-2.0, 0.3, N)
        if mode == 1:
            out = O.ref_call(lib, "lean_cuda_mlp_ppo_grad_md", VP, FA(params), FA(obs), FA(acts), FA(adv), FA(ret),
                             FA(olp), FA(hs), N, H, D, W, 0.5, 0.01, 0.2, ("u8", bf16))
        else:
            out = O.ref_call(lib, "lean_cuda_mlp_ppo_grad_cont", VP, FA(params), FA(obs), FA(acts), FA(adv), FA(ret),
                             FA(olp), N, H, D, W, 0.5, 0.01, 0.2, ("u8", bf16))
        got = O.read_float_array(out)
        want = plb.cuda_mlp_ppo_grad_wide(params, obs, acts, adv, ret, olp, None, N, H, D, O_, W, mode, hs, 0.5, 0.01,
                                          0.2, 0.0, bf16)
        assert got.size == P and np.array_equal(got, want)
        if not bf16:
            ref, _, _ = O.mlp_ppo_grad_wide(params, obs, acts, adv, ret, olp, N, D, H, O_, W, mode, hs=hs)
            assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5


def test_lean_mg_chain_ready_follows_the_rollout_stamp(lib):
    N, T, D, LH = 4, 8, 6, 32
    r = O.ref_call(lib, "lean_cuda_mg_prep", VP, *[FA(np.zeros(N * T)) for _ in range(5)], FA(np.zeros(N)), N, T, 1,
                   ("obj", 1))
    assert O.ctor_tag(r) == 0
    ready = lambda n, d, lh: O.ctor_field(O.ref_call(lib, "lean_cuda_mg_chain_ready", VP, n, d, lh, ("obj", 1)), 0)
    box = lambda b: (b << 1) | 1  # lean_box
    assert ready(N, D, LH) == box(0)
    L = plb.lib()
    lib.pl_lean_mg_session.restype = VP
    L.pl_mg_chain_stamp.argtypes = [VP, C.c_size_t, C.c_size_t, C.c_size_t]
    sess = lib.pl_lean_mg_session()
    assert L.pl_mg_chain_stamp(sess, N, D, LH) == 0
    assert ready(N, D, LH) == box(1)
    assert ready(N, D + 1, LH) == box(0)
    assert L.pl_mg_chain_stamp(sess, 0, 0, 0) == 0
    assert ready(N, D, LH) == box(0)
