"""CPU checks of the boundary: the C-ABI library loads without a GPU and exports every function
declared in include/*.h; calls fail loudly (no CPU fallback) when no device is present."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import pufferlean_b200 as plb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b((?:pl|lean)_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(plb.LIB_PATH)
    names = declared("pufferlean_b200.h") + declared("pufferlean_b200_testing.h")
    assert len(names) > 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_no_cpu_fallback_without_device():
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is visible")
    except ImportError:
        pass
    with pytest.raises(plb.PufferError, match="no usable CUDA device|no CPU fallback"):
        plb.cuda_vtrace(np.zeros(4), np.zeros(4), np.zeros(4), np.ones(4), 1, 4, 0.99, 0.95, 1.0, 1.0)


def test_host_bookkeeping_matches_oracle():
    from oracle import oracle as O

    for NT, E, seed in [(48, 3, 0x1234), (1000, 2, 99), (0, 1, 5)]:
        assert np.array_equal(plb.shuffle_perm(NT, E, seed), O.shuffle_perm(NT, E, seed))
    g = np.random.default_rng(1)
    vals, rews = g.standard_normal(200), g.uniform(-2, 2, 200)
    terms = (g.random(200) < 0.1).astype(float)
    assert np.array_equal(plb.gae_soa(vals, rews, terms, 10, 20, 0.995, 0.9), O.gae_soa(vals, rews, terms, 10, 20, 0.995, 0.9))


def _gather_golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "gather_minibatch.npz"))


def test_gather_minibatch_and_slice_bit_exact_against_golden():
    """The reference's lean_ffi_gather_minibatch over every minibatch of three shuffled epochs (ragged
    last minibatch) and lean_ffi_slice, against the plain-ABI twins."""
    g = _gather_golden()
    NT, D, E, MB = (int(x) for x in g["meta"])
    mb = NT // MB
    cols = [g[x] for x in ("mbObs", "mbAct", "mbAdv", "mbRet", "mbOlp")]
    pos = [0] * 5
    for e in range(E):
        for m in range(MB):
            lo, hi = m * mb, (NT if m + 1 == MB else (m + 1) * mb)
            n = hi - lo
            got = plb.gather_minibatch(g["obs"], g["acts"], g["advs"], g["rets"], g["olps"],
                                       g["perm"][e * NT + lo:e * NT + hi], n, D)
            for i, (x, w) in enumerate(zip(got, (D, 1, 1, 1, 1))):
                assert np.array_equal(x, cols[i][pos[i]:pos[i] + n * w]), (e, m, i)
                pos[i] += n * w
    for i, (off, ln) in enumerate(g["slices"]):
        assert np.array_equal(plb.slice(g["obs"], int(off), int(ln)), g[f"slice{i}"])


def test_gather_minibatch_edge_cases():
    g = np.random.default_rng(3)
    obs, a, ad, r, ol = g.standard_normal(40), g.standard_normal(10), g.standard_normal(10), g.standard_normal(10), \
        g.standard_normal(10)
    # empty minibatch, fractional indices truncated like the reference's cast, D = 0
    assert all(x.size == 0 for x in plb.gather_minibatch(obs, a, ad, r, ol, np.zeros(0), 0, 4))
    got = plb.gather_minibatch(obs, a, ad, r, ol, np.array([2.9, 0.0]), 2, 4)
    assert np.array_equal(got[0], np.concatenate([obs[8:12], obs[0:4]])) and np.array_equal(got[1], a[[2, 0]])
    assert np.array_equal(plb.gather_minibatch(obs, a, ad, r, ol, np.array([9.0]), 1, 0)[2], ad[[9]])
    # an index that is not a row fails before anything is written
    for bad in (10.0, -1.0, np.nan):
        with pytest.raises(plb.PufferError, match="not a row"):
            plb.gather_minibatch(obs, a, ad, r, ol, np.array([1.0, bad]), 2, 4)
    with pytest.raises(plb.PufferError, match="outside"):
        plb.slice(obs, 38, 3)
    assert plb.slice(obs, 40, 0).size == 0


def test_mingru_host_twins_bit_exact_against_golden():
    """pl_prio_sample and pl_gather_seq_minibatch reproduce the reference's host C bit for bit."""
    gp = np.load(os.path.join(ROOT, "tests", "golden", "prio.npz"))
    m = gp["meta"]
    seg, mp = plb.prio_sample(gp["L1"], int(m[0]), int(m[1]), int(m[2]), m[3], m[4], int(m[5]))
    assert np.array_equal(seg, gp["idx"]) and np.array_equal(mp, gp["mbPrio"])
    gs = np.load(os.path.join(ROOT, "tests", "golden", "gather_seq.npz"))
    N, T, D, Bmb = (int(x) for x in gs["meta"])
    out = plb.gather_seq_minibatch(gs["act"], gs["logp"], gs["term"], gs["adv"], gs["value"], gs["seg"], gs["mbPrio"], T,
                                   Bmb)
    assert np.array_equal(out, gs["out"])


def test_mingru_host_twins_edge_cases():
    from oracle import oracle as O

    g = np.random.default_rng(3)
    # a single segment; zero priorities everywhere (the 1e-6 floor); large N with many draws
    for N, B in ((1, 5), (7, 7), (4000, 900)):
        l1 = np.zeros(N) if N == 7 else g.uniform(0, 50, N)
        seg, mp = plb.prio_sample(l1, N, 64, B, 0.6, 0.4, 0xDEADBEEF + N)
        so, mo = O.prio_sample(l1, N, B, 0.6, 0.4, 0xDEADBEEF + N)
        assert np.array_equal(seg, so) and np.array_equal(mp, mo)
        assert seg.min() >= 0 and seg.max() <= N - 1
    # a segment drawn several times, T = 1
    adv = g.standard_normal(12)
    out = plb.gather_seq_minibatch(np.arange(12.0) % 3, g.standard_normal(12), (g.random(12) < 0.3) * 1.0, adv,
                                   g.standard_normal(12), np.array([3.0, 3.0, 0.0]), np.array([1.0, 0.5, 2.0]), 1, 3)
    assert out.size == 18 and np.isfinite(out).all()


def test_mingru_param_count_and_no_device():
    assert plb.mg_param_count(118, 512, 1, 4) == 849925  # the Breakout net, 3H layers
    assert plb.mg_param_count(118, 512, 1, 4, K=2) == 849925 - 512 * 512
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is visible")
    except ImportError:
        pass
    with pytest.raises(plb.PufferError, match="no usable CUDA device|no CPU fallback"):
        plb.MgSession(4, 8)
    with pytest.raises(plb.PufferError, match="no usable CUDA device|no CPU fallback"):
        plb.cuda_mingru_ppo_grad(np.zeros(plb.mg_param_count(2, 8, 1, 2)), np.zeros(8), np.zeros(24), 2, 2, 8, 2, 1, 2,
                                 0.5, 0.01, 0.2, 0.2)


def test_checkpoint_bytes_match_the_reference_layout(tmp_path):
    """ckptToBytes (Puffer/RL/FFITrain.lean:55-62): u64 P then P f64 bit patterns, little-endian; the
    parser is bounded by the file size (bytesToCkpt, :66-69)."""
    import struct

    g = np.random.default_rng(4)
    w = np.concatenate([g.standard_normal(37), [0.0, -0.0, np.inf, 1e-310]])
    path = tmp_path / "123.bin"
    plb.ckpt_write(str(path), w)
    raw = path.read_bytes()
    assert raw == struct.pack("<Q", w.size) + w.astype("<f8").tobytes()
    back = plb.ckpt_read(str(path))
    assert back.tobytes() == w.tobytes()
    # a truncated file yields the doubles it holds; a header claiming fewer yields that many
    path.write_bytes(raw[:8 + 8 * 5 + 3])
    assert np.array_equal(plb.ckpt_read(str(path)), w[:5])
    path.write_bytes(struct.pack("<Q", 2) + w.astype("<f8").tobytes())
    assert np.array_equal(plb.ckpt_read(str(path)), w[:2])
    path.write_bytes(b"\x01\x02")
    assert plb.ckpt_read(str(path)).size == 0
    with pytest.raises(plb.PufferError):
        plb.ckpt_read(str(tmp_path / "missing.bin"))


# ---------------------------------------------------------------- Lean adapter (libpufferlean_lean.so)
LEAN_LIB = os.path.join(os.path.dirname(plb.LIB_PATH), "libpufferlean_lean.so")


def test_lean_adapter_exports_every_declared_symbol():
    lib = C.CDLL(LEAN_LIB)
    names = declared("pufferlean_lean.h")
    assert len(names) >= 23
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_lean_adapter_host_bookkeeping_against_golden():
    from oracle import oracle as O

    lib = C.CDLL(LEAN_LIB)
    g = np.load(os.path.join(ROOT, "tests", "golden", "shuffle.npz"))
    for i in range(3):
        NT, E, seed = (int(x) for x in g[f"args{i}"])
        out = O.ref_call(lib, "lean_ffi_shuffle_perm", C.c_void_p, NT, E, ("u64", seed))
        assert np.array_equal(O.read_float_array(out), g[f"perm{i}"])
    g = np.load(os.path.join(ROOT, "tests", "golden", "gae.npz"))
    N, T, gm, lm = g["meta"]
    out = O.ref_call(lib, "lean_ffi_gae_soa", C.c_void_p, O.FA(g["vals"]), O.FA(g["rews"]), O.FA(g["terms"]), int(N),
                     int(T), float(gm), float(lm))
    assert np.array_equal(O.read_float_array(out), g["out"])


def test_lean_adapter_gather_minibatch_and_slice_against_golden():
    from oracle import oracle as O

    lib = C.CDLL(LEAN_LIB)
    g = _gather_golden()
    NT, D, E, MB = (int(x) for x in g["meta"])
    n = NT - (MB - 1) * (NT // MB)  # the ragged last minibatch of the last epoch
    lo = (E - 1) * NT + (MB - 1) * (NT // MB)
    t = O.ref_call(lib, "lean_ffi_gather_minibatch", C.c_void_p, O.FA(g["obs"]), O.FA(g["acts"]), O.FA(g["advs"]),
                   O.FA(g["rets"]), O.FA(g["olps"]), O.FA(g["perm"][lo:lo + n]), n, D)
    got = []
    for _ in range(4):
        got.append(O.read_float_array(O.ctor_field(t, 0)))
        t = O.ctor_field(t, 1)
    got.append(O.read_float_array(t))
    k0 = (E - 1) * NT + (MB - 1) * (NT // MB)
    assert np.array_equal(got[0], g["mbObs"][k0 * D:(k0 + n) * D])
    for x, name in zip(got[1:], ("mbAct", "mbAdv", "mbRet", "mbOlp")):
        assert np.array_equal(x, g[name][k0:k0 + n])
    for i, (off, ln) in enumerate(g["slices"]):
        out = O.ref_call(lib, "lean_ffi_slice", C.c_void_p, O.FA(g["obs"]), int(off), int(ln))
        assert np.array_equal(O.read_float_array(out), g[f"slice{i}"])
    # out of range: NaNs, never zeros
    out = O.ref_call(lib, "lean_ffi_slice", C.c_void_p, O.FA(np.ones(4)), 3, 2)
    assert np.all(np.isnan(O.read_float_array(out)))
    t = O.ref_call(lib, "lean_ffi_gather_minibatch", C.c_void_p, O.FA(np.ones(8)), O.FA(np.ones(2)),
                   O.FA(np.ones(2)), O.FA(np.ones(2)), O.FA(np.ones(2)), O.FA(np.array([5.0])), 1, 4)
    assert np.all(np.isnan(O.read_float_array(O.ctor_field(t, 0))))


def test_lean_adapter_mingru_host_bookkeeping_against_golden():
    from oracle import oracle as O

    lib = C.CDLL(LEAN_LIB)
    gp = np.load(os.path.join(ROOT, "tests", "golden", "prio.npz"))
    m = gp["meta"]
    pr = O.ref_call(lib, "lean_ffi_prio_sample", C.c_void_p, O.FA(gp["L1"]), int(m[0]), int(m[1]), int(m[2]),
                    float(m[3]), float(m[4]), ("u64", int(m[5])))
    assert np.array_equal(O.read_float_array(O.ctor_field(pr, 0)), gp["idx"])
    assert np.array_equal(O.read_float_array(O.ctor_field(pr, 1)), gp["mbPrio"])
    gs = np.load(os.path.join(ROOT, "tests", "golden", "gather_seq.npz"))
    N, T, D, Bmb = (int(x) for x in gs["meta"])
    out = O.ref_call(lib, "lean_ffi_gather_seq_minibatch", C.c_void_p, O.FA(np.zeros(N * T * D)), O.FA(gs["act"]),
                     O.FA(gs["logp"]), O.FA(gs["term"]), O.FA(gs["adv"]), O.FA(gs["value"]), O.FA(gs["seg"]),
                     O.FA(gs["mbPrio"]), T, Bmb, D, N)
    assert np.array_equal(O.read_float_array(out), gs["out"])


def test_lean_adapter_mingru_io_errors_without_state():
    """Without columns, or asking for multi-discrete heads, the MinGRU IO symbols return IO errors."""
    from oracle import oracle as O

    lib = C.CDLL(LEAN_LIB)
    r = O.ref_call(lib, "lean_cuda_mg_vtrace", C.c_void_p, 3, 4, 0.99, 0.95, 1.0, 1.0, ("obj", 1))
    assert O.ctor_tag(r) == 1
    r = O.ref_call(lib, "lean_cuda_mg_prep", C.c_void_p, *[O.FA(np.zeros(8)) for _ in range(6)], 2, 4, 2, ("obj", 1))
    assert O.ctor_tag(r) == 1
    r = O.ref_call(lib, "lean_cuda_mg_cols_ready", C.c_void_p, 2, 4, ("obj", 1))
    assert O.ctor_tag(r) == 0


def test_lean_adapter_pure_failure_is_nan_not_zero():
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is visible")
    except ImportError:
        pass
    from oracle import oracle as O

    lib = C.CDLL(LEAN_LIB)
    out = O.ref_call(lib, "lean_cuda_vtrace", C.c_void_p, O.FA(np.zeros(6)), O.FA(np.zeros(6)), O.FA(np.zeros(6)),
                     O.FA(np.ones(6)), 2, 3, 0.99, 0.95, 1.0, 1.0)
    assert np.all(np.isnan(O.read_float_array(out)))
    # IO functions report an IO error (constructor 1) instead
    r = O.ref_call(lib, "lean_cuda_policy_load", C.c_void_p, O.FA(np.zeros(4)), 2, ("obj", 1))
    assert O.ctor_tag(r) == 1
