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


# ---------------------------------------------------------------- Lean adapter (libpufferlean_lean.so)
LEAN_LIB = os.path.join(os.path.dirname(plb.LIB_PATH), "libpufferlean_lean.so")


def test_lean_adapter_exports_every_declared_symbol():
    lib = C.CDLL(LEAN_LIB)
    names = declared("pufferlean_lean.h")
    assert len(names) >= 15
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
