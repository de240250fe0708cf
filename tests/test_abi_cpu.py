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
