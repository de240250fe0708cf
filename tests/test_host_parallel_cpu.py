"""The library's host shuffle and GAE take a multi-threaded path for large inputs (draws of the
counter-based splitmix64 stream on all threads, one epoch's swap pass per thread; environments split
over threads for GAE): their outputs are bit-identical to the oracle's sequential restatement, which
is pinned to the reference's own outputs (tests/test_oracle.py)."""
import numpy as np

import pufferlean_b200 as plb
from oracle import oracle as O


def test_parallel_shuffle_matches_oracle():
    NT, E = (1 << 18) + 37, 3
    for seed in (1, 0xDEADBEEF12345, 2 ** 64 - 5):
        assert np.array_equal(plb.shuffle_perm(NT, E, seed), O.shuffle_perm(NT, E, seed))


def test_parallel_gae_matches_oracle():
    rng = np.random.default_rng(4)
    N, T = 4099, 64
    vals, rews = rng.standard_normal(N * T), 1.5 * rng.standard_normal(N * T)
    terms = (rng.random(N * T) < 0.05).astype(float)
    got = plb.gae_soa(vals, rews, terms, N, T, 0.995, 0.90)
    want = O.gae_soa(vals, rews, terms, N, T, 0.995, 0.90)
    assert np.array_equal(got, want)
