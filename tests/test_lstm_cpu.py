"""LSTM on the CPU: the oracle's restatement against the reference's own C (golden fixtures from
lean_ffi_lstm_ppo_grad_seq and lean_ffi_lstm_gae_boot_norm), the batched form as the ordered sum of the
per-sequence gradients, and the library's host GAE twin."""
import os

import numpy as np

from oracle import oracle as O

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "lstm.npz"))


def test_lstm_seq_grad_matches_reference_c():
    T, H, D, A, B = (int(x) for x in GOLD["meta"])
    f = GOLD
    for b in range(B):
        rows = [t * B + b for t in range(T)]
        o = np.concatenate([f["obsB"][r * D:(r + 1) * D] for r in rows])
        g, _, _ = O.lstm_grad_seq(f["params"], o, f["actB"][rows], f["advB"][rows], f["retB"][rows], f["olpB"][rows],
                                  f["termB"][rows], f["h0s"][b * H:(b + 1) * H], f["c0s"][b * H:(b + 1) * H], T, H, D,
                                  A)
        assert np.array_equal(g, f["seqs"][b]), b


def test_lstm_batch_is_the_ordered_sum():
    T, H, D, A, B = (int(x) for x in GOLD["meta"])
    f = GOLD
    out = O.lstm_grad_batch(f["params"], f["obsB"], f["actB"], f["advB"], f["retB"], f["olpB"], f["termB"], f["h0s"],
                            f["c0s"], B, T, H, D, A)
    acc = np.zeros(f["seqs"].shape[1])
    for b in range(B):
        acc = acc + f["seqs"][b]
    assert np.array_equal(out[:acc.size], acc)


def test_lstm_gae_oracle_and_host_twin_match_reference_c():
    f = GOLD
    N, T = int(f["gae_meta"][0]), int(f["gae_meta"][1])
    gamma, lam = f["gae_meta"][2], f["gae_meta"][3]
    assert np.array_equal(O.lstm_gae_boot_norm(f["vals"], f["rews"], f["terms"], f["boot"], N, T, gamma, lam), f["gae"])
    import pufferlean_b200 as plb
    assert np.array_equal(plb.lstm_gae_boot_norm(f["vals"], f["rews"], f["terms"], f["boot"], N, T, gamma, lam),
                          f["gae"])
