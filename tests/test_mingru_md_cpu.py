"""Multi-discrete heads on the MinGRU path, on the CPU: the oracle's restatement of k_mg_ppo_b_md
(ffi/puffercuda.cu:4940-4980; the reference has no CPU form of it) against the pinned categorical
gradient (one head of size A), against central finite differences of the PPO objective through the
whole BPTT (three heads, a terminal mid-sequence), and the W-wide packed layouts of the gather and the
batched gradient."""
import numpy as np

from oracle import oracle as O


def _seq(seed, T, D, H, L, A, K, hs):
    g = np.random.default_rng(seed)
    params, _ = O.init_mingru(D, H, L, A, 0x77 + seed, K)
    params = params + 0.05 * g.standard_normal(params.size)
    obs = g.uniform(-1, 1, T * D)
    W = len(hs) if hs else 1
    acts = (np.stack([g.integers(0, s, T) for s in hs], axis=1).astype(float).ravel() if hs
            else g.integers(0, A, T).astype(float))
    advs, rets = g.standard_normal(T), g.standard_normal(T)
    olps = g.uniform(-4, -1, T)
    terms = np.zeros(T)
    terms[T // 2] = 1.0
    ovs = rets + 0.3 * g.standard_normal(T)
    return params, obs, acts, advs, rets, olps, terms, ovs, W


def test_one_head_is_the_categorical_gradient():
    T, D, H, L, A, K = 6, 5, 8, 2, 5, 3
    params, obs, acts, advs, rets, olps, terms, ovs, _ = _seq(1, T, D, H, L, A, K, None)
    gc, nlc, nvc = O.mingru_grad_seq(params, obs, acts, advs, rets, olps, terms, ovs, T, H, D, L, A, K)
    gm, nlm, nvm = O.mingru_grad_seq(params, obs, acts, advs, rets, olps, terms, ovs, T, H, D, L, A, K, hs=[A])
    np.testing.assert_allclose(gm, gc, rtol=1e-10, atol=1e-13)
    np.testing.assert_allclose(nlm, nlc, rtol=1e-12, atol=1e-13)
    assert np.array_equal(nvm, nvc)


def test_md_gradient_is_the_objective_gradient():
    """Entropy coefficient 0 and no value clip, so the objective is a function of the oracle's own
    outputs: sum_t min(adv r_t, adv clip(r_t)) - vf/2 (v_t - ret_t)^2 with r_t = exp(newlp_t - old_t).
    Old log-probs sit within 0.05 of the new ones (no ratio on a clip edge)."""
    T, D, H, L, A, K, hs = 5, 3, 4, 1, 7, 3, [2, 3, 2]
    params, obs, acts, advs, rets, olps, terms, ovs, _ = _seq(2, T, D, H, L, A, K, hs)
    _, nl, _ = O.mingru_grad_seq(params, obs, acts, advs, rets, olps, terms, ovs, T, H, D, L, A, K, ent=0.0, vfClip=0.0,
                                 hs=hs)
    olps = nl + np.random.default_rng(3).uniform(-0.05, 0.05, T)

    def J(p):
        _, lp, v = O.mingru_grad_seq(p, obs, acts, advs, rets, olps, terms, ovs, T, H, D, L, A, K, ent=0.0, vfClip=0.0,
                                     hs=hs)
        r = np.exp(lp - olps)
        return float(np.sum(np.minimum(advs * r, advs * np.clip(r, 0.8, 1.2)) - 0.25 * (v - rets) ** 2))

    g, _, _ = O.mingru_grad_seq(params, obs, acts, advs, rets, olps, terms, ovs, T, H, D, L, A, K, vf=0.5, ent=0.0,
                                vfClip=0.0, hs=hs)
    h = 1e-6
    fd = np.array([(J(params + h * e) - J(params - h * e)) / (2 * h) for e in np.eye(params.size)])
    np.testing.assert_allclose(g, fd, rtol=1e-5, atol=1e-7)


def test_md_gather_and_batch_layouts():
    """Gather: W actions per row move with their row ([os*W + h]); the batched gradient with the packed
    [(W+5) T B] scalars is the sum of the per-sequence gradients."""
    N, T, Bmb, W = 6, 4, 3, 3
    g = np.random.default_rng(4)
    act = g.integers(0, 4, N * T * W).astype(float)
    logp, term = g.uniform(-3, -1, N * T), (g.random(N * T) < 0.2).astype(float)
    adv, value = g.standard_normal(N * T), g.standard_normal(N * T)
    seg, mbp = np.array([4.0, 1.0, 4.0]), np.array([1.0, 0.8, 1.2])
    out = O.gather_seq_minibatch(act, logp, term, adv, value, seg, mbp, T, Bmb, W=W)
    one = O.gather_seq_minibatch(act.reshape(N * T, W)[:, 0].copy(), logp, term, adv, value, seg, mbp, T, Bmb)
    nb = T * Bmb
    for t in range(T):
        for b in range(Bmb):
            e = int(seg[b])
            assert np.array_equal(out[(t * Bmb + b) * W:(t * Bmb + b + 1) * W], act[(e * T + t) * W:(e * T + t + 1) * W])
    assert np.array_equal(out[W * nb:], one[nb:])
    # batched gradient = sum over sequences
    D, H, L, A, K, hs = 3, 8, 1, 9, 2, [4, 3, 2]
    B = 3
    params, _ = O.init_mingru(D, H, L, A, 9, K)
    obsTB = g.uniform(-1, 1, T * B * D)
    actsTB = np.stack([g.integers(0, s, T * B) for s in hs], axis=1).astype(float)
    sc = np.concatenate([actsTB.ravel(), g.standard_normal(T * B), g.standard_normal(T * B), g.uniform(-3, -1, T * B),
                         (g.random(T * B) < 0.2).astype(float), g.standard_normal(T * B)])
    tot = O.mingru_grad_batch(params, obsTB, sc, B, T, H, D, L, A, K, hs=hs)
    P = params.size
    acc = np.zeros(P)
    for b in range(B):
        rows = [t * B + b for t in range(T)]
        o = np.concatenate([obsTB[r * D:(r + 1) * D] for r in rows])
        a = actsTB[rows].ravel()
        s1 = [sc[(W + q) * T * B:(W + q + 1) * T * B][rows] for q in range(5)]
        gb, nl, nv = O.mingru_grad_seq(params, o, a, *s1, T, H, D, L, A, K, hs=hs)
        acc = acc + gb
        assert np.array_equal(tot[P + np.array(rows)], nl)
    np.testing.assert_allclose(tot[:P], acc, rtol=1e-12, atol=1e-14)
