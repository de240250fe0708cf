"""Seeded known-answer inputs of the reference's verify-* modes. TEST INFRASTRUCTURE.

The reference stores no golden vectors for the update path: each of its verify-* modes regenerates
its inputs from a seed with the splitmix64 `randF` (Exe/Puffer.lean:65-67, Puffer/RL/Train.lean:18-28).
These functions restate those input loops draw for draw, so the same inputs can be fed both to the
reference's compiled C (to produce golden outputs) and to this project's kernels.
"""
from __future__ import annotations

import math

import numpy as np

GOLD = 0x9E3779B97F4A7C15
M64 = (1 << 64) - 1


class Rng:
    """splitmix64 `rngNext` state (Puffer/RL/Train.lean:18-24)."""

    def __init__(self, s: int):
        self.s = s & M64

    def next(self) -> int:
        self.s = (self.s + GOLD) & M64
        z = self.s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
        return z ^ (z >> 31)

    def uniform01(self) -> float:
        return (self.next() >> 11) / 9007199254740992.0

    def randF(self, lo: float, hi: float) -> float:
        return lo + (hi - lo) * self.uniform01()


def _adv_inputs(rng: Rng, n: int):
    rew, val, term, imp = [], [], [], []
    for _ in range(n):
        rew.append(rng.randF(-1.5, 1.5))
        val.append(rng.randF(-2.0, 2.0))
        term.append(1.0 if rng.randF(0.0, 1.0) < 0.12 else 0.0)
        imp.append(rng.randF(0.1, 2.0))
    return [np.array(x) for x in (rew, val, term, imp)]


def kat_vtrace():
    """verify-vtrace-gpu (Exe/Puffer.lean:1072-1098): B=8, T=12, non-unit clips, seed 0x5C1A."""
    B, T = 8, 12
    rng = Rng(0x5C1A)
    rew, val, term, imp = _adv_inputs(rng, B * T)
    return dict(B=B, T=T, gamma=0.99, lam=0.95, rho=2.1, c=1.08, rew=rew, val=val, term=term, imp=imp)


def kat_vtrace_mingru():
    """verify-vtrace-mingru-gpu (Exe/Puffer.lean:1099-1125): as above, seed 0x5C1B, plus bootv[B]."""
    B, T = 8, 12
    rng = Rng(0x5C1B)
    rew, val, term, imp = _adv_inputs(rng, B * T)
    bootv = np.array([rng.randF(-2.0, 2.0) for _ in range(B)])
    return dict(B=B, T=T, gamma=0.99, lam=0.95, rho=2.1, c=1.08, rew=rew, val=val, term=term, imp=imp, bootv=bootv)


def kat_muon():
    """verify-muon-gpu (Exe/Puffer.lean:1126-1151): shapes 16x24, 24x16, 20x20, one chained stream."""
    rng = Rng(0x3E7A)
    cases = []
    for rows, cols in [(16, 24), (24, 16), (20, 20)]:
        W, G, M = [], [], []
        for _ in range(rows * cols):
            W.append(rng.randF(-0.5, 0.5))
            G.append(rng.randF(-0.3, 0.3))
            M.append(rng.randF(-0.2, 0.2))
        cases.append(dict(rows=rows, cols=cols, W=np.array(W), G=np.array(G), M=np.array(M)))
    return dict(lr=0.1, wd=0.0, mu=0.95, eps=1e-7, cases=cases)


def kat_advnorm():
    """verify-advnorm-gpu (Exe/Puffer.lean:1180-1191): n=257, seed 0xAD7, adv in [-3,3)."""
    rng = Rng(0xAD7)
    return dict(adv=np.array([rng.randF(-3.0, 3.0) for _ in range(257)]))


def kat_muon_cpu():
    """verify-muon-cpu (Exe/Puffer.lean:1328-1362): H=24 D=16 O=6, gscale 1/64, seed 0x51A7."""
    H, D, O = 24, 16, 6
    P = H * D + H + O * H + O
    rng = Rng(0x51A7)
    params, grad, mom = [], [], []
    for _ in range(P):
        params.append(rng.randF(-0.5, 0.5))
        grad.append(rng.randF(-2.0, 2.0))
        mom.append(rng.randF(-0.1, 0.1))
    return dict(H=H, D=D, O=O, P=P, lr=0.1, wd=0.0, mu=0.95, eps=1e-7, gscale=1.0 / 64.0,
                params=np.array(params), grad=np.array(grad), mom=np.array(mom))


def init_mlp(din: int, H: int, dout: int, seed: int):
    """initMLP (Puffer/RL/NNTrain.lean:418-422) flattened by flattenMLP; returns (flat, rng)."""
    rng = Rng(seed)

    def rand_mat(rows, cols, scale):
        return [rng.uniform01() * (2.0 * scale) - scale for _ in range(rows * cols)]

    W1 = rand_mat(H, din, math.sqrt(2.0) * (1.0 / math.sqrt(din)))
    W2 = rand_mat(dout, H, 1.0 / math.sqrt(H))
    flat = np.array(W1 + [0.0] * H + W2 + [0.0] * dout)
    return flat, rng


def _rows(rng: Rng, N: int, D: int, A: int, adv_lo: float, adv_hi: float):
    obs, acts, advs, rets, olps = [], [], [], [], []
    for _ in range(N):
        for _ in range(D):
            obs.append(rng.randF(-1.0, 1.0))
        acts.append(math.floor(rng.randF(0.0, float(A))))
        advs.append(rng.randF(adv_lo, adv_hi))
        rets.append(rng.randF(-1.0, 1.0))
        olps.append(rng.randF(-1.5, 0.0))
    return [np.array(x, dtype=np.float64) for x in (obs, acts, advs, rets, olps)]


def kat_ppo_grad():
    """verify-ppo-grad-gpu (Exe/Puffer.lean:1152-1179): N=64 D=12 H=16 A=5, initMLP seed 0x9A73."""
    N, D, H, A = 64, 12, 16, 5
    params, rng = init_mlp(D, H, A + 1, 0x9A73)
    obs, acts, advs, rets, olps = _rows(rng, N, D, A, -1.0, 1.0)
    return dict(N=N, D=D, H=H, A=A, vf=0.5, ent=0.01, clip=0.2, params=params, obs=obs, acts=acts, advs=advs,
                rets=rets, olps=olps)


def kat_train_step():
    """verify-train-step-gpu (Exe/Puffer.lean:1192-1243): N=96 D=12 H=16 A=5, seed 0x77E5, lr 0.1."""
    N, D, H, A = 96, 12, 16, 5
    O = A + 1
    P = H * D + H + O * H + O
    params, rng = init_mlp(D, H, O, 0x77E5)
    obs, acts, advs, rets, olps = _rows(rng, N, D, A, -2.0, 2.0)
    mom = np.array([rng.randF(-0.1, 0.1) for _ in range(P)])
    return dict(N=N, D=D, H=H, A=A, P=P, vf=0.5, ent=0.01, clip=0.2, lr=0.1, wd=0.0, mu=0.95, eps=1e-7,
                params=params, mom=mom, obs=obs, acts=acts, adv=advs, rets=rets, olps=olps)


def kat_train_update():
    """verify-train-update-resident (Exe/Puffer.lean:1244-1287): NT=48 D=12 H=16 A=5, 3 epochs x 4 mb."""
    NT, D, H, A = 48, 12, 16, 5
    O = A + 1
    P = H * D + H + O * H + O
    rng = Rng(0x9A7C33)
    pm0 = np.array([rng.randF(-0.3, 0.3) for _ in range(2 * P)])
    obs = np.array([rng.randF(-1.0, 1.0) for _ in range(NT * D)])
    acts, adv, rets, olps = [], [], [], []
    for _ in range(NT):
        acts.append(math.floor(rng.randF(0.0, float(A))))
        adv.append(rng.randF(-2.0, 2.0))
        rets.append(rng.randF(-1.0, 1.0))
        olps.append(rng.randF(-1.5, 0.0))
    return dict(NT=NT, D=D, H=H, A=A, P=P, epochs=3, numMB=4, vf=0.5, ent=0.01, clip=0.2, lr=0.05, wd=0.0,
                mu=0.95, eps=1e-7, perm_seed=0x1234, pm0=pm0, obs=obs, acts=np.array(acts, dtype=np.float64),
                adv=np.array(adv), rets=np.array(rets), olps=np.array(olps))


def synthetic_rollout(N: int, T: int, D: int, A: int, seed: int, obs_kind: str = "normal", reward_kind: str = "bern",
                      done_p: float = 0.01):
    """Seeded synthetic rollout columns in the shapes BASELINE's configs name (obs N(0,1) or U(0,1);
    actions uniform; rewards Bernoulli(0.5) / U(-1,1) / N(0,1); dones Bernoulli(done_p)). numpy's
    Generator stands in for the env; the seed is recorded by the caller."""
    g = np.random.default_rng(seed)
    NT = N * T
    if obs_kind == "uniform":
        obs = g.random((NT, D), dtype=np.float32)
    else:
        obs = g.standard_normal((NT, D), dtype=np.float32)
    acts = g.integers(0, A, NT).astype(np.float64)
    if reward_kind == "bern":
        rew = (g.random(NT) < 0.5).astype(np.float64)
    elif reward_kind == "uniform":
        rew = g.uniform(-1.0, 1.0, NT)
    else:
        rew = g.standard_normal(NT)
    term = (g.random(NT) < done_p).astype(np.float64)
    return obs, acts, rew, term


def kat_mingru_grad():
    """verify-mingru-grad-gpu (Exe/Puffer.lean:2398-2440): D=5 H=32 L=3 A=4 T=7, B=2 sequences, initMinGRU
    seed 0x6A5D, a terminal at t=3 in every sequence; vf .5 ent .01 clip .2 vfClip .2. Returns the
    per-sequence arrays and the time-major packing the batched kernel takes."""
    from oracle import oracle as O

    D, H, L, A, T, B = 5, 32, 3, 4, 7, 2
    params, s = O.init_mingru(D, H, L, A, 0x6A5D)
    rng = Rng(s)
    seqs = {k: [] for k in ("obs", "act", "adv", "ret", "old", "term", "ov")}
    for _ in range(B):
        o, ac, ad, re, ol, tm, ov = [], [], [], [], [], [], []
        for t in range(T):
            for _ in range(D):
                o.append(rng.randF(-1.0, 1.0))
            ac.append(float(rng.next() % A))
            ad.append(rng.randF(-1.0, 1.0))
            re.append(rng.randF(0.0, 2.0))
            ol.append(-1.0)
            tm.append(1.0 if t == 3 else 0.0)
            ov.append(rng.randF(-0.5, 0.5))
        for k, v in zip(seqs, (o, ac, ad, re, ol, tm, ov)):
            seqs[k].append(np.array(v))
    obsTB = np.zeros(T * B * D)
    scal = np.zeros(6 * T * B)
    for b in range(B):
        for t in range(T):
            obsTB[(t * B + b) * D:(t * B + b + 1) * D] = seqs["obs"][b][t * D:(t + 1) * D]
            for q, k in enumerate(("act", "adv", "ret", "old", "term", "ov")):
                scal[q * T * B + t * B + b] = seqs[k][b][t]
    return dict(D=D, H=H, L=L, A=A, T=T, B=B, K=3, vf=0.5, ent=0.01, clip=0.2, vfClip=0.2, params=params, seqs=seqs,
                obsTB=obsTB, scal=scal)


def kat_mingru_update(K=3, enc_act=0):
    """A small whole MinGRU update (no reference verify mode exists for it): N=12 segments x T=6, D=5 H=16 L=2
    A=3, 3 minibatches of 4 sampled segments, seed 0x3617. Rewards U(-1,1), dones Bernoulli(.15), actions
    uniform, old log-probs U(-2,-0.5), values U(-1,1), bootstrap U(-1,1); initMinGRU(0x6A5E)."""
    from oracle import oracle as O

    N, T, D, H, L, A = 12, 6, 5, 16, 2, 3
    params, _ = O.init_mingru(D, H, L, A, 0x6A5E, K)
    rng = Rng(0x3617)
    NT = N * T
    obs = np.array([rng.randF(0.0, 1.0) for _ in range(NT * D)])
    rew = np.array([rng.randF(-1.0, 1.0) for _ in range(NT)])
    term = np.array([1.0 if rng.randF(0.0, 1.0) < 0.15 else 0.0 for _ in range(NT)])
    act = np.array([float(rng.next() % A) for _ in range(NT)])
    logp = np.array([rng.randF(-2.0, -0.5) for _ in range(NT)])
    val0 = np.array([rng.randF(-1.0, 1.0) for _ in range(NT)])
    boot = np.array([rng.randF(-1.0, 1.0) for _ in range(N)])
    P = params.size
    pm0 = np.concatenate([params, np.zeros(P)])
    return dict(N=N, T=T, D=D, H=H, L=L, A=A, K=K, enc_act=enc_act, numMB=3, mbSegs=4, rng=0xC0FFEE, lr=0.02,
                gamma=0.995, lam=0.90, rho=1.0, c=1.0, alpha=0.8, beta=0.2, wd=0.0, mu=0.95, eps=1e-7, vf=0.5,
                ent=0.01, clip=0.2, vfClip=0.2, maxGradNorm=1.5, pm0=pm0, obs=obs, rew=rew, term=term, act=act,
                logp=logp, val0=val0, boot=boot)
