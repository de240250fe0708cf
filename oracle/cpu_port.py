"""CPU restatement of the MLP PPO+Muon update in numpy (f64, OpenBLAS on every host core).
TEST INFRASTRUCTURE / CPU BASELINE, NOT PRODUCT CODE.

The reference's CPU path for this update is ffi/pufferblas.c:699-747 (cblas_dgemm forward and
backward of a one-hidden-layer MLP plus a scalar per-row PPO backward) followed by muon_mat_cpu
(ffi/pufferblas.c:1369-1400). This module restates that pattern per layer for L hidden layers and
a chosen activation, with the Newton-Schulz matmuls also on BLAS (the reference's naive triple
loops would take minutes per 2048x2048 matrix), so it can time the deep configuration the reference
itself cannot run. bench.py uses it for cpu_baseline and for `--impl reference` when the workload is
outside what the reference's compiled C supports.
"""
from __future__ import annotations

import time

import numpy as np


def act_fwd(z, act):
    if act == 0:
        return np.maximum(z, 0.0)
    u = 0.7978845608028654 * (z + 0.044715 * (z * z * z))
    return 0.5 * z * (1.0 + np.tanh(u))


def act_grad(z, act):
    if act == 0:
        return (z > 0).astype(z.dtype)
    u = 0.7978845608028654 * (z + 0.044715 * (z * z * z))
    t = np.tanh(u)
    return 0.5 * (1 + t) + 0.5 * z * (1 - t * t) * 0.7978845608028654 * (1 + 3 * 0.044715 * z * z)


def layers_of(D, H, A, L):
    out, off = [], 0
    for l in range(L + 1):
        fin = D if l == 0 else H
        fout = A + 1 if l == L else H
        out.append((off, off + fout * fin, fout, fin))
        off += fout * fin + fout
    return out, off


def ppo_grad(params, obs, acts, adv, ret, olp, D, H, A, L, act, vf=0.5, ent=0.01, clip=0.2, ov=None, vfclip=0.0):
    """Summed PPO-objective gradient (pufferblas.c:699-747 generalised to L layers)."""
    lay, P = layers_of(D, H, A, L)
    g = np.zeros(P)
    hs, zs = [obs], []
    h = obs
    for l in range(L):
        oW, ob, fout, fin = lay[l]
        W = params[oW:oW + fout * fin].reshape(fout, fin)
        z = h @ W.T + params[ob:ob + fout]
        zs.append(z)
        h = act_fwd(z, act)
        hs.append(h)
    oW, ob, fout, fin = lay[L]
    Wo = params[oW:oW + fout * fin].reshape(fout, fin)
    out = h @ Wo.T + params[ob:ob + fout]
    logits = out[:, :A]
    lse = np.log(np.exp(logits).sum(1))
    p = np.exp(logits - lse[:, None])
    pout = (p * logits).sum(1)
    a = acts.astype(np.int64)
    logpA = logits[np.arange(len(a)), a] - lse
    ratio = np.exp(logpA - olp)
    lo, hi = 1 - clip, 1 + clip
    rc = np.clip(ratio, lo, hi)
    dPol = np.where(adv * ratio <= adv * rc, adv * ratio, adv * ((lo < ratio) & (ratio < hi)) * ratio)
    dout = np.empty_like(out)
    onehot = np.zeros_like(logits)
    onehot[np.arange(len(a)), a] = 1.0
    dout[:, :A] = dPol[:, None] * (onehot - p) + ent * p * (pout[:, None] - logits)
    vnew = out[:, A]
    dv = vnew - ret
    if ov is not None and vfclip > 0:
        dd = vnew - ov
        vc = ov + np.clip(dd, -vfclip, vfclip)
        keep = ((vnew - ret) ** 2 >= (vc - ret) ** 2) | ((dd > -vfclip) & (dd < vfclip))
        dv = np.where(keep, dv, 0.0)
    dout[:, A] = -vf * dv
    d = dout
    for l in range(L, -1, -1):
        oW, ob, fout, fin = lay[l]
        g[ob:ob + fout] = d.sum(0)
        g[oW:oW + fout * fin] = (d.T @ hs[l]).ravel()
        if l == 0:
            break
        W = params[oW:oW + fout * fin].reshape(fout, fin)
        d = (d @ W) * act_grad(zs[l - 1], act)
    return g


def newton_schulz(U, coeffs, eps):
    X = U / (np.linalg.norm(U) + eps)
    tr = X.shape[0] > X.shape[1]
    if tr:
        X = X.T
    for a, b, c in coeffs:
        A = X @ X.T
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    return X.T if tr else X


def muon_step(pm, g, D, H, A, L, lr, wd, mu, eps, coeffs, maxgn, sc):
    lay, P = layers_of(D, H, A, L)
    gn = np.sqrt(np.sum((g * sc) ** 2))
    cc = ((maxgn / gn) if (maxgn > 0 and gn > maxgn) else 1.0) * sc
    g = g * cc
    par, mom = pm[:P], pm[P:]
    for oW, ob, fout, fin in lay:
        n = fout * fin
        m = mu * mom[oW:oW + n] + g[oW:oW + n]
        mom[oW:oW + n] = m
        u = (g[oW:oW + n] + mu * m).reshape(fout, fin)
        X = newton_schulz(u, coeffs, eps)
        par[oW:oW + n] = (1 - lr * wd) * par[oW:oW + n] + lr * np.sqrt(max(1.0, fout / fin)) * X.ravel()
        mb = mu * mom[ob:ob + fout] + g[ob:ob + fout]
        mom[ob:ob + fout] = mb
        par[ob:ob + fout] = par[ob:ob + fout] * (1 - lr * wd) + lr * (g[ob:ob + fout] + mu * mb)
    return pm


def timed_update_sample(D, H, A, L, act, Nmb, epochs, num_mb, coeffs, rows=4096, seed=0):
    """Times one minibatch's gradient on `rows` rows and one whole-network Muon step, and scales to
    one update of epochs x num_mb minibatches of Nmb rows. Returns (seconds per update, detail)."""
    g = np.random.default_rng(seed)
    lay, P = layers_of(D, H, A, L)
    pm = np.zeros(2 * P)
    for oW, ob, fout, fin in lay:
        lim = np.sqrt(6.0 / (fin + fout))
        pm[oW:oW + fout * fin] = g.uniform(-lim, lim, fout * fin)
    obs = g.standard_normal((rows, D))
    acts = g.integers(0, A, rows).astype(float)
    adv = g.standard_normal(rows)
    ret = g.standard_normal(rows)
    olp = np.full(rows, np.log(1.0 / A))
    t0 = time.perf_counter()
    advn = (adv - adv.mean()) / (adv.std() + 1e-8)
    grad = ppo_grad(pm[:P], obs, acts, advn, ret, olp, D, H, A, L, act, ov=ret, vfclip=0.2)
    t1 = time.perf_counter()
    muon_step(pm, grad, D, H, A, L, 0.02, 0.0, 0.95, 1e-12, coeffs, 1.5, 1.0 / rows)
    t2 = time.perf_counter()
    t_rows, t_muon = t1 - t0, t2 - t1
    per_update = epochs * num_mb * (Nmb / rows * t_rows + t_muon)
    return per_update, dict(rows=rows, t_rows=t_rows, t_muon=t_muon)


def mingru_timed_sample(D, H, L, A, K, enc_act, T, mb_segs, num_mb, coeffs, nseq=None, threads=None, seed=0):
    """Host-core time of one MinGRU update, from a bounded sample: the BPTT gradient of `nseq` sequences
    (the reference's scalar C lean_ffi_mingru_ppo_grad_seq, ffi/pufferffi.c:763-876, when K = 3 and the
    encoder is linear, else our C restatement of it), one sequence per host thread, plus one Muon step
    of every MinGRU matrix with the Newton-Schulz matmuls on numpy BLAS. Returns (seconds per update,
    details). The reference's own trainer runs one sequence at a time on one core."""
    import concurrent.futures as cf
    import ctypes as C
    import os

    from oracle import oracle as O

    threads = threads or os.cpu_count() or 1
    nseq = nseq or 8 * threads
    g = np.random.default_rng(seed)
    params, _ = O.init_mingru(D, H, L, A, 0x51 + seed, K)
    P = params.size
    use_ref = K == 3 and enc_act == 0 and O.ref_available()
    seqs = []
    for _ in range(nseq):
        seqs.append([g.uniform(0, 1, T * D), g.integers(0, A, T).astype(float), g.standard_normal(T),
                     g.uniform(-1, 1, T), np.full(T, np.log(1.0 / A)), (g.random(T) < 0.005).astype(float),
                     g.standard_normal(T)])

    def one(s):
        if use_ref:
            r = O.ref_call(O.ref_cpu(), "lean_ffi_mingru_ppo_grad_seq", C.c_void_p, O.FA(params), *[O.FA(x) for x in s],
                           T, H, D, L, A, 0.5, 0.01, 0.2, 0.2)
            return O.read_float_array(r)[:P]
        return O.mingru_grad_seq(params, *s, T, H, D, L, A, K, enc_act)[0]

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        grads = list(ex.map(one, seqs))
    t_grad = time.perf_counter() - t0
    gsum = np.sum(grads, axis=0)
    # one Muon step over the flattenMG matrices (wEnc H x D, layers K*H x H, wDec A x H, wVal 1 x H)
    shapes = [(H, D)] + [(K * H, H)] * L + [(A, H), (1, H)]
    t0 = time.perf_counter()
    for r_, c_ in shapes:
        newton_schulz(g.standard_normal((r_, c_)), coeffs, 1e-7)
    t_muon = time.perf_counter() - t0
    per_mb = t_grad * (mb_segs / nseq) + t_muon
    return per_mb * num_mb, {"nseq": nseq, "threads": threads, "t_grad": t_grad, "t_muon": t_muon,
                             "grad_source": "reference C" if use_ref else "restatement", "finite":
                             bool(np.isfinite(gsum).all())}
