"""The reference's own CPU update of its one-hidden-layer MLP, composed from the reference's compiled C.
TEST INFRASTRUCTURE / CPU BASELINE, NOT PRODUCT CODE.

oracle/_ref/libref_cpu.so is ffi/pufferffi.c + ffi/pufferblas.c compiled from the reference's sources
(oracle/Makefile). One update follows the reference's CPU trainer (Puffer/RL/FFITrain.lean, the BLAS
minibatch step updatePPOIdxBlasFFI, :291-306) call for call:

    lean_ffi_gae_soa                      advantages + returns          ffi/pufferffi.c:946-971
    lean_ffi_shuffle_perm                 epochs x Fisher-Yates          ffi/pufferffi.c:1017-1041
    per epoch x minibatch (mbSize = NT / numMB, the last takes the remainder):
      lean_ffi_gather_minibatch           rows of the minibatch          ffi/pufferffi.c:1046-1081
      normalizeAdv                        (Lean in the reference: Puffer/RL/NNTrain.lean:274-279; here
                                          the restatement's bit-exact form, oracle/restate.c)
      lean_ffi_mlp_ppo_grad_batch_blas    summed objective gradient      ffi/pufferblas.c:699-747
      global clip of the mean gradient    (Lean, FFITrain.lean:298-302; numpy here)
      lean_ffi_muon_step_mlp              Muon step, gscale = clip / n   ffi/pufferblas.c:1411-1428

with the reference's BLAS on every host core (lean_ffi_blas_set_threads, ffi/pufferblas.c:1332).
"""
from __future__ import annotations

import ctypes as C
import os
import time

import numpy as np

from oracle import oracle as O

VP = C.c_void_p


def _arr(p):
    return O.read_float_array(p)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def set_threads(n: int) -> None:
    """The reference's BLAS thread count (lean_ffi_blas_set_threads), whatever OMP_NUM_THREADS says."""
    O.ref_call(O.ref_cpu(), "lean_ffi_blas_set_threads", VP, n, ("obj", 1))


def update(pm, obs, acts, olps, vals, rews, terms, N, T, D, H, A, epochs, num_mb, seed, lr=0.02, wd=0.0, mu=0.95,
           eps=1e-7, vf=0.5, ent=0.01, clip=0.2, max_grad_norm=0.0, gamma=0.995, lam=0.90):
    """One whole update on the host through the reference's C; returns the new [params; mom]."""
    lib = O.ref_cpu()
    FA = O.FA
    NT = N * T
    P = H * D + H + (A + 1) * H + A + 1
    ga = _arr(O.ref_call(lib, "lean_ffi_gae_soa", VP, FA(vals), FA(rews), FA(terms), N, T, gamma, lam))
    adv, ret = ga[:NT], ga[NT:]
    perm = _arr(O.ref_call(lib, "lean_ffi_shuffle_perm", VP, NT, epochs, ("u64", seed)))
    mb = max(1, NT // num_mb)
    for e in range(epochs):
        for m in range(num_mb):
            lo, hi = m * mb, (NT if m + 1 == num_mb else min(NT, (m + 1) * mb))
            if hi <= lo:
                continue
            n = hi - lo
            tup = O.ref_call(lib, "lean_ffi_gather_minibatch", VP, FA(obs), FA(acts), FA(adv), FA(ret), FA(olps),
                             FA(perm[e * NT + lo:e * NT + hi]), n, D)
            cols = []
            for _ in range(4):
                cols.append(_arr(O.ctor_field(tup, 0)))
                tup = O.ctor_field(tup, 1)
            cols.append(_arr(tup))
            mb_obs, mb_act, mb_adv, mb_ret, mb_olp = cols
            advn = O.normalize_adv(mb_adv)
            g = _arr(O.ref_call(lib, "lean_ffi_mlp_ppo_grad_batch_blas", VP, FA(pm[:P]), FA(mb_obs), FA(mb_act),
                                FA(advn), FA(mb_ret), FA(mb_olp), n, H, D, A, vf, ent, clip))
            mean_norm = float(np.sqrt(np.sum(g[:P] * g[:P]))) / n
            cc = max_grad_norm / mean_norm if (max_grad_norm > 0 and mean_norm > max_grad_norm) else 1.0
            pm = _arr(O.ref_call(lib, "lean_ffi_muon_step_mlp", VP, FA(pm), FA(g[:P]), H, D, A + 1, cc / n, lr, wd,
                                 mu, eps))
    return pm


def timed_updates(pm, cols, N, T, D, H, A, epochs, num_mb, steps, warmup=1, threads=None, **hyper):
    """Seconds per update of `steps` whole updates (after `warmup`) on `threads` host cores (all by
    default), and the final [params; mom]."""
    threads = threads or host_cores()
    set_threads(threads)
    obs, acts, olps, vals, rews, terms = cols
    for i in range(warmup):
        pm = update(pm, obs, acts, olps, vals, rews, terms, N, T, D, H, A, epochs, num_mb, 0xC1 + i, **hyper)
    t0 = time.perf_counter()
    for i in range(steps):
        pm = update(pm, obs, acts, olps, vals, rews, terms, N, T, D, H, A, epochs, num_mb, 0x1C1 + i, **hyper)
    return (time.perf_counter() - t0) / max(1, steps), pm, threads
