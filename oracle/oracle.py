"""Python handle on the test oracle. TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Two libraries sit behind it:

* ``oracle/_build/liborc.so`` -- our f64 C restatement of the reference algorithms (restate.c),
  each function citing the reference file:line it follows;
* ``oracle/_ref/libref_cpu.so`` / ``libref_cudafb.so`` -- the reference's own C sources
  (ffi/pufferffi.c, ffi/pufferblas.c, ffi/puffercuda.cu) compiled where they lie, used to pin the
  restatement and, on the GPU box, as the timed CPU baseline of the reference arm.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_ORC = None
_REF_CPU = None
_REF_CUDAFB = None

_dp = C.POINTER(C.c_double)
_sz = C.c_size_t
_d = C.c_double


def _ptr(a):
    return a.ctypes.data_as(_dp) if a is not None else None


def build():
    """Compile liborc.so (and, when the reference tree is present, oracle/_ref)."""
    import subprocess

    subprocess.check_call(["make", "-s", "-C", HERE, "all"])
    ref = reference_dir()
    if ref:
        subprocess.check_call(["make", "-s", "-C", HERE, "ref", "REF=" + ref])


def reference_dir():
    """The reference checkout: $PL_REFERENCE_DIR, else a directory named `reference` beside this
    repository; None when neither exists (the GPU box, which uses the prebuilt oracle/_ref files)."""
    cand = os.environ.get("PL_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isdir(cand) else None


def orc():
    global _ORC
    if _ORC is None:
        path = os.path.join(HERE, "_build", "liborc.so")
        if not os.path.exists(path):
            build()
        lib = C.CDLL(path)
        lib.orc_rng_next.restype = C.c_uint64
        lib.orc_rng_next.argtypes = [C.POINTER(C.c_uint64)]
        lib.orc_vtrace.argtypes = [_dp] * 4 + [_sz, _sz] + [_d] * 4 + [_dp]
        lib.orc_vtrace_mingru.argtypes = [_dp] * 5 + [_sz, _sz] + [_d] * 4 + [_dp]
        lib.orc_adv_l1.argtypes = [_dp, _sz, _sz, _dp]
        lib.orc_gae_soa.argtypes = [_dp] * 3 + [_sz, _sz, _d, _d, _dp]
        lib.orc_shuffle_perm.argtypes = [_sz, _sz, C.c_uint64, _dp]
        lib.orc_normalize_adv.argtypes = [_dp, _sz, _dp]
        lib.orc_frob_norm.restype = _d
        lib.orc_frob_norm.argtypes = [_dp, C.c_int, C.c_int]
        lib.orc_newton_schulz.argtypes = [_dp, C.c_int, C.c_int, _d, _dp, C.c_int, _dp]
        lib.orc_muon_stepmat.argtypes = [_dp, _dp, _dp, C.c_int, C.c_int, _d, _d, _d, _d, _dp, C.c_int, _dp, _dp]
        lib.orc_muon_stepvec.argtypes = [_dp, _dp, _dp, C.c_int, _d, _d, _d, _dp, _dp]
        lib.orc_mlp_param_count.restype = _sz
        lib.orc_mlp_param_count.argtypes = [_sz] * 4
        lib.orc_mlp_ppo_grad.argtypes = [_dp] * 7 + [_sz] * 5 + [C.c_int] + [_d] * 4 + [_dp] * 3
        lib.orc_grad_clip.argtypes = [_dp, _sz, _d, _d]
        lib.orc_apply_muon.argtypes = [_dp, _dp] + [_sz] * 4 + [_d] * 4 + [_dp, C.c_int]
        lib.orc_train_update.argtypes = ([_dp] * 8 + [_sz] * 5 + [C.c_int] + [_sz] * 2 + [_d] * 9
                                         + [_dp, C.c_int])
        lib.orc_init_mlp.restype = C.c_uint64
        lib.orc_init_mlp.argtypes = [_sz, _sz, _sz, C.c_uint64, _dp]
        lib.orc_cosine_lr.restype = _d
        lib.orc_cosine_lr.argtypes = [_d, _d, _sz, _sz]
        lib.orc_mg_param_count.restype = _sz
        lib.orc_mg_param_count.argtypes = [_sz] * 5
        lib.orc_mingru_grad_seq.argtypes = [_dp] * 8 + [_sz] * 6 + [C.c_int] + [_d] * 4 + [_dp] * 3
        lib.orc_mingru_grad_batch.argtypes = [_dp] * 3 + [_sz] * 7 + [C.c_int] + [_d] * 4 + [_dp]
        lib.orc_prio_sample.argtypes = [_dp, _sz, _sz, _d, _d, C.c_uint64, _dp, _dp]
        lib.orc_gather_seq_minibatch.argtypes = [_dp] * 7 + [_sz, _sz, _dp]
        lib.orc_apply_muon_mg.argtypes = [_dp, _dp] + [_sz] * 5 + [_d] * 4 + [_dp, C.c_int]
        _ip = C.POINTER(C.c_int)
        lib.orc_mingru_grad_seq_md.argtypes = [_dp] * 8 + [_sz] * 6 + [C.c_int] + [_d] * 4 + [_sz, _ip] + [_dp] * 3
        lib.orc_mingru_grad_batch_md.argtypes = [_dp] * 3 + [_sz] * 7 + [C.c_int] + [_d] * 4 + [_sz, _ip, _dp]
        lib.orc_gather_seq_minibatch_md.argtypes = [_dp] * 7 + [_sz, _sz, _sz, _dp]
        lib.orc_mingru_update_md.restype = C.c_uint64
        lib.orc_mingru_update_md.argtypes = ([_dp] * 8 + [_sz] * 7 + [C.c_int] + [_sz] * 2 + [_d] * 6 + [C.c_uint64]
                                             + [_d] * 9 + [_dp, C.c_int, _sz, _ip])
        lib.orc_lstm_param_count.restype = _sz
        lib.orc_lstm_param_count.argtypes = [_sz] * 3
        lib.orc_lstm_grad_seq.argtypes = [_dp] * 9 + [_sz] * 4 + [_d] * 3 + [_dp] * 3
        lib.orc_lstm_grad_batch.argtypes = [_dp] * 9 + [_sz] * 5 + [_d] * 3 + [_dp]
        lib.orc_lstm_gae_boot_norm.argtypes = [_dp] * 4 + [_sz, _sz, _d, _d, _dp]
        lib.orc_mingru_update.restype = C.c_uint64
        lib.orc_mingru_update.argtypes = ([_dp] * 8 + [_sz] * 7 + [C.c_int] + [_sz] * 2 + [_d] * 6 + [C.c_uint64]
                                          + [_d] * 9 + [_dp, C.c_int])
        lib.orc_mlp_ppo_grad_wide.argtypes = ([_dp] * 7 + [_sz] * 5 + [C.c_int, C.POINTER(C.c_int)] + [_d] * 5
                                              + [_dp] * 3)
        lib.orc_train_update_wide.argtypes = ([_dp] * 8 + [C.POINTER(C.c_int)] + [_sz] * 5 + [C.c_int] + [_sz] * 2
                                              + [_d] * 10 + [_dp, C.c_int])
        lib.orc_init_mingru.restype = C.c_uint64
        lib.orc_init_mingru.argtypes = [_sz] * 5 + [C.c_uint64, _dp]
        _ORC = lib
    return _ORC


# ---------------------------------------------------------------------------------------------
# The reference's PufferLib-tuned Newton-Schulz table (Puffer/Float/Muon.lean:64-67) and the
# single-row quintic schedule BASELINE's timing configs name.
MUON_COEFFS = np.array([[4.0848, -6.8946, 2.9270], [3.9505, -6.3029, 2.6377], [3.7418, -5.5913, 2.3037],
                        [2.8769, -3.1427, 1.2046], [2.8366, -3.0525, 1.2012]], dtype=np.float64)
QUINTIC_COEFFS = np.array([[3.4445, -4.7750, 2.0315]] * 5, dtype=np.float64)


def f64(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def vtrace(rew, val, term, imp, B, T, gamma, lam, rho, c):
    out = np.zeros(B * T)
    rew, val, term, imp = map(f64, (rew, val, term, imp))
    orc().orc_vtrace(_ptr(rew), _ptr(val), _ptr(term), _ptr(imp), B, T, gamma, lam, rho, c, _ptr(out))
    return out


def vtrace_mingru(rew, val, term, imp, bootv, B, T, gamma, lam, rho, c):
    out = np.zeros(B * T)
    rew, val, term, imp, bootv = map(f64, (rew, val, term, imp, bootv))
    orc().orc_vtrace_mingru(_ptr(rew), _ptr(val), _ptr(term), _ptr(imp), _ptr(bootv), B, T, gamma, lam, rho, c,
                            _ptr(out))
    return out


def adv_l1(adv, N, T):
    out = np.zeros(N)
    adv = f64(adv)
    orc().orc_adv_l1(_ptr(adv), N, T, _ptr(out))
    return out


def gae_soa(vals, rews, terms, N, T, gamma, lam):
    out = np.zeros(2 * N * T)
    vals, rews, terms = map(f64, (vals, rews, terms))
    orc().orc_gae_soa(_ptr(vals), _ptr(rews), _ptr(terms), N, T, gamma, lam, _ptr(out))
    return out


def shuffle_perm(NT, epochs, rng):
    out = np.zeros(NT * epochs)
    orc().orc_shuffle_perm(NT, epochs, C.c_uint64(rng & 0xFFFFFFFFFFFFFFFF), _ptr(out))
    return out


def normalize_adv(adv):
    adv = f64(adv)
    out = np.zeros_like(adv)
    orc().orc_normalize_adv(_ptr(adv), adv.size, _ptr(out))
    return out


def frob_norm(X, rows, cols):
    X = f64(X)
    return orc().orc_frob_norm(_ptr(X), rows, cols)


def newton_schulz(X0, rows, cols, eps, coeffs=MUON_COEFFS):
    X0 = f64(X0)
    co = f64(coeffs)
    out = np.zeros(rows * cols)
    orc().orc_newton_schulz(_ptr(X0), rows, cols, eps, _ptr(co), co.shape[0], _ptr(out))
    return out


def muon_stepmat(W, G, M, rows, cols, lr, wd, mu, eps, coeffs=MUON_COEFFS):
    W, G, M = map(f64, (W, G, M))
    co = f64(coeffs)
    nW = np.zeros(rows * cols)
    nM = np.zeros(rows * cols)
    orc().orc_muon_stepmat(_ptr(W), _ptr(G), _ptr(M), rows, cols, lr, wd, mu, eps, _ptr(co), co.shape[0], _ptr(nW),
                           _ptr(nM))
    return nW, nM


def param_count(D, H, A, L=1):
    return int(orc().orc_mlp_param_count(D, H, A, L))


def mlp_ppo_grad(params, obs, acts, advs, rets, olps, N, D, H, A, L=1, act=0, vf=0.5, ent=0.01, clip=0.2, ov=None,
                 vfClip=0.0):
    P = param_count(D, H, A, L)
    g = np.zeros(P)
    nlp = np.zeros(N)
    nv = np.zeros(N)
    params, obs, acts, advs, rets, olps = map(f64, (params, obs, acts, advs, rets, olps))
    ovp = _ptr(f64(ov)) if ov is not None else None
    orc().orc_mlp_ppo_grad(_ptr(params), _ptr(obs), _ptr(acts), _ptr(advs), _ptr(rets), _ptr(olps), ovp, N, D, H,
                           A, L, act, vf, ent, clip, vfClip, _ptr(g), _ptr(nlp), _ptr(nv))
    return g, nlp, nv


def grad_clip(g, maxNorm, sc):
    g = f64(g).copy()
    orc().orc_grad_clip(_ptr(g), g.size, maxNorm, sc)
    return g


def apply_muon(pm, g, D, H, A, L, lr, wd, mu, eps, coeffs=MUON_COEFFS):
    pm = f64(pm).copy()
    g = f64(g)
    co = f64(coeffs)
    orc().orc_apply_muon(_ptr(pm), _ptr(g), D, H, A, L, lr, wd, mu, eps, _ptr(co), co.shape[0])
    return pm


def train_update(pm, obs, acts, adv, ret, olp, perm, NT, D, H, A, epochs, numMB, lr, wd, mu, eps, vf, ent, clip,
                 L=1, act=0, ov=None, vfClip=0.0, maxGradNorm=0.0, coeffs=MUON_COEFFS):
    pm = f64(pm).copy()
    obs, acts, adv, ret, olp, perm = map(f64, (obs, acts, adv, ret, olp, perm))
    co = f64(coeffs)
    ovp = _ptr(f64(ov)) if ov is not None else None
    orc().orc_train_update(_ptr(pm), _ptr(obs), _ptr(acts), _ptr(adv), _ptr(ret), _ptr(olp), ovp, _ptr(perm), NT,
                           D, H, A, L, act, epochs, numMB, lr, wd, mu, eps, vf, ent, clip, vfClip, maxGradNorm,
                           _ptr(co), co.shape[0])
    return pm


def init_mlp(din, H, dout, seed):
    P = H * din + H + dout * H + dout
    flat = np.zeros(P)
    s = orc().orc_init_mlp(din, H, dout, C.c_uint64(seed), _ptr(flat))
    return flat, int(s)


def cosine_lr(lr, min_ratio, u, updates):
    return float(orc().orc_cosine_lr(lr, min_ratio, u, updates))


# ---------------------------------------------------------------------------------------------
# MinGRU (flattenMG layout; K = 3 is the reference layer, K = 2 the gate+candidate variant)
def mg_param_count(D, H, L, A, K=3):
    return int(orc().orc_mg_param_count(D, H, L, A, K))


def init_mingru(D, H, L, A, seed, K=3):
    flat = np.zeros(mg_param_count(D, H, L, A, K))
    s = orc().orc_init_mingru(D, H, L, A, K, C.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), _ptr(flat))
    return flat, int(s)


def _heads(hs):
    """(W, int array) for a head-size list; None = one categorical head (W = 1)."""
    if hs is None:
        return 1, None
    return len(hs), (C.c_int * len(hs))(*[int(x) for x in hs])


def mingru_grad_seq(params, obs, acts, advs, rets, olps, terms, ovs, T, H, D, L, A, K=3, enc_act=0, vf=0.5, ent=0.01,
                    clip=0.2, vfClip=0.2, hs=None):
    """hs: multi-discrete head sizes (sum A); acts then holds len(hs) actions per step."""
    P = mg_param_count(D, H, L, A, K)
    g, nl, nv = np.zeros(P), np.zeros(T), np.zeros(T)
    arrs = list(map(f64, (params, obs, acts, advs, rets, olps, terms, ovs)))
    W, hsa = _heads(hs)
    orc().orc_mingru_grad_seq_md(*[_ptr(a) for a in arrs], T, H, D, L, A, K, enc_act, vf, ent, clip, vfClip, W, hsa,
                                 _ptr(g), _ptr(nl), _ptr(nv))
    return g, nl, nv


def mingru_grad_batch(params, obsTB, scal, B, T, H, D, L, A, K=3, enc_act=0, vf=0.5, ent=0.01, clip=0.2, vfClip=0.2,
                      hs=None):
    """[g(P); newlp(T*B); newval(T*B)] for B time-major packed sequences (scal = [act|adv|ret|old|term|ov], the act
    block len(hs) wide per row with multi-discrete heads)."""
    P = mg_param_count(D, H, L, A, K)
    out = np.zeros(P + 2 * T * B)
    params, obsTB, scal = map(f64, (params, obsTB, scal))
    W, hsa = _heads(hs)
    orc().orc_mingru_grad_batch_md(_ptr(params), _ptr(obsTB), _ptr(scal), B, T, H, D, L, A, K, enc_act, vf, ent, clip,
                                   vfClip, W, hsa, _ptr(out))
    return out


def prio_sample(advL1, N, mbSegs, alpha, beta, rng):
    seg, mp = np.zeros(mbSegs), np.zeros(mbSegs)
    advL1 = f64(advL1)
    orc().orc_prio_sample(_ptr(advL1), N, mbSegs, alpha, beta, C.c_uint64(rng & 0xFFFFFFFFFFFFFFFF), _ptr(seg),
                          _ptr(mp))
    return seg, mp


def gather_seq_minibatch(act, logp, term, adv, value, seg, mbPrio, T, Bmb, W=1):
    out = np.zeros((W + 5) * T * Bmb)
    arrs = list(map(f64, (act, logp, term, adv, value, seg, mbPrio)))
    orc().orc_gather_seq_minibatch_md(*[_ptr(a) for a in arrs], T, Bmb, W, _ptr(out))
    return out


def apply_muon_mg(pm, g, D, H, L, A, lr, wd, mu, eps, K=3, coeffs=MUON_COEFFS):
    pm = f64(pm).copy()
    g, co = f64(g), f64(coeffs)
    orc().orc_apply_muon_mg(_ptr(pm), _ptr(g), D, H, L, A, K, lr, wd, mu, eps, _ptr(co), co.shape[0])
    return pm


def mingru_update(pm, obs, rew, term, act, logp, val0, boot, N, T, D, H, L, A, numMB, mbSegs, rng, lr, K=3,
                  enc_act=0, gamma=0.995, lam=0.90, rho=1.0, c=1.0, alpha=0.8, beta=0.2, wd=0.0, mu=0.95, eps=1e-7,
                  vf=0.5, ent=0.01, clip=0.2, vfClip=0.2, maxGradNorm=1.5, coeffs=MUON_COEFFS, hs=None):
    """One whole MinGRU update (orc_mingru_update_md); returns (pm', rng'). hs: multi-discrete head sizes."""
    pm = f64(pm).copy()
    arrs = list(map(f64, (obs, rew, term, act, logp, val0, boot)))
    co = f64(coeffs)
    W, hsa = _heads(hs)
    r = orc().orc_mingru_update_md(_ptr(pm), *[_ptr(a) for a in arrs], N, T, D, H, L, A, K, enc_act, numMB, mbSegs,
                                   gamma, lam, rho, c, alpha, beta, C.c_uint64(rng & 0xFFFFFFFFFFFFFFFF), lr, wd, mu,
                                   eps, vf, ent, clip, vfClip, maxGradNorm, _ptr(co), co.shape[0], W, hsa)
    return pm, int(r)


# ---------------------------------------------------------------------------------------------
# LSTM (the third recurrent core)
def lstm_param_count(D, H, A):
    return int(orc().orc_lstm_param_count(D, H, A))


def lstm_grad_seq(params, obs, acts, advs, rets, olps, terms, h0, c0, T, H, D, A, vf=0.5, ent=0.01, clip=0.2):
    P = lstm_param_count(D, H, A)
    g, nl, nv = np.zeros(P), np.zeros(T), np.zeros(T)
    arrs = list(map(f64, (params, obs, acts, advs, rets, olps, terms, h0, c0)))
    orc().orc_lstm_grad_seq(*[_ptr(a) for a in arrs], T, H, D, A, vf, ent, clip, _ptr(g), _ptr(nl), _ptr(nv))
    return g, nl, nv


def lstm_grad_batch(params, obsB, acts, advs, rets, olps, terms, h0s, c0s, B, T, H, D, A, vf=0.5, ent=0.01, clip=0.2):
    """[g(P); newlp(T*B); newval(T*B)] of B time-major packed sequences."""
    P = lstm_param_count(D, H, A)
    out = np.zeros(P + 2 * T * B)
    arrs = list(map(f64, (params, obsB, acts, advs, rets, olps, terms, h0s, c0s)))
    orc().orc_lstm_grad_batch(*[_ptr(a) for a in arrs], B, T, H, D, A, vf, ent, clip, _ptr(out))
    return out


def lstm_gae_boot_norm(vals, rews, terms, boot, N, T, gamma, lam):
    out = np.zeros(2 * N * T)
    arrs = list(map(f64, (vals, rews, terms, boot)))
    orc().orc_lstm_gae_boot_norm(*[_ptr(a) for a in arrs], N, T, gamma, lam, _ptr(out))
    return out


# ---------------------------------------------------------------------------------------------
# Wide action heads (mode 1 multi-discrete, mode 2 Gaussian) of the one-hidden-layer ReLU MLP
def _hs(hs, W):
    a = (C.c_int * max(W, 1))(*([int(x) for x in hs] if hs is not None else [0] * W))
    return a


def mlp_ppo_grad_wide(params, obs, acts, advs, rets, olps, N, D, H, O, W, mode, hs=None, ov=None, vf=0.5, ent=0.01,
                      clip=0.2, vfClip=0.0, lsLo=-20.0):
    P = H * D + H + O * H + O
    g, nl, nv = np.zeros(P), np.zeros(N), np.zeros(N)
    arrs = list(map(f64, (params, obs, acts, advs, rets, olps)))
    ovp = _ptr(f64(ov)) if ov is not None else None
    orc().orc_mlp_ppo_grad_wide(*[_ptr(a) for a in arrs], ovp, N, D, H, O, W, mode, _hs(hs, W), vf, ent, clip, vfClip,
                                lsLo, _ptr(g), _ptr(nl), _ptr(nv))
    return g, nl, nv


def train_update_wide(pm, obs, acts, adv, ret, olp, perm, NT, D, H, O, W, mode, epochs, numMB, hs=None, ov=None,
                      lr=0.02, wd=0.0, mu=0.95, eps=1e-7, vf=0.5, ent=0.01, clip=0.2, vfClip=0.0, maxGradNorm=0.0,
                      lsLo=-20.0, coeffs=MUON_COEFFS):
    pm = f64(pm).copy()
    arrs = list(map(f64, (obs, acts, adv, ret, olp)))
    ovp = _ptr(f64(ov)) if ov is not None else None
    co = f64(coeffs)
    orc().orc_train_update_wide(_ptr(pm), *[_ptr(a) for a in arrs], ovp, _ptr(f64(perm)), _hs(hs, W), NT, D, H, O, W,
                                mode, epochs, numMB, lr, wd, mu, eps, vf, ent, clip, vfClip, maxGradNorm, lsLo, _ptr(co),
                                co.shape[0])
    return pm


# ---------------------------------------------------------------------------------------------
# The reference's own C, loaded with a malloc-backed Lean object shim (include/lean_compat).
_libc = C.CDLL(None)
_libc.malloc.restype = C.c_void_p
_libc.malloc.argtypes = [C.c_size_t]
_SARRAY_DATA = 24  # m_rc(4) + packed tag word(4) + m_size(8) + m_capacity(8)


def ref_available():
    return os.path.exists(os.path.join(HERE, "_ref", "libref_cpu.so"))


def ref_cpu():
    global _REF_CPU
    if _REF_CPU is None:
        _REF_CPU = C.CDLL(os.path.join(HERE, "_ref", "libref_cpu.so"))
    return _REF_CPU


def ref_cudafb():
    """puffercuda.cu built for its host fallbacks. Loading it on a machine WITH a GPU would send its
    calls to the reference's own kernels, so it is refused whenever a device is visible."""
    global _REF_CUDAFB
    if _REF_CUDAFB is None:
        try:
            import torch

            if torch.cuda.is_available():
                raise RuntimeError("libref_cudafb.so is for golden-vector generation on a GPU-less host only")
        except ImportError:
            pass
        _REF_CUDAFB = C.CDLL(os.path.join(HERE, "_ref", "libref_cudafb.so"))
    return _REF_CUDAFB


def lean_float_array(a) -> int:
    """A fresh Lean FloatArray (rc 1) holding a copy of `a`; the callee consumes it (lean_dec)."""
    a = f64(a).ravel()
    n = a.size
    p = _libc.malloc(_SARRAY_DATA + 8 * max(n, 1))
    hdr = struct.pack("<iIQQ", 1, (248 << 24) | (8 << 16), n, n)
    C.memmove(p, hdr, len(hdr))
    if n:
        C.memmove(p + _SARRAY_DATA, a.ctypes.data, 8 * n)
    return p


def read_float_array(p) -> np.ndarray:
    n = struct.unpack("<Q", C.string_at(p + 8, 8))[0]
    return np.frombuffer(C.string_at(p + _SARRAY_DATA, 8 * n), dtype=np.float64).copy()


def ctor_field(p, i) -> int:
    return struct.unpack("<Q", C.string_at(p + 8 + 8 * i, 8))[0]


def ctor_tag(p) -> int:
    return C.string_at(p + 7, 1)[0]


def ref_call(lib, name, restype, *args):
    f = getattr(lib, name)
    f.restype = restype
    conv = []
    for a in args:
        if isinstance(a, float):
            conv.append(C.c_double(a))
        elif isinstance(a, tuple) and a[0] == "u64":
            conv.append(C.c_uint64(a[1]))
        elif isinstance(a, tuple) and a[0] == "u32":
            conv.append(C.c_uint32(a[1]))
        elif isinstance(a, tuple) and a[0] == "u8":
            conv.append(C.c_uint8(a[1]))
        elif isinstance(a, tuple) and a[0] == "obj":
            conv.append(C.c_void_p(a[1]))
        else:
            conv.append(C.c_size_t(a))
    return f(*conv)


def FA(a):
    return ("obj", lean_float_array(a))
