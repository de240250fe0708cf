"""pufferlean_b200: B200-native PPO+Muon update path of pufferlean, host-side Python binding.

The compute lives in the C-ABI library ``pufferlean_b200/_build/libpufferlean_b200.so`` (CUDA for
sm_100a, declared in include/pufferlean_b200.h). This module loads it with ctypes and mirrors the
reference's Lean-facing interface for the path (Puffer/Float/CUDA.lean, Puffer/Float/FFI.lean): the
same entry points, argument order and meaning, f64 arrays in and out. There is no CPU fallback: if the
library is missing or no device is usable, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libpufferlean_b200.so")

_lib = None

_dp = C.POINTER(C.c_double)
_sz = C.c_size_t
_d = C.c_double
_vp = C.c_void_p


class PufferError(RuntimeError):
    """A library call returned a non-zero status."""


def lib():
    """The loaded CUDA library (raises if it was not built: run `python -m pufferlean_b200.build`)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise PufferError(f"{LIB_PATH} is missing; build it with `python -m pufferlean_b200.build`")
        L = C.CDLL(LIB_PATH)
        L.pl_last_error.restype = C.c_char_p
        L.pl_kernel_launch_count.restype = C.c_uint64
        L.pl_vtrace.argtypes = [_dp] * 4 + [_sz, _sz] + [_d] * 4 + [_dp]
        L.pl_vtrace_mingru.argtypes = [_dp] * 5 + [_sz, _sz] + [_d] * 4 + [_dp]
        L.pl_vtrace_f32_dev.argtypes = [_vp] * 5 + [_sz, _sz] + [_d] * 4 + [_vp, _vp, _vp]
        L.pl_vtrace_f64_dev.argtypes = [_vp] * 5 + [_sz, _sz] + [_d] * 4 + [_vp, _vp, _vp]
        L.pl_shuffle_perm.argtypes = [_sz, _sz, C.c_uint64, _dp]
        L.pl_gae_soa.argtypes = [_dp] * 3 + [_sz, _sz, _d, _d, _dp]
        L.pl_muon_stepmat.argtypes = [_dp] * 3 + [_sz, _sz] + [_d] * 4 + [_dp]
        _lib = L
        _bind_optional(L)
    return _lib


def _bind_optional(L):
    """Bindings for entry points added after the first milestone (absent symbols are skipped)."""
    specs = {
        "pl_ns_batched_bf16_dev": ([_vp, _sz, _sz, _sz, _d, _dp, _sz, _vp], C.c_int),
        "pl_mlp_ppo_grad": ([_dp] * 6 + [_sz] * 4 + [_d] * 3 + [C.c_uint8, _dp], C.c_int),
        "pl_adv_normalize": ([_dp, _sz, _dp], C.c_int),
        "pl_train_step": ([_dp] * 6 + [_sz] * 4 + [_d] * 7 + [C.c_uint8, _dp], C.c_int),
        "pl_train_update": ([_dp] * 7 + [_sz] * 6 + [_d] * 7 + [C.c_uint8, _dp], C.c_int),
        "pl_policy_load": ([_dp, _sz, C.POINTER(_sz)], C.c_int),
        "pl_policy_download": ([_sz, _sz, _dp], C.c_int),
        "pl_policy_free": ([_sz], C.c_int),
        "pl_train_update_resident": ([_sz] + [_dp] * 6 + [_sz, _dp] + [_sz] * 6 + [_d] * 9 + [C.c_uint8, _dp],
                                     C.c_int),
        "pl_mlp_param_count": ([_sz] * 4, _sz),
        "pl_loss_enable": ([C.c_uint8], C.c_int),
        "pl_read_losses": ([_dp], C.c_int),
    }
    for name, (args, res) in specs.items():
        if hasattr(L, name):
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res


def _check(rc: int, what: str):
    if rc != 0:
        msg = lib().pl_last_error().decode(errors="replace")
        raise PufferError(f"{what} failed (status {rc}): {msg}")


def _f64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def _p(a: np.ndarray):
    return a.ctypes.data_as(_dp)


def device_count() -> int:
    return int(lib().pl_device_count())


def kernel_launch_count() -> int:
    return int(lib().pl_kernel_launch_count())


# ------------------------------------------------------------------------------------------------
# Advantage scans -- Puffer/Float/CUDA.lean:20-31
def cuda_vtrace(rewards, values, terminals, importance, B, T, gamma, lam, rho_clip, c_clip):
    """cudaVtraceFFI: vector-delta V-trace over B x T row-major segments (f64, bit-exact)."""
    r, v, t, i = (_f64(x) for x in (rewards, values, terminals, importance))
    out = np.empty(B * T)
    _check(lib().pl_vtrace(_p(r), _p(v), _p(t), _p(i), B, T, gamma, lam, rho_clip, c_clip, _p(out)), "pl_vtrace")
    return out


def cuda_vtrace_mingru(rewards, values, terms, imps, bootv, B, T, gamma, lam, rho_clip, c_clip):
    """cudaVtraceMinGRUFFI: scalar-delta V-trace with bootstrap (f64, bit-exact)."""
    r, v, t, i, b = (_f64(x) for x in (rewards, values, terms, imps, bootv))
    out = np.empty(B * T)
    _check(lib().pl_vtrace_mingru(_p(r), _p(v), _p(t), _p(i), _p(b), B, T, gamma, lam, rho_clip, c_clip, _p(out)),
           "pl_vtrace_mingru")
    return out


# ------------------------------------------------------------------------------------------------
# Host bookkeeping -- Puffer/Float/FFI.lean
def shuffle_perm(NT, epochs, rng):
    """shufflePermFFI: epochs x Fisher-Yates, f64-encoded."""
    out = np.empty(NT * epochs)
    _check(lib().pl_shuffle_perm(NT, epochs, C.c_uint64(rng & (2**64 - 1)), _p(out)), "pl_shuffle_perm")
    return out


def gae_soa(vals, rews, terms, N, T, gamma, lam):
    """gaeSoaFFI: truncated GAE + returns, [adv(NT); ret(NT)]."""
    v, r, t = (_f64(x) for x in (vals, rews, terms))
    out = np.empty(2 * N * T)
    _check(lib().pl_gae_soa(_p(v), _p(r), _p(t), N, T, gamma, lam, _p(out)), "pl_gae_soa")
    return out


# ------------------------------------------------------------------------------------------------
# Muon -- Puffer/Float/CUDA.lean:37-39
def cuda_muon_stepmat(W, grad, mom, rows, cols, lr, wd, mu, eps):
    """cudaMuonStepMatFFI: returns [newW; newMom] (f64 Newton-Schulz, bit-exact)."""
    w, g, m = (_f64(x) for x in (W, grad, mom))
    out = np.empty(2 * rows * cols)
    _check(lib().pl_muon_stepmat(_p(w), _p(g), _p(m), rows, cols, lr, wd, mu, eps, _p(out)), "pl_muon_stepmat")
    return out


# ------------------------------------------------------------------------------------------------
# MLP PPO -- Puffer/Float/CUDA.lean:45-75, 225-244
def cuda_mlp_ppo_grad(params, obsB, acts, advs, rets, oldlps, N, H, D, A, vf_coef, ent_coef, clip_eps, bf16):
    """cudaMlpPpoGradFFI: summed PPO-objective gradient g[P]."""
    P = H * D + H + (A + 1) * H + A + 1
    arrs = [_f64(x) for x in (params, obsB, acts, advs, rets, oldlps)]
    out = np.empty(P)
    _check(lib().pl_mlp_ppo_grad(*[_p(a) for a in arrs], N, H, D, A, vf_coef, ent_coef, clip_eps, bf16, _p(out)),
           "pl_mlp_ppo_grad")
    return out


def cuda_adv_normalize(adv, n):
    """cudaAdvNormalizeFFI."""
    a = _f64(adv)
    out = np.empty(n)
    _check(lib().pl_adv_normalize(_p(a), n, _p(out)), "pl_adv_normalize")
    return out


def cuda_train_step(pm, obsB, acts, adv_raw, rets, oldlps, N, H, D, A, lr, wd, mu, eps, vf_coef, ent_coef, clip_eps,
                    bf16):
    """cudaTrainStepFFI: returns the new [params; mom]."""
    arrs = [_f64(x) for x in (pm, obsB, acts, adv_raw, rets, oldlps)]
    out = np.empty(arrs[0].size)
    _check(lib().pl_train_step(*[_p(a) for a in arrs], N, H, D, A, lr, wd, mu, eps, vf_coef, ent_coef, clip_eps, bf16,
                               _p(out)), "pl_train_step")
    return out


def cuda_train_update(pm, obs, acts, adv, ret, olp, perm, NT, D, H, A, epochs, num_mb, lr, wd, mu, eps, vf_coef,
                      ent_coef, clip_eps, bf16):
    """cudaTrainUpdateFFI: whole update, returns the new [params; mom]."""
    arrs = [_f64(x) for x in (pm, obs, acts, adv, ret, olp, perm)]
    out = np.empty(arrs[0].size)
    _check(lib().pl_train_update(*[_p(a) for a in arrs], NT, D, H, A, epochs, num_mb, lr, wd, mu, eps, vf_coef,
                                 ent_coef, clip_eps, bf16, _p(out)), "pl_train_update")
    return out


def policy_load(pm, P):
    """policyLoadFFI: uploads [params; mom], returns the handle."""
    a = _f64(pm)
    h = _sz(0)
    _check(lib().pl_policy_load(_p(a), P, C.byref(h)), "pl_policy_load")
    return h.value


def policy_download(handle, P):
    out = np.empty(2 * P)
    _check(lib().pl_policy_download(handle, P, _p(out)), "pl_policy_download")
    return out


def policy_free(handle):
    _check(lib().pl_policy_free(handle), "pl_policy_free")


def cuda_train_update_resident(handle, obs, acts, adv, ret, olp, old_val, perm, NT, D, H, A, epochs, num_mb, lr, wd,
                               mu, eps, vf_coef, ent_coef, clip_eps, vf_clip, max_grad_norm, bf16):
    """cudaTrainUpdateResidentFFI: in-place update of the resident policy; returns [params[0]]."""
    arrs = [_f64(x) for x in (obs, acts, adv, ret, olp)]
    ov = _f64(old_val) if old_val is not None else np.empty(0)
    pr = _f64(perm)
    out = np.empty(1)
    _check(lib().pl_train_update_resident(handle, *[_p(a) for a in arrs], _p(ov), ov.size, _p(pr), NT, D, H, A,
                                          epochs, num_mb, lr, wd, mu, eps, vf_coef, ent_coef, clip_eps, vf_clip,
                                          max_grad_norm, bf16, _p(out)), "pl_train_update_resident")
    return out
