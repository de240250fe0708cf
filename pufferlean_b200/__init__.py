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


class MgNet(C.Structure):
    """pl_mg_net: the MinGRU network (K = 3 the reference layer, K = 2 gate + candidate only)."""
    _fields_ = [("D", _sz), ("H", _sz), ("L", _sz), ("A", _sz), ("K", _sz), ("enc_act", C.c_int)]


class MgHyper(C.Structure):
    """pl_mg_hyper: the MinGRU update's hyperparameters."""
    _fields_ = [(x, _d) for x in ("gamma", "lam", "rhoClip", "cClip", "prioAlpha", "annealBeta", "wd", "mu", "eps",
                                  "vfCoef", "entCoef", "clipEps", "vfClip", "maxGradNorm")] + [
        ("ns_coeffs", _dp), ("ns_iters", _sz), ("bf16", C.c_uint8)]


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
        "pl_mg_param_count": ([C.POINTER(MgNet)], _sz),
        "pl_mingru_ppo_grad": ([_dp] * 3 + [_sz, _sz, C.POINTER(MgNet)] + [_d] * 4 + [C.c_uint8, _dp], C.c_int),
        "pl_prio_sample": ([_dp, _sz, _sz, _d, _d, C.c_uint64, _dp, _dp], C.c_int),
        "pl_gather_seq_minibatch": ([_dp] * 7 + [_sz, _sz, _dp], C.c_int),
        "pl_slice": ([_dp, _sz, _sz, _sz, _dp], C.c_int),
        "pl_gather_minibatch": ([_dp] * 5 + [_sz, _dp, _sz, _sz] + [_dp] * 5, C.c_int),
        "pl_mg_create": ([_sz, _sz, C.POINTER(_vp)], C.c_int),
        "pl_mg_destroy": ([_vp], C.c_int),
        "pl_mg_set_columns": ([_vp] + [_dp] * 6, C.c_int),
        "pl_mg_set_columns_dev": ([_vp] * 8, C.c_int),
        "pl_mg_set_obs": ([_vp, _dp, _sz], C.c_int),
        "pl_mg_set_obs_dev": ([_vp, _vp, _sz], C.c_int),
        "pl_mg_vtrace": ([_vp] + [_d] * 4 + [_dp, _vp], C.c_int),
        "pl_mg_vtrace_prio": ([_vp] + [_d] * 4 + [_sz, _d, _d, C.c_uint64, _vp], C.c_int),
        "pl_mg_grad": ([_vp, C.POINTER(MgNet), _sz, _dp, _dp, _dp, _sz] + [_d] * 4 + [C.c_uint8, _vp], C.c_int),
        "pl_mg_grad_download": ([_vp, _dp, _dp, _dp], C.c_int),
        "pl_mg_muon": ([_vp, C.POINTER(MgNet), _sz, _dp] + [_d] * 6 + [_dp, _sz, C.c_uint8, _vp], C.c_int),
        "pl_mg_read_state": ([_vp, _dp, _dp, _dp], C.c_int),
        "pl_mg_update": ([_vp, C.POINTER(MgNet), _sz, C.POINTER(MgHyper), _sz, _sz, C.POINTER(C.c_uint64), _d, _vp],
                         C.c_int),
        "pl_mg_last_launches": ([_vp], C.c_uint64),
        "pl_mg_set_comm": ([_vp, _vp, C.c_int, C.c_int], C.c_int),
        "pl_mg_set_heads": ([_vp, _sz, _dp], C.c_int),
        "pl_mg_stamp_step": ([_vp, _sz, _sz, _sz, _vp, _vp, _vp, _vp, _sz, _vp], C.c_int),
        "pl_mg_stamp_finish": ([_vp] * 5, C.c_int),
        "pl_mg_take_stamped": ([_vp, C.POINTER(C.c_int)], C.c_int),
        "pl_stamp_rows_f64": ([_vp, _sz, _sz, _sz, _sz, _sz, _sz, _vp, _vp], C.c_int),
        "pl_stamp_rows_f32": ([_vp, _sz, _sz, _sz, _sz, _sz, _sz, _vp, _vp], C.c_int),
        "pl_stamp_plane_f64": ([_vp, _sz, _sz, _vp, _vp], C.c_int),
        "pl_mingru_ppo_grad_md": ([_dp] * 3 + [_sz, _sz, C.POINTER(MgNet), _sz, _dp] + [_d] * 4 + [C.c_uint8, _dp],
                                  C.c_int),
        "pl_train_update_wide_resident": ([_sz] + [_dp] * 6 + [_sz, _dp, _dp] + [_sz] * 5 + [C.c_uint32, _sz, _sz]
                                          + [_d] * 9 + [C.c_uint8, _dp], C.c_int),
        "pl_mlp_ppo_grad_wide": ([_dp] * 7 + [_sz] * 5 + [C.c_uint32, _dp] + [_d] * 4 + [C.c_uint8, _dp], C.c_int),
        "pl_muon_step_mlp_resident": ([_sz, _dp] + [_sz] * 3 + [_d] * 5 + [_dp], C.c_int),
        "pl_lstm_ppo_grad_batch": ([_dp] * 9 + [_sz] * 5 + [_d] * 3 + [C.c_int, _dp, _dp, _dp], C.c_int),
        "pl_lstm_reuse_inputs": ([C.c_int], C.c_int),
        "pl_lstm_gae_boot_norm": ([_dp] * 4 + [_sz, _sz, _d, _d, _dp], C.c_int),
        "pl_ckpt_write": ([C.c_char_p, _dp, _sz], C.c_int),
        "pl_ckpt_read": ([C.c_char_p, _dp, _sz, C.POINTER(_sz)], C.c_int),
        "pl_policy_save": ([_sz, _sz, C.c_char_p], C.c_int),
        "pl_policy_restore": ([C.c_char_p, C.POINTER(_sz), C.POINTER(_sz)], C.c_int),
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


def slice(arr, off, length):  # noqa: A001 - the reference's name (sliceFFI)
    """sliceFFI: arr[off : off + length] (the range must lie inside arr)."""
    a = _f64(arr)
    out = np.empty(length)
    _check(lib().pl_slice(_p(a), a.size, off, length, _p(out)), "pl_slice")
    return out


def gather_minibatch(obs_col, actions, advs, rets, olps, idxs, Nmb, D):
    """gatherMinibatchFFI: rows idxs[0:Nmb] (f64-encoded) of the SoA columns ->
    (mbObs[Nmb*D], mbAct, mbAdv, mbRet, mbOlp); NT is the length of the action column."""
    o, a, ad, r, ol, ix = (_f64(x) for x in (obs_col, actions, advs, rets, olps, idxs))
    NT = min(a.size, ad.size, r.size, ol.size, o.size // D if D else a.size)
    if ix.size < Nmb:
        raise PufferError(f"gather_minibatch: {ix.size} indices for {Nmb} rows")
    outs = [np.empty(Nmb * D)] + [np.empty(Nmb) for _ in range(4)]
    _check(lib().pl_gather_minibatch(_p(o), _p(a), _p(ad), _p(r), _p(ol), NT, _p(ix), Nmb, D, *[_p(x) for x in outs]),
           "pl_gather_minibatch")
    return tuple(outs)


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


# ------------------------------------------------------------------------------------ wide action heads
def _heads(head_sizes, W):
    return _f64(head_sizes) if head_sizes is not None else np.zeros(max(int(W), 1))


def cuda_train_update_wide_resident(handle, obs, acts, adv, ret, olp, old_val, perm, head_sizes, NT, D, H, O, W, mode,
                                    epochs, num_mb, lr, wd, mu, eps, vf_coef, ent_coef, clip_eps, vf_clip,
                                    max_grad_norm, bf16):
    """cudaTrainUpdateWideResidentFFI: the resident update with W multi-discrete heads (mode 1, head_sizes
    summing to O-1) or W Gaussian dims (mode 2, O = 2W+1); acts is NT x W. Returns [params[0]]."""
    arrs = [_f64(x) for x in (obs, acts, adv, ret, olp)]
    ov = _f64(old_val) if old_val is not None else np.empty(0)
    pr, hs = _f64(perm), _heads(head_sizes, W)
    out = np.empty(1)
    _check(lib().pl_train_update_wide_resident(handle, *[_p(a) for a in arrs], _p(ov), ov.size, _p(pr), _p(hs), NT,
                                               D, H, O, W, mode, epochs, num_mb, lr, wd, mu, eps, vf_coef, ent_coef,
                                               clip_eps, vf_clip, max_grad_norm, bf16, _p(out)),
           "pl_train_update_wide_resident")
    return out


def cuda_mlp_ppo_grad_wide(params, obs, acts, advs, rets, oldlps, old_val, N, H, D, O, W, mode, head_sizes, vf_coef,
                           ent_coef, clip_eps, vf_clip, bf16):
    """Summed wide-head objective gradient over N rows (P values, ascent convention)."""
    arrs = [_f64(x) for x in (params, obs, acts, advs, rets, oldlps)]
    ov = _f64(old_val) if old_val is not None else None
    out = np.empty(H * D + H + O * H + O)
    _check(lib().pl_mlp_ppo_grad_wide(*[_p(a) for a in arrs], _p(ov) if ov is not None else None, N, H, D, O, W, mode,
                                      _p(_heads(head_sizes, W)), vf_coef, ent_coef, clip_eps, vf_clip, bf16, _p(out)),
           "pl_mlp_ppo_grad_wide")
    return out


def cuda_muon_step_mlp_resident(handle, g_raw, H, D, O, gscale, lr, wd, mu, eps):
    """cudaMuonStepMlpResidentFFI: in-place f64 Muon of the resident [W1|b1|W2|b2] from a raw summed gradient;
    returns the new params."""
    out = np.empty(H * D + H + O * H + O)
    _check(lib().pl_muon_step_mlp_resident(handle, _p(_f64(g_raw)), H, D, O, gscale, lr, wd, mu, eps, _p(out)),
           "pl_muon_step_mlp_resident")
    return out


# --------------------------------------------------------------------------------------------- LSTM
def lstm_param_count(D, H, A):
    return 4 * H * D + 4 * H * H + 4 * H + (A + 1) * H + (A + 1)


def cuda_lstm_ppo_grad_batch(params, obsB, acts, advs, rets, oldlps, terms, h0s, c0s, B, T, H, D, A, vf_coef,
                             ent_coef, clip_eps, tier=1, with_outputs=False):
    """lstmPPOGradBatchBlas*FFI: the summed BPTT gradient (P values); tier 0 f64, 1 f32, 2 the bf16 tier.
    with_outputs: also return the T*B new log-probs and values."""
    arrs = [_f64(x) for x in (params, obsB, acts, advs, rets, oldlps, terms, h0s, c0s)]
    g = np.empty(lstm_param_count(D, H, A))
    nl, nv = (np.empty(T * B), np.empty(T * B)) if with_outputs else (None, None)
    _check(lib().pl_lstm_ppo_grad_batch(*[_p(a) for a in arrs], B, T, H, D, A, vf_coef, ent_coef, clip_eps, tier,
                                        _p(g), _p(nl) if nl is not None else None,
                                        _p(nv) if nv is not None else None), "pl_lstm_ppo_grad_batch")
    return (g, nl, nv) if with_outputs else g


def lstm_gae_boot_norm(vals, rews, terms, boot, N, T, gamma, lam):
    out = np.empty(2 * N * T)
    arrs = [_f64(x) for x in (vals, rews, terms, boot)]
    _check(lib().pl_lstm_gae_boot_norm(*[_p(a) for a in arrs], N, T, gamma, lam, _p(out)), "pl_lstm_gae_boot_norm")
    return out


# ------------------------------------------------------------------------------------------- MinGRU
def mg_net(D, H, L, A, K=3, enc_act=0):
    return MgNet(D, H, L, A, K, enc_act)


def mg_param_count(D, H, L, A, K=3, enc_act=0):
    return int(lib().pl_mg_param_count(C.byref(mg_net(D, H, L, A, K, enc_act))))


def cuda_mingru_ppo_grad(params, obs, scal, B, T, H, D, L, A, vf_coef, ent_coef, clip_eps, vf_clip, bf16=0, K=3,
                         enc_act=0, hs=None):
    """Host mode of lean_cuda_mingru_ppo_grad: [grad(P); new_logp(T*B); new_value(T*B)] (f64). hs: multi-discrete
    head sizes (sum A); scal's act block then holds len(hs) actions per row."""
    net = mg_net(D, H, L, A, K, enc_act)
    P = int(lib().pl_mg_param_count(C.byref(net)))
    out = np.zeros(P + 2 * T * B)
    params, obs, scal = _f64(params), _f64(obs), _f64(scal)
    if hs is None:
        _check(lib().pl_mingru_ppo_grad(_p(params), _p(obs), _p(scal), B, T, C.byref(net), vf_coef, ent_coef,
                                        clip_eps, vf_clip, bf16, _p(out)), "pl_mingru_ppo_grad")
    else:
        h = _f64(hs)
        _check(lib().pl_mingru_ppo_grad_md(_p(params), _p(obs), _p(scal), B, T, C.byref(net), h.size, _p(h), vf_coef,
                                           ent_coef, clip_eps, vf_clip, bf16, _p(out)), "pl_mingru_ppo_grad_md")
    return out


def prio_sample(adv_l1, N, T, mb_segs, prio_alpha, anneal_beta, rng):
    """lean_ffi_prio_sample: (segment indices as f64, importance weights)."""
    seg, mp = np.zeros(mb_segs), np.zeros(mb_segs)
    adv_l1 = _f64(adv_l1)
    _check(lib().pl_prio_sample(_p(adv_l1), N, mb_segs, prio_alpha, anneal_beta, rng & 0xFFFFFFFFFFFFFFFF, _p(seg),
                                _p(mp)), "pl_prio_sample")
    return seg, mp


def gather_seq_minibatch(act_col, logp_col, term_col, adv_flat, value_buf, seg_idx, mb_prio, T, Bmb):
    """lean_ffi_gather_seq_minibatch's packed [act|adv|ret|old|term|ov] (6*T*Bmb)."""
    out = np.zeros(6 * T * Bmb)
    arrs = [_f64(a) for a in (act_col, logp_col, term_col, adv_flat, value_buf, seg_idx, mb_prio)]
    _check(lib().pl_gather_seq_minibatch(*[_p(a) for a in arrs], T, Bmb, _p(out)), "pl_gather_seq_minibatch")
    return out


class MgSession:
    """The resident MinGRU state (pl_mg_*): columns, obs trajectory, sample, workspace, gradient."""

    def __init__(self, N, T):
        self.N, self.T = N, T
        self.h = _vp()
        _check(lib().pl_mg_create(N, T, C.byref(self.h)), "pl_mg_create")

    def close(self):
        if self.h:
            lib().pl_mg_destroy(self.h)
            self.h = _vp()

    def set_heads(self, W, hs=None):
        """W multi-discrete heads (act columns W wide per row); call before set_columns."""
        h = _f64(hs) if hs is not None else None
        _check(lib().pl_mg_set_heads(self.h, W, _p(h) if h is not None else None), "pl_mg_set_heads")

    def stamp_step(self, step, e0, ne, act, logp, val, obs=None, D=0, stream=None):
        """Rollout step `step` of envs [e0, e0 + ne) from device arrays (addresses): act [ne x W], logp, val
        [ne] f64; obs [ne x D] f32 or None."""
        _check(lib().pl_mg_stamp_step(self.h, step, e0, ne, act, logp, val, obs, D, stream), "pl_mg_stamp_step")

    def stamp_finish(self, rew, term, boot, stream=None):
        """The update's reward / terminal planes, step-major [T x N] device f64, and boot [N]."""
        _check(lib().pl_mg_stamp_finish(self.h, rew, term, boot, stream), "pl_mg_stamp_finish")

    def take_stamped(self):
        r = C.c_int(0)
        _check(lib().pl_mg_take_stamped(self.h, C.byref(r)), "pl_mg_take_stamped")
        return bool(r.value)

    def set_columns(self, rew, term, act, logp, val, boot):
        arrs = [_f64(a) for a in (rew, term, act, logp, val, boot)]
        _check(lib().pl_mg_set_columns(self.h, *[_p(a) for a in arrs]), "pl_mg_set_columns")

    def set_comm(self, comm, rank, world):
        _check(lib().pl_mg_set_comm(self.h, comm, rank, world), "pl_mg_set_comm")

    def set_obs(self, obs, D):
        obs = _f64(obs)
        _check(lib().pl_mg_set_obs(self.h, _p(obs), D), "pl_mg_set_obs")

    def vtrace(self, gamma, lam, rho, c):
        l1 = np.zeros(self.N)
        _check(lib().pl_mg_vtrace(self.h, gamma, lam, rho, c, _p(l1), None), "pl_mg_vtrace")
        return l1

    def vtrace_prio(self, gamma, lam, rho, c, mb_segs, alpha, beta, rng):
        _check(lib().pl_mg_vtrace_prio(self.h, gamma, lam, rho, c, mb_segs, alpha, beta, rng & 0xFFFFFFFFFFFFFFFF,
                                       None), "pl_mg_vtrace_prio")

    def grad(self, net, handle=0, params=None, seg=None, mbp=None, Bmb=0, vf=0.5, ent=0.01, clip=0.2, vfclip=0.2,
             bf16=0):
        pr = _f64(params) if params is not None else None
        sg = _f64(seg) if seg is not None else None
        mp = _f64(mbp) if mbp is not None else None
        _check(lib().pl_mg_grad(self.h, C.byref(net), handle, _p(pr) if pr is not None else None,
                                _p(sg) if sg is not None else None, _p(mp) if mp is not None else None, Bmb, vf, ent,
                                clip, vfclip, bf16, None), "pl_mg_grad")

    def grad_download(self, P, R):
        g, nl, nv = np.zeros(P), np.zeros(R), np.zeros(R)
        _check(lib().pl_mg_grad_download(self.h, _p(g), _p(nl), _p(nv)), "pl_mg_grad_download")
        return g, nl, nv

    def muon(self, net, handle, lr, wd, mu, eps, max_grad_norm, gscale, gclip=None, coeffs=None, bf16=0):
        gc = _f64(gclip) if gclip is not None else None
        co = _f64(coeffs) if coeffs is not None else None
        _check(lib().pl_mg_muon(self.h, C.byref(net), handle, _p(gc) if gc is not None else None, lr, wd, mu, eps,
                                max_grad_norm, gscale, _p(co) if co is not None else None,
                                (co.size // 3) if co is not None else 0, bf16, None), "pl_mg_muon")

    def state(self):
        n = self.N * self.T
        v, r, a = np.zeros(n), np.zeros(n), np.zeros(n)
        _check(lib().pl_mg_read_state(self.h, _p(v), _p(r), _p(a)), "pl_mg_read_state")
        return v, r, a

    def update(self, net, handle, hyper, num_mb, mb_segs, rng, lr):
        r = C.c_uint64(rng & 0xFFFFFFFFFFFFFFFF)
        _check(lib().pl_mg_update(self.h, C.byref(net), handle, C.byref(hyper), num_mb, mb_segs, C.byref(r), lr, None),
               "pl_mg_update")
        return r.value

    def last_launches(self):
        return int(lib().pl_mg_last_launches(self.h))


# ------------------------------------------------------------------------------------------- checkpoints
def ckpt_write(path, w):
    """The reference's `<step>.bin` layout (Puffer/RL/FFITrain.lean:55-62): u64 P, then P f64, little-endian."""
    w = _f64(w)
    _check(lib().pl_ckpt_write(os.fsencode(path), _p(w), w.size), "pl_ckpt_write")


def ckpt_read(path):
    n = _sz(0)
    _check(lib().pl_ckpt_read(os.fsencode(path), None, 0, C.byref(n)), "pl_ckpt_read")
    w = np.zeros(n.value)
    _check(lib().pl_ckpt_read(os.fsencode(path), _p(w), w.size, C.byref(n)), "pl_ckpt_read")
    return w


def policy_save(handle, P, path):
    _check(lib().pl_policy_save(handle, P, os.fsencode(path)), "pl_policy_save")


def policy_restore(path):
    """(handle, P): a policy handle with the file's weights and zero momentum."""
    P, h = _sz(0), _sz(0)
    _check(lib().pl_policy_restore(os.fsencode(path), C.byref(P), C.byref(h)), "pl_policy_restore")
    return h.value, P.value
