/* Lean-runtime adapter: the reference's `@[extern]` symbols for the PPO+Muon update path, each a
 * thin unboxing shim over the plain C ABI of libpufferlean_b200.so.
 *
 * The Lean declarations (Puffer/Float/CUDA.lean, Puffer/Float/FFI.lean) stay as they are; linking
 * this file (compiled against Lean's own lean.h) instead of ffi/puffercuda.cu's definitions routes
 * the trainer through the B200 kernels. Conventions kept from the reference (Puffer/Float/CUDA.lean
 * and ffi/puffercuda.cu): FloatArray arguments are owned (released with lean_dec), pure functions
 * return a fresh FloatArray, IO functions take the world token and return an IO result.
 *
 * Failure behaviour (there is no CPU fallback): IO functions return an IO error carrying the
 * library's message; pure functions print the message to stderr and return a NaN-filled array of
 * the expected size, so a failure can never masquerade as a zero gradient or a zero advantage.
 */
#include <lean/lean.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pufferlean_b200.h"

static double* fa(b_lean_obj_arg a) { return lean_float_array_cptr(a); }
static size_t fan(b_lean_obj_arg a) { return lean_sarray_size(a); }

static lean_obj_res new_fa(size_t n) { return lean_alloc_sarray(sizeof(double), n, n); }

static lean_obj_res pure_fail(lean_obj_res out, const char* what) {
  fprintf(stderr, "pufferlean_b200: %s failed: %s\n", what, pl_last_error());
  double* p = fa(out);
  for (size_t i = 0; i < fan(out); i++) p[i] = NAN;
  return out;
}
static lean_obj_res io_fail(const char* what) {
  char buf[1200];
  snprintf(buf, sizeof buf, "pufferlean_b200: %s failed: %s", what, pl_last_error());
  return lean_io_result_mk_error(lean_mk_io_user_error(lean_mk_string(buf)));
}

/* ---------------------------------------------------------------- V-trace (CUDA.lean:20-31) */
LEAN_EXPORT lean_obj_res lean_cuda_vtrace(lean_obj_arg rew, lean_obj_arg val, lean_obj_arg term, lean_obj_arg imp,
                                          size_t B, size_t T, double gamma, double lam, double rhoClip,
                                          double cClip) {
  lean_obj_res out = new_fa(B * T);
  int rc = pl_vtrace(fa(rew), fa(val), fa(term), fa(imp), B, T, gamma, lam, rhoClip, cClip, fa(out));
  lean_dec(rew);
  lean_dec(val);
  lean_dec(term);
  lean_dec(imp);
  return rc ? pure_fail(out, "lean_cuda_vtrace") : out;
}

LEAN_EXPORT lean_obj_res lean_cuda_vtrace_mingru(lean_obj_arg rew, lean_obj_arg val, lean_obj_arg term,
                                                 lean_obj_arg imp, lean_obj_arg bv, size_t B, size_t T, double gamma,
                                                 double lam, double rhoClip, double cClip) {
  lean_obj_res out = new_fa(B * T);
  int rc = pl_vtrace_mingru(fa(rew), fa(val), fa(term), fa(imp), fa(bv), B, T, gamma, lam, rhoClip, cClip, fa(out));
  lean_dec(rew);
  lean_dec(val);
  lean_dec(term);
  lean_dec(imp);
  lean_dec(bv);
  return rc ? pure_fail(out, "lean_cuda_vtrace_mingru") : out;
}

/* ---------------------------------------------------------------- Muon (CUDA.lean:37-39) */
LEAN_EXPORT lean_obj_res lean_cuda_muon_stepmat(lean_obj_arg W, lean_obj_arg G, lean_obj_arg M, size_t rows,
                                                size_t cols, double lr, double wd, double mu, double eps) {
  lean_obj_res out = new_fa(2 * rows * cols);
  int rc = pl_muon_stepmat(fa(W), fa(G), fa(M), rows, cols, lr, wd, mu, eps, fa(out));
  lean_dec(W);
  lean_dec(G);
  lean_dec(M);
  return rc ? pure_fail(out, "lean_cuda_muon_stepmat") : out;
}

/* ---------------------------------------------------------------- MLP PPO (CUDA.lean:45-75) */
LEAN_EXPORT lean_obj_res lean_cuda_mlp_ppo_grad(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts,
                                                lean_obj_arg advs, lean_obj_arg rets, lean_obj_arg olps, size_t N,
                                                size_t H, size_t D, size_t A, double vf, double ent, double clip,
                                                uint8_t bf16) {
  lean_obj_res out = new_fa(pl_mlp_param_count(D, H, A, 1));
  int rc = pl_mlp_ppo_grad(fa(pa), fa(obs), fa(acts), fa(advs), fa(rets), fa(olps), N, H, D, A, vf, ent, clip, bf16,
                           fa(out));
  lean_dec(pa);
  lean_dec(obs);
  lean_dec(acts);
  lean_dec(advs);
  lean_dec(rets);
  lean_dec(olps);
  return rc ? pure_fail(out, "lean_cuda_mlp_ppo_grad") : out;
}

/* Multi-discrete and Gaussian twins of lean_cuda_mlp_ppo_grad (CUDA.lean:93-106): the summed gradient
 * g[P] of the one-hidden-layer network with O = sum(headSizes) + 1 or O = 2d + 1 outputs. */
LEAN_EXPORT lean_obj_res lean_cuda_mlp_ppo_grad_md(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts,
                                                   lean_obj_arg advs, lean_obj_arg rets, lean_obj_arg olps,
                                                   lean_obj_arg hs, size_t N, size_t H, size_t D, size_t K, double vf,
                                                   double ent, double clip, uint8_t bf16) {
  size_t A = 0;
  int bad = fan(hs) < K;
  for (size_t i = 0; !bad && i < K; i++) {
    const double h = fa(hs)[i];
    if (!(h >= 1.0)) bad = 1;
    else A += (size_t)h;
  }
  const size_t O = A + 1;
  lean_obj_res out = new_fa(H * D + H + O * H + O);
  int rc = bad ? -1
               : pl_mlp_ppo_grad_wide(fa(pa), fa(obs), fa(acts), fa(advs), fa(rets), fa(olps), NULL, N, H, D, O, K, 1,
                                      fa(hs), vf, ent, clip, 0.0, bf16, fa(out));
  lean_dec(pa);
  lean_dec(obs);
  lean_dec(acts);
  lean_dec(advs);
  lean_dec(rets);
  lean_dec(olps);
  lean_dec(hs);
  return rc ? pure_fail(out, "lean_cuda_mlp_ppo_grad_md") : out;
}

LEAN_EXPORT lean_obj_res lean_cuda_mlp_ppo_grad_cont(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts,
                                                     lean_obj_arg advs, lean_obj_arg rets, lean_obj_arg olps, size_t N,
                                                     size_t H, size_t D, size_t d, double vf, double ent, double clip,
                                                     uint8_t bf16) {
  const size_t O = 2 * d + 1;
  lean_obj_res out = new_fa(H * D + H + O * H + O);
  int rc = pl_mlp_ppo_grad_wide(fa(pa), fa(obs), fa(acts), fa(advs), fa(rets), fa(olps), NULL, N, H, D, O, d, 2, NULL,
                                vf, ent, clip, 0.0, bf16, fa(out));
  lean_dec(pa);
  lean_dec(obs);
  lean_dec(acts);
  lean_dec(advs);
  lean_dec(rets);
  lean_dec(olps);
  return rc ? pure_fail(out, "lean_cuda_mlp_ppo_grad_cont") : out;
}

LEAN_EXPORT lean_obj_res lean_cuda_adv_normalize(lean_obj_arg adv, size_t n) {
  lean_obj_res out = new_fa(n);
  int rc = pl_adv_normalize(fa(adv), n, fa(out));
  lean_dec(adv);
  return rc ? pure_fail(out, "lean_cuda_adv_normalize") : out;
}

LEAN_EXPORT lean_obj_res lean_cuda_train_step(lean_obj_arg pm, lean_obj_arg obs, lean_obj_arg acts,
                                              lean_obj_arg advRaw, lean_obj_arg rets, lean_obj_arg olps, size_t N,
                                              size_t H, size_t D, size_t A, double lr, double wd, double mu,
                                              double eps, double vf, double ent, double clip, uint8_t bf16) {
  lean_obj_res out = new_fa(2 * pl_mlp_param_count(D, H, A, 1));
  int rc = pl_train_step(fa(pm), fa(obs), fa(acts), fa(advRaw), fa(rets), fa(olps), N, H, D, A, lr, wd, mu, eps, vf,
                         ent, clip, bf16, fa(out));
  lean_dec(pm);
  lean_dec(obs);
  lean_dec(acts);
  lean_dec(advRaw);
  lean_dec(rets);
  lean_dec(olps);
  return rc ? pure_fail(out, "lean_cuda_train_step") : out;
}

LEAN_EXPORT lean_obj_res lean_cuda_train_update(lean_obj_arg pm, lean_obj_arg obs, lean_obj_arg acts,
                                                lean_obj_arg adv, lean_obj_arg ret, lean_obj_arg olp,
                                                lean_obj_arg perm, size_t NT, size_t D, size_t H, size_t A,
                                                size_t epochs, size_t numMB, double lr, double wd, double mu,
                                                double eps, double vf, double ent, double clip, uint8_t bf16) {
  lean_obj_res out = new_fa(2 * pl_mlp_param_count(D, H, A, 1));
  int rc = pl_train_update(fa(pm), fa(obs), fa(acts), fa(adv), fa(ret), fa(olp), fa(perm), NT, D, H, A, epochs, numMB,
                           lr, wd, mu, eps, vf, ent, clip, bf16, fa(out));
  lean_dec(pm);
  lean_dec(obs);
  lean_dec(acts);
  lean_dec(adv);
  lean_dec(ret);
  lean_dec(olp);
  lean_dec(perm);
  return rc ? pure_fail(out, "lean_cuda_train_update") : out;
}

/* ---------------------------------------------------------------- resident policy (CUDA.lean:225-244) */
LEAN_EXPORT lean_obj_res lean_cuda_policy_load(lean_obj_arg pm, size_t P, lean_obj_arg w) {
  (void)w;
  size_t h = 0;
  int rc = pl_policy_load(fa(pm), P, &h);
  lean_dec(pm);
  if (rc) return io_fail("lean_cuda_policy_load");
  return lean_io_result_mk_ok(lean_box_usize(h));
}

LEAN_EXPORT lean_obj_res lean_cuda_policy_download(size_t handle, size_t P, lean_obj_arg w) {
  (void)w;
  lean_obj_res out = new_fa(2 * P);
  if (pl_policy_download(handle, P, fa(out))) {
    lean_dec(out);
    return io_fail("lean_cuda_policy_download");
  }
  return lean_io_result_mk_ok(out);
}

LEAN_EXPORT lean_obj_res lean_cuda_policy_free(size_t handle, lean_obj_arg w) {
  (void)w;
  if (pl_policy_free(handle)) return io_fail("lean_cuda_policy_free");
  return lean_io_result_mk_ok(lean_box(0));
}

LEAN_EXPORT lean_obj_res lean_cuda_train_update_resident(size_t handle, lean_obj_arg obs, lean_obj_arg acts,
                                                         lean_obj_arg adv, lean_obj_arg ret, lean_obj_arg olp,
                                                         lean_obj_arg ov, lean_obj_arg perm, size_t NT, size_t D,
                                                         size_t H, size_t A, size_t epochs, size_t numMB, double lr,
                                                         double wd, double mu, double eps, double vf, double ent,
                                                         double clip, double vfClip, double maxGradNorm, uint8_t bf16,
                                                         lean_obj_arg w) {
  (void)w;
  lean_obj_res out = new_fa(1);
  int rc = pl_train_update_resident(handle, fa(obs), fa(acts), fa(adv), fa(ret), fa(olp), fa(ov), fan(ov), fa(perm), NT,
                                    D, H, A, epochs, numMB, lr, wd, mu, eps, vf, ent, clip, vfClip, maxGradNorm, bf16,
                                    fa(out));
  lean_dec(obs);
  lean_dec(acts);
  lean_dec(adv);
  lean_dec(ret);
  lean_dec(olp);
  lean_dec(ov);
  lean_dec(perm);
  if (rc) {
    lean_dec(out);
    return io_fail("lean_cuda_train_update_resident");
  }
  return lean_io_result_mk_ok(out);
}

/* Deep variant (no reference symbol): L hidden layers of width H, act 0 = ReLU / 1 = GELU, the
 * reference's Newton-Schulz table. Same conventions as lean_cuda_train_update_resident. */
LEAN_EXPORT lean_obj_res lean_cuda_train_update_resident_deep(size_t handle, lean_obj_arg obs, lean_obj_arg acts,
                                                              lean_obj_arg adv, lean_obj_arg ret, lean_obj_arg olp,
                                                              lean_obj_arg ov, lean_obj_arg perm, size_t NT, size_t D,
                                                              size_t H, size_t A, size_t L, uint8_t act, size_t epochs,
                                                              size_t numMB, double lr, double wd, double mu,
                                                              double eps, double vf, double ent, double clip,
                                                              double vfClip, double maxGradNorm, uint8_t bf16,
                                                              lean_obj_arg w) {
  (void)w;
  pl_mlp_arch arch = {L, (int)act, NULL, 0};
  lean_obj_res out = new_fa(1);
  int rc = pl_train_update_resident_deep(handle, &arch, fa(obs), fa(acts), fa(adv), fa(ret), fa(olp), fa(ov), fan(ov),
                                         fa(perm), NT, D, H, A, epochs, numMB, lr, wd, mu, eps, vf, ent, clip, vfClip,
                                         maxGradNorm, bf16, fa(out));
  lean_dec(obs);
  lean_dec(acts);
  lean_dec(adv);
  lean_dec(ret);
  lean_dec(olp);
  lean_dec(ov);
  lean_dec(perm);
  if (rc) {
    lean_dec(out);
    return io_fail("lean_cuda_train_update_resident_deep");
  }
  return lean_io_result_mk_ok(out);
}

/* Wide action heads: W multi-discrete heads (mode 1, sizes in hs) or W Gaussian dims (mode 2) on the
 * resident one-hidden-layer policy; O = sum(hs)+1 or 2W+1, acts NT x W. Returns [params[0]] like
 * lean_cuda_train_update_resident. */
LEAN_EXPORT lean_obj_res lean_cuda_train_update_wide_resident(size_t handle, lean_obj_arg obs, lean_obj_arg acts,
                                                              lean_obj_arg adv, lean_obj_arg ret, lean_obj_arg olp,
                                                              lean_obj_arg ov, lean_obj_arg perm, lean_obj_arg hs,
                                                              size_t NT, size_t D, size_t H, size_t O, size_t W,
                                                              uint32_t mode, size_t epochs, size_t numMB, double lr,
                                                              double wd, double mu, double eps, double vf, double ent,
                                                              double clip, double vfClip, double maxGradNorm,
                                                              uint8_t bf16, lean_obj_arg w) {
  (void)w;
  lean_obj_res out = new_fa(1);
  const double* hsp = fan(hs) >= W ? fa(hs) : NULL;
  int rc = pl_train_update_wide_resident(handle, fa(obs), fa(acts), fa(adv), fa(ret), fa(olp), fa(ov), fan(ov),
                                         fa(perm), hsp, NT, D, H, O, W, mode, epochs, numMB, lr, wd, mu, eps, vf, ent,
                                         clip, vfClip, maxGradNorm, bf16, fa(out));
  lean_dec(obs);
  lean_dec(acts);
  lean_dec(adv);
  lean_dec(ret);
  lean_dec(olp);
  lean_dec(ov);
  lean_dec(perm);
  lean_dec(hs);
  if (rc) {
    lean_dec(out);
    return io_fail("lean_cuda_train_update_wide_resident");
  }
  return lean_io_result_mk_ok(out);
}

/* In-place f64 Muon of the resident [W1|b1|W2|b2] from the raw summed gradient gRaw (scaled by gscale);
 * returns the new params (P). */
LEAN_EXPORT lean_obj_res lean_cuda_muon_step_mlp_resident(size_t handle, lean_obj_arg gRaw, size_t H, size_t D,
                                                          size_t O, double gscale, double lr, double wd, double mu,
                                                          double eps, lean_obj_arg w) {
  (void)w;
  const size_t P = H * D + H + O * H + O;
  lean_obj_res out = new_fa(P);
  int rc = fan(gRaw) >= P ? pl_muon_step_mlp_resident(handle, fa(gRaw), H, D, O, gscale, lr, wd, mu, eps, fa(out))
                          : PL_ERR_INVALID;
  lean_dec(gRaw);
  if (rc) {
    lean_dec(out);
    return io_fail("lean_cuda_muon_step_mlp_resident");
  }
  return lean_io_result_mk_ok(out);
}

/* ---------------------------------------------------------------- LSTM (Puffer/Float/BLAS.lean:153-173) */
static lean_obj_res lstm_grad(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts, lean_obj_arg advs,
                              lean_obj_arg rets, lean_obj_arg olps, lean_obj_arg terms, lean_obj_arg h0s,
                              lean_obj_arg c0s, size_t B, size_t T, size_t H, size_t D, size_t A, double vf,
                              double ent, double clip, int tier, const char* what) {
  const size_t P = 4 * H * D + 4 * H * H + 4 * H + (A + 1) * H + (A + 1);
  lean_obj_res out = new_fa(P);
  int rc = (fan(pa) < P || fan(obs) < B * T * D || fan(acts) < B * T || fan(h0s) < B * H || fan(c0s) < B * H)
               ? PL_ERR_INVALID
               : pl_lstm_ppo_grad_batch(fa(pa), fa(obs), fa(acts), fa(advs), fa(rets), fa(olps), fa(terms), fa(h0s),
                                        fa(c0s), B, T, H, D, A, vf, ent, clip, tier, fa(out), NULL, NULL);
  lean_dec(pa);
  lean_dec(obs);
  lean_dec(acts);
  lean_dec(advs);
  lean_dec(rets);
  lean_dec(olps);
  lean_dec(terms);
  lean_dec(h0s);
  lean_dec(c0s);
  if (rc) return pure_fail(out, what);
  return out;
}
LEAN_EXPORT lean_obj_res lean_ffi_lstm_ppo_grad_batch_blas(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts,
                                                          lean_obj_arg advs, lean_obj_arg rets, lean_obj_arg olps,
                                                          lean_obj_arg terms, lean_obj_arg h0s, lean_obj_arg c0s,
                                                          size_t B, size_t T, size_t H, size_t D, size_t A,
                                                          double vf, double ent, double clip) {
  return lstm_grad(pa, obs, acts, advs, rets, olps, terms, h0s, c0s, B, T, H, D, A, vf, ent, clip, 0,
                   "lean_ffi_lstm_ppo_grad_batch_blas");
}
LEAN_EXPORT lean_obj_res lean_ffi_lstm_ppo_grad_batch_blas_f32(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts,
                                                              lean_obj_arg advs, lean_obj_arg rets, lean_obj_arg olps,
                                                              lean_obj_arg terms, lean_obj_arg h0s, lean_obj_arg c0s,
                                                              size_t B, size_t T, size_t H, size_t D, size_t A,
                                                              double vf, double ent, double clip) {
  return lstm_grad(pa, obs, acts, advs, rets, olps, terms, h0s, c0s, B, T, H, D, A, vf, ent, clip, 1,
                   "lean_ffi_lstm_ppo_grad_batch_blas_f32");
}
LEAN_EXPORT lean_obj_res lean_ffi_lstm_ppo_grad_batch_blas_bf16(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts,
                                                               lean_obj_arg advs, lean_obj_arg rets,
                                                               lean_obj_arg olps, lean_obj_arg terms,
                                                               lean_obj_arg h0s, lean_obj_arg c0s, size_t B, size_t T,
                                                               size_t H, size_t D, size_t A, double vf, double ent,
                                                               double clip) {
  return lstm_grad(pa, obs, acts, advs, rets, olps, terms, h0s, c0s, B, T, H, D, A, vf, ent, clip, 2,
                   "lean_ffi_lstm_ppo_grad_batch_blas_bf16");
}
LEAN_EXPORT lean_obj_res lean_cuda_lstm_reuse_inputs(uint8_t on, lean_obj_arg w) {
  (void)w;
  pl_lstm_reuse_inputs(on);
  return lean_io_result_mk_ok(lean_box(0));
}
LEAN_EXPORT lean_obj_res lean_ffi_lstm_gae_boot_norm(lean_obj_arg vals, lean_obj_arg rews, lean_obj_arg terms,
                                                    lean_obj_arg boot, size_t N, size_t T, double gamma,
                                                    double lam) {
  lean_obj_res out = new_fa(2 * N * T);
  int rc = pl_lstm_gae_boot_norm(fa(vals), fa(rews), fa(terms), fa(boot), N, T, gamma, lam, fa(out));
  lean_dec(vals);
  lean_dec(rews);
  lean_dec(terms);
  lean_dec(boot);
  if (rc) return pure_fail(out, "lean_ffi_lstm_gae_boot_norm");
  return out;
}

/* ---------------------------------------------------------------- dashboard losses (CUDA.lean:165-178) */
LEAN_EXPORT lean_obj_res lean_cuda_mg_loss_enable(uint8_t on, lean_obj_arg w) {
  (void)w;
  pl_loss_enable(on);
  return lean_io_result_mk_ok(lean_box(0));
}

LEAN_EXPORT lean_obj_res lean_cuda_mg_read_losses(lean_obj_arg w) {
  (void)w;
  lean_obj_res out = new_fa(7);
  pl_read_losses(fa(out));
  return lean_io_result_mk_ok(out);
}

/* ---------------------------------------------------------------- MinGRU path (CUDA.lean:126-160, 354-371) */
/* The reference keeps the MinGRU columns, sample and resident gradient in process globals; the adapter
 * keeps one pl_mg session for them (recreated when N or T change) and remembers the policy handle of the
 * last resident Muon step, whose weights a grad call with empty params then uses. The network is the
 * reference's (K = 3, linear encoder). PUFFER_MG_BF16=0 selects the fp32 tier; the default is the bf16
 * tensor-core tier (the reference's default is bf16 tensor-core compute as well). */
static pl_mg* g_mg = NULL;
static size_t g_mg_N = 0, g_mg_T = 0;
static size_t g_mg_handle = 0;

/* The session behind the MinGRU symbols (no reference counterpart): the rollout hands it the device obs
 * trajectory with pl_mg_set_obs_dev, as the reference's rollout fills g_dMGObsTraj. NULL before the first
 * lean_cuda_mg_prep. */
LEAN_EXPORT pl_mg* pl_lean_mg_session(void) { return g_mg; }

static uint8_t mg_bf16(void) {
  const char* e = getenv("PUFFER_MG_BF16");
  return (e && e[0] == '0') ? 0 : 1;
}
static int mg_session(size_t N, size_t T) {
  if (g_mg && g_mg_N == N && g_mg_T == T) return 0;
  if (g_mg) pl_mg_destroy(g_mg);
  g_mg = NULL;
  int rc = pl_mg_create(N, T, &g_mg);
  if (rc) return rc;
  g_mg_N = N;
  g_mg_T = T;
  return 0;
}

LEAN_EXPORT lean_obj_res lean_cuda_mg_prep(lean_obj_arg rew, lean_obj_arg term, lean_obj_arg act, lean_obj_arg logp,
                                           lean_obj_arg val, lean_obj_arg boot, size_t N, size_t T, size_t K,
                                           lean_obj_arg w) {
  (void)w;
  /* K > 1: the act column holds K multi-discrete actions per row; their head sizes arrive with the
   * gradient call (lean_cuda_mingru_ppo_grad's hs) */
  int rc = mg_session(N, T);
  if (!rc) rc = pl_mg_set_heads(g_mg, K < 1 ? 1 : K, NULL);
  if (!rc && fan(act) < N * T * (K < 1 ? 1 : K)) rc = PL_ERR_INVALID;
  if (!rc) rc = pl_mg_set_columns(g_mg, fa(rew), fa(term), fa(act), fa(logp), fa(val), fa(boot));
  lean_dec(rew);
  lean_dec(term);
  lean_dec(act);
  lean_dec(logp);
  lean_dec(val);
  lean_dec(boot);
  if (rc) return io_fail("lean_cuda_mg_prep");
  return lean_io_result_mk_ok(lean_box(0));
}

/* 1 when a rollout stamped this update's columns into the session (pl_mg_stamp_step / _finish on
 * pl_lean_mg_session()): the trainer then skips its prep call. Read once per update. */
LEAN_EXPORT lean_obj_res lean_cuda_mg_cols_ready(size_t N, size_t T, lean_obj_arg w) {
  (void)w;
  int r = 0;
  if (g_mg && g_mg_N == N && g_mg_T == T && pl_mg_take_stamped(g_mg, &r)) r = 0;
  return lean_io_result_mk_ok(lean_box(r ? 1 : 0));
}

/* Resident chaining (CUDA.lean:338, ffi/puffercuda.cu:255-289): true when the rollout that fed this
 * session stamped that it keeps its observations and recurrent state resident for (N, D, L*H)
 * (pl_mg_chain_stamp), so the trainer may pass empty obs0 / state0 to the next rollout. */
LEAN_EXPORT lean_obj_res lean_cuda_mg_chain_ready(size_t N, size_t D, size_t LH, lean_obj_arg w) {
  (void)w;
  int r = 0;
  if (g_mg && pl_mg_chain_ready(g_mg, N, D, LH, &r)) r = 0;
  return lean_io_result_mk_ok(lean_box(r ? 1 : 0));
}

LEAN_EXPORT lean_obj_res lean_cuda_mg_vtrace(size_t N, size_t T, double gamma, double lam, double rhoClip,
                                             double cClip, lean_obj_arg w) {
  (void)w;
  lean_obj_res out = new_fa(N);
  int rc = (g_mg && g_mg_N == N && g_mg_T == T) ? pl_mg_vtrace(g_mg, gamma, lam, rhoClip, cClip, fa(out), NULL) : -1;
  if (rc) {
    lean_dec(out);
    return io_fail("lean_cuda_mg_vtrace (no columns for this N x T: call lean_cuda_mg_prep first)");
  }
  return lean_io_result_mk_ok(out);
}

LEAN_EXPORT lean_obj_res lean_cuda_mg_vtrace_prio(size_t N, size_t T, double gamma, double lam, double rhoClip,
                                                  double cClip, size_t mbSegs, double prioAlpha, double annealBeta,
                                                  uint64_t rng, lean_obj_arg w) {
  (void)w;
  int rc = (g_mg && g_mg_N == N && g_mg_T == T)
               ? pl_mg_vtrace_prio(g_mg, gamma, lam, rhoClip, cClip, mbSegs, prioAlpha, annealBeta, rng, NULL)
               : -1;
  if (rc) return io_fail("lean_cuda_mg_vtrace_prio (no columns for this N x T: call lean_cuda_mg_prep first)");
  return lean_io_result_mk_ok(lean_box(1));
}

/* Host mode (obs and scal given): returns [grad(P); new_logp(T*B); new_value(T*B)]. Device-column mode
 * (obs and scal empty): gathers the sample (segIdx/mbPrio, or the resident one of
 * lean_cuda_mg_vtrace_prio when both are empty) from the session's columns and obs trajectory, leaves
 * the gradient resident and returns an empty array. */
LEAN_EXPORT lean_obj_res lean_cuda_mingru_ppo_grad(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg scal, size_t B,
                                                   size_t T, size_t H, size_t D, size_t L, size_t A, size_t K,
                                                   lean_obj_arg hs, double vfCoef, double entCoef, double clipEps,
                                                   double vfClip, lean_obj_arg segIdx, lean_obj_arg mbPrio,
                                                   lean_obj_arg w) {
  (void)w;
  pl_mg_net net = {D, H, L, A, 3, 0};
  const size_t P = pl_mg_param_count(&net);
  const int host = fan(obs) > 0 && fan(scal) > 0;
  lean_obj_res out = NULL;
  int rc = 0;
  const char* why = "lean_cuda_mingru_ppo_grad";
  const size_t W = K < 1 ? 1 : K; /* K > 1: multi-discrete heads of sizes hs (sum A) */
  if (W > 1 && fan(hs) < W) {
    rc = -1;
    why = "lean_cuda_mingru_ppo_grad (K > 1 heads without their K sizes in hs)";
  } else if (host) {
    out = new_fa(P + 2 * T * B);
    if (fan(pa) < P || fan(obs) < T * B * D || fan(scal) < (W + 5) * T * B) {
      rc = -1;
      why = "lean_cuda_mingru_ppo_grad (host mode: params, obs or scal shorter than P, T*B*D, (K+5)*T*B)";
    } else {
      rc = pl_mingru_ppo_grad_md(fa(pa), fa(obs), fa(scal), B, T, &net, W, W > 1 ? fa(hs) : NULL, vfCoef, entCoef,
                                 clipEps, vfClip, mg_bf16(), fa(out));
    }
  } else {
    const int resident_sample = fan(segIdx) == 0 && fan(mbPrio) == 0;
    const size_t handle = fan(pa) >= P ? 0 : g_mg_handle;
    if (!g_mg || g_mg_T != T) {
      rc = -1;
      why = "lean_cuda_mingru_ppo_grad (device-column mode without columns: call lean_cuda_mg_prep first)";
    } else if (fan(pa) < P && !handle) {
      rc = -1;
      why = "lean_cuda_mingru_ppo_grad (empty params and no resident Muon step has run yet)";
    } else {
      rc = pl_mg_set_heads(g_mg, W, W > 1 ? fa(hs) : NULL);
      if (!rc)
        rc = pl_mg_grad(g_mg, &net, handle, handle ? NULL : fa(pa), resident_sample ? NULL : fa(segIdx),
                      resident_sample ? NULL : fa(mbPrio), B, vfCoef, entCoef, clipEps, vfClip, mg_bf16(), NULL);
    }
    out = new_fa(0);
  }
  lean_dec(pa);
  lean_dec(obs);
  lean_dec(scal);
  lean_dec(hs);
  lean_dec(segIdx);
  lean_dec(mbPrio);
  if (rc) {
    lean_dec(out);
    return io_fail(why);
  }
  return lean_io_result_mk_ok(out);
}

/* gClip empty: clip and consume the resident gradient, return an empty array; gClip of P entries: an
 * already clipped host gradient, return the new weights (P). */
LEAN_EXPORT lean_obj_res lean_cuda_mingru_muon_resident(size_t handle, lean_obj_arg gClip, size_t H, size_t D, size_t L,
                                                        size_t A, double lr, double wd, double mu, double eps,
                                                        double maxGradNorm, double gscale, lean_obj_arg w) {
  (void)w;
  pl_mg_net net = {D, H, L, A, 3, 0};
  const size_t P = pl_mg_param_count(&net);
  const int host = fan(gClip) > 0;
  int rc;
  const char* why = "lean_cuda_mingru_muon_resident";
  if (!g_mg) {
    rc = -1;
    why = "lean_cuda_mingru_muon_resident (no MinGRU session: call lean_cuda_mg_prep first)";
  } else if (host && fan(gClip) < P) {
    rc = -1;
    why = "lean_cuda_mingru_muon_resident (host gClip shorter than the parameter vector)";
  } else {
    rc = pl_mg_muon(g_mg, &net, handle, host ? fa(gClip) : NULL, lr, wd, mu, eps, maxGradNorm, gscale, NULL, 0,
                    mg_bf16(), NULL);
  }
  lean_dec(gClip);
  if (rc) return io_fail(why);
  g_mg_handle = handle;
  lean_obj_res out = new_fa(host ? P : 0);
  if (host && pl_policy_download(handle, P, fa(out))) {
    lean_dec(out);
    return io_fail("lean_cuda_mingru_muon_resident (weights download)");
  }
  return lean_io_result_mk_ok(out);
}

/* ---------------------------------------------------------------- MinGRU host bookkeeping (FFI.lean:113-125) */
LEAN_EXPORT lean_obj_res lean_ffi_prio_sample(lean_obj_arg advL1, size_t N, size_t T, size_t mbSegs, double prioAlpha,
                                              double annealBeta, uint64_t rng) {
  (void)T;
  lean_obj_res idx = new_fa(mbSegs), mp = new_fa(mbSegs);
  int rc = fan(advL1) < N ? -1 : pl_prio_sample(fa(advL1), N, mbSegs, prioAlpha, annealBeta, rng, fa(idx), fa(mp));
  lean_dec(advL1);
  if (rc) {
    pure_fail(idx, "lean_ffi_prio_sample");
    pure_fail(mp, "lean_ffi_prio_sample");
  }
  lean_obj_res pr = lean_alloc_ctor(0, 2, 0);
  lean_ctor_set(pr, 0, idx);
  lean_ctor_set(pr, 1, mp);
  return pr;
}

LEAN_EXPORT lean_obj_res lean_ffi_gather_seq_minibatch(lean_obj_arg obsCol, lean_obj_arg actCol, lean_obj_arg logpCol,
                                                       lean_obj_arg termCol, lean_obj_arg advFlat,
                                                       lean_obj_arg valueBuf, lean_obj_arg segIdx,
                                                       lean_obj_arg mbPrio, size_t T, size_t Bmb, size_t D, size_t N) {
  (void)D;
  (void)N;
  lean_obj_res out = new_fa(6 * T * Bmb);
  int rc = pl_gather_seq_minibatch(fa(actCol), fa(logpCol), fa(termCol), fa(advFlat), fa(valueBuf), fa(segIdx),
                                   fa(mbPrio), T, Bmb, fa(out));
  lean_dec(obsCol);
  lean_dec(actCol);
  lean_dec(logpCol);
  lean_dec(termCol);
  lean_dec(advFlat);
  lean_dec(valueBuf);
  lean_dec(segIdx);
  lean_dec(mbPrio);
  return rc ? pure_fail(out, "lean_ffi_gather_seq_minibatch") : out;
}

/* ---------------------------------------------------------------- host bookkeeping (FFI.lean) */
LEAN_EXPORT lean_obj_res lean_ffi_shuffle_perm(size_t NT, size_t epochs, uint64_t rng) {
  lean_obj_res out = new_fa(NT * epochs);
  if (pl_shuffle_perm(NT, epochs, rng, fa(out))) return pure_fail(out, "lean_ffi_shuffle_perm");
  return out;
}

LEAN_EXPORT lean_obj_res lean_ffi_slice(lean_obj_arg arr, size_t off, size_t len) {
  lean_obj_res out = new_fa(len);
  int rc = pl_slice(fa(arr), fan(arr), off, len, fa(out));
  lean_dec(arr);
  return rc ? pure_fail(out, "lean_ffi_slice") : out;
}

LEAN_EXPORT lean_obj_res lean_ffi_gather_minibatch(lean_obj_arg obsCol, lean_obj_arg actions, lean_obj_arg advs,
                                                   lean_obj_arg rets, lean_obj_arg olps, lean_obj_arg idxs, size_t Nmb,
                                                   size_t D) {
  lean_obj_res o[5] = {new_fa(Nmb * D), new_fa(Nmb), new_fa(Nmb), new_fa(Nmb), new_fa(Nmb)};
  /* rows that exist in every column */
  size_t NT = fan(actions);
  if (fan(advs) < NT) NT = fan(advs);
  if (fan(rets) < NT) NT = fan(rets);
  if (fan(olps) < NT) NT = fan(olps);
  if (D && fan(obsCol) / D < NT) NT = fan(obsCol) / D;
  int rc = fan(idxs) < Nmb ? -1
                           : pl_gather_minibatch(fa(obsCol), fa(actions), fa(advs), fa(rets), fa(olps), NT, fa(idxs),
                                                 Nmb, D, fa(o[0]), fa(o[1]), fa(o[2]), fa(o[3]), fa(o[4]));
  lean_dec(obsCol);
  lean_dec(actions);
  lean_dec(advs);
  lean_dec(rets);
  lean_dec(olps);
  lean_dec(idxs);
  if (rc)
    for (int i = 0; i < 5; i++) pure_fail(o[i], "lean_ffi_gather_minibatch");
  /* (mbObs, (mbAct, (mbAdv, (mbRet, mbOlp)))): Prod.mk, constructor 0 with 2 fields */
  lean_obj_res t = o[4];
  for (int i = 3; i >= 0; i--) {
    lean_obj_res p = lean_alloc_ctor(0, 2, 0);
    lean_ctor_set(p, 0, o[i]);
    lean_ctor_set(p, 1, t);
    t = p;
  }
  return t;
}

LEAN_EXPORT lean_obj_res lean_ffi_gae_soa(lean_obj_arg vals, lean_obj_arg rews, lean_obj_arg terms, size_t N, size_t T,
                                          double gamma, double lam) {
  lean_obj_res out = new_fa(2 * N * T);
  int rc = pl_gae_soa(fa(vals), fa(rews), fa(terms), N, T, gamma, lam, fa(out));
  lean_dec(vals);
  lean_dec(rews);
  lean_dec(terms);
  return rc ? pure_fail(out, "lean_ffi_gae_soa") : out;
}
