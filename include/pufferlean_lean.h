/* The reference's Lean `@[extern]` symbols for the PPO+Muon update path, as provided by
 * libpufferlean_lean.so (pufferlean_b200/csrc/pl_lean_abi.c) on top of include/pufferlean_b200.h.
 * Signatures are those of the reference's definitions; each line names the Lean declaration and the
 * reference definition it replaces. Requires <lean/lean.h> (Lean's own, or include/lean_compat). */
#ifndef PUFFERLEAN_LEAN_H
#define PUFFERLEAN_LEAN_H
#include <lean/lean.h>
#include <stdint.h>

#include "pufferlean_b200.h"
#ifdef __cplusplus
extern "C" {
#endif

/* cudaVtraceFFI, Puffer/Float/CUDA.lean:20-22; replaces ffi/puffercuda.cu:94-136 */
lean_obj_res lean_cuda_vtrace(lean_obj_arg rew, lean_obj_arg val, lean_obj_arg term, lean_obj_arg imp, size_t B,
                              size_t T, double gamma, double lam, double rhoClip, double cClip);
/* cudaVtraceMinGRUFFI, CUDA.lean:29-31; replaces ffi/puffercuda.cu:171-216 */
lean_obj_res lean_cuda_vtrace_mingru(lean_obj_arg rew, lean_obj_arg val, lean_obj_arg term, lean_obj_arg imp,
                                     lean_obj_arg bootv, size_t B, size_t T, double gamma, double lam, double rhoClip,
                                     double cClip);
/* cudaMuonStepMatFFI, CUDA.lean:37-39; replaces ffi/puffercuda.cu:559-631 */
lean_obj_res lean_cuda_muon_stepmat(lean_obj_arg W, lean_obj_arg G, lean_obj_arg M, size_t rows, size_t cols,
                                    double lr, double wd, double mu, double eps);
/* cudaMlpPpoGradFFI, CUDA.lean:45-47; replaces ffi/puffercuda.cu:748-816 */
lean_obj_res lean_cuda_mlp_ppo_grad(lean_obj_arg params, lean_obj_arg obs, lean_obj_arg acts, lean_obj_arg advs,
                                    lean_obj_arg rets, lean_obj_arg olps, size_t N, size_t H, size_t D, size_t A,
                                    double vf, double ent, double clip, uint8_t bf16);
/* cudaMlpPpoGradMDFFI / cudaMlpPpoGradContFFI, CUDA.lean:93-106; replace ffi/puffercuda.cu:1570, 1873.
 * Summed gradient g[P]: O = sum(headSizes) + 1 (acts N x K) or O = 2d + 1 (acts N x d). */
lean_obj_res lean_cuda_mlp_ppo_grad_md(lean_obj_arg params, lean_obj_arg obsB, lean_obj_arg acts, lean_obj_arg advs,
                                       lean_obj_arg rets, lean_obj_arg oldlps, lean_obj_arg headSizes, size_t N,
                                       size_t H, size_t D, size_t K, double vfCoef, double entCoef, double clipEps,
                                       uint8_t bf16);
lean_obj_res lean_cuda_mlp_ppo_grad_cont(lean_obj_arg params, lean_obj_arg obsB, lean_obj_arg acts, lean_obj_arg advs,
                                         lean_obj_arg rets, lean_obj_arg oldlps, size_t N, size_t H, size_t D, size_t d,
                                         double vfCoef, double entCoef, double clipEps, uint8_t bf16);
/* cudaAdvNormalizeFFI, CUDA.lean:50-52; replaces ffi/puffercuda.cu:836-855 */
lean_obj_res lean_cuda_adv_normalize(lean_obj_arg adv, size_t n);
/* cudaTrainStepFFI, CUDA.lean:61-63; replaces ffi/puffercuda.cu:988-1080 */
lean_obj_res lean_cuda_train_step(lean_obj_arg pm, lean_obj_arg obs, lean_obj_arg acts, lean_obj_arg advRaw,
                                  lean_obj_arg rets, lean_obj_arg olps, size_t N, size_t H, size_t D, size_t A,
                                  double lr, double wd, double mu, double eps, double vf, double ent, double clip,
                                  uint8_t bf16);
/* cudaTrainUpdateFFI, CUDA.lean:72-75; replaces ffi/puffercuda.cu:1094-1167 */
lean_obj_res lean_cuda_train_update(lean_obj_arg pm, lean_obj_arg obs, lean_obj_arg acts, lean_obj_arg adv,
                                    lean_obj_arg ret, lean_obj_arg olp, lean_obj_arg perm, size_t NT, size_t D,
                                    size_t H, size_t A, size_t epochs, size_t numMB, double lr, double wd, double mu,
                                    double eps, double vf, double ent, double clip, uint8_t bf16);
/* policyLoadFFI / policyDownloadFFI / policyFreeFFI, CUDA.lean:225-230; replace ffi/puffercuda.cu:6100-6116 */
lean_obj_res lean_cuda_policy_load(lean_obj_arg pm, size_t P, lean_obj_arg w);
lean_obj_res lean_cuda_policy_download(size_t handle, size_t P, lean_obj_arg w);
lean_obj_res lean_cuda_policy_free(size_t handle, lean_obj_arg w);
/* cudaTrainUpdateResidentFFI, CUDA.lean:241-244; replaces ffi/puffercuda.cu:1187-1294 */
lean_obj_res lean_cuda_train_update_resident(size_t handle, lean_obj_arg obs, lean_obj_arg acts, lean_obj_arg adv,
                                             lean_obj_arg ret, lean_obj_arg olp, lean_obj_arg ov, lean_obj_arg perm,
                                             size_t NT, size_t D, size_t H, size_t A, size_t epochs, size_t numMB,
                                             double lr, double wd, double mu, double eps, double vf, double ent,
                                             double clip, double vfClip, double maxGradNorm, uint8_t bf16,
                                             lean_obj_arg w);
/* No reference symbol: the deep-MLP form (L hidden layers, act 0 ReLU / 1 GELU) of the call above */
lean_obj_res lean_cuda_train_update_resident_deep(size_t handle, lean_obj_arg obs, lean_obj_arg acts,
                                                  lean_obj_arg adv, lean_obj_arg ret, lean_obj_arg olp,
                                                  lean_obj_arg ov, lean_obj_arg perm, size_t NT, size_t D, size_t H,
                                                  size_t A, size_t L, uint8_t act, size_t epochs, size_t numMB,
                                                  double lr, double wd, double mu, double eps, double vf, double ent,
                                                  double clip, double vfClip, double maxGradNorm, uint8_t bf16,
                                                  lean_obj_arg w);
/* cudaTrainUpdateWideResidentFFI, CUDA.lean:259-262; replaces ffi/puffercuda.cu:1307-1409 (multi-discrete / Gaussian heads) */
lean_obj_res lean_cuda_train_update_wide_resident(size_t handle, lean_obj_arg obs, lean_obj_arg acts, lean_obj_arg adv,
                                                  lean_obj_arg ret, lean_obj_arg olp, lean_obj_arg ov,
                                                  lean_obj_arg perm, lean_obj_arg hs, size_t NT, size_t D, size_t H,
                                                  size_t O, size_t W, uint32_t mode, size_t epochs, size_t numMB,
                                                  double lr, double wd, double mu, double eps, double vf, double ent,
                                                  double clip, double vfClip, double maxGradNorm, uint8_t bf16,
                                                  lean_obj_arg w);
/* cudaMuonStepMlpResidentFFI, CUDA.lean:287-289; replaces ffi/puffercuda.cu:5985-6020 */
lean_obj_res lean_cuda_muon_step_mlp_resident(size_t handle, lean_obj_arg gRaw, size_t H, size_t D, size_t O,
                                              double gscale, double lr, double wd, double mu, double eps,
                                              lean_obj_arg w);
/* lstmPPOGradBatchBlasFFI / ...F32FFI / ...Bf16FFI, Puffer/Float/BLAS.lean:153-174; replace
 * ffi/pufferblas.c:897-1246 (tiers f64 / f32 / bf16-as-f32) */
lean_obj_res lean_ffi_lstm_ppo_grad_batch_blas(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts, lean_obj_arg advs,
                                               lean_obj_arg rets, lean_obj_arg olps, lean_obj_arg terms,
                                               lean_obj_arg h0s, lean_obj_arg c0s, size_t B, size_t T, size_t H,
                                               size_t D, size_t A, double vf, double ent, double clip);
lean_obj_res lean_ffi_lstm_ppo_grad_batch_blas_f32(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts,
                                                   lean_obj_arg advs, lean_obj_arg rets, lean_obj_arg olps,
                                                   lean_obj_arg terms, lean_obj_arg h0s, lean_obj_arg c0s, size_t B,
                                                   size_t T, size_t H, size_t D, size_t A, double vf, double ent,
                                                   double clip);
lean_obj_res lean_ffi_lstm_ppo_grad_batch_blas_bf16(lean_obj_arg pa, lean_obj_arg obs, lean_obj_arg acts,
                                                    lean_obj_arg advs, lean_obj_arg rets, lean_obj_arg olps,
                                                    lean_obj_arg terms, lean_obj_arg h0s, lean_obj_arg c0s, size_t B,
                                                    size_t T, size_t H, size_t D, size_t A, double vf, double ent,
                                                    double clip);
/* cudaLstmReuseInputsFFI, CUDA.lean:172; replaces ffi/puffercuda.cu:344 */
lean_obj_res lean_cuda_lstm_reuse_inputs(uint8_t on, lean_obj_arg w);
/* lstmGaeBootNormFFI, FFI.lean:91-92; replaces ffi/pufferffi.c:975-1010 */
lean_obj_res lean_ffi_lstm_gae_boot_norm(lean_obj_arg vals, lean_obj_arg rews, lean_obj_arg terms, lean_obj_arg boot,
                                         size_t N, size_t T, double gamma, double lam);
/* cudaMgLossEnableFFI / cudaMgReadLossesFFI, CUDA.lean:165-178; replace ffi/puffercuda.cu:336-352 */
lean_obj_res lean_cuda_mg_loss_enable(uint8_t on, lean_obj_arg w);
lean_obj_res lean_cuda_mg_read_losses(lean_obj_arg w);
/* shufflePermFFI / gaeSoaFFI, Puffer/Float/FFI.lean; replace ffi/pufferffi.c:1017-1041 and :946-971 */
lean_obj_res lean_ffi_shuffle_perm(size_t NT, size_t epochs, uint64_t rng);
lean_obj_res lean_ffi_gae_soa(lean_obj_arg vals, lean_obj_arg rews, lean_obj_arg terms, size_t N, size_t T,
                              double gamma, double lam);
/* sliceFFI, FFI.lean:76-77; replaces ffi/pufferffi.c:13-20. A range outside the array gives NaNs. */
lean_obj_res lean_ffi_slice(lean_obj_arg arr, size_t off, size_t len);
/* gatherMinibatchFFI, FFI.lean:105-107; replaces ffi/pufferffi.c:1046-1081. Returns
 * (mbObs, (mbAct, (mbAdv, (mbRet, mbOlp)))); NT is the length of the action column, and an index that
 * is not a row of it gives NaN-filled arrays. */
lean_obj_res lean_ffi_gather_minibatch(lean_obj_arg obsCol, lean_obj_arg actions, lean_obj_arg advs, lean_obj_arg rets,
                                       lean_obj_arg olps, lean_obj_arg idxs, size_t Nmb, size_t D);

/* MinGRU path. cudaMgPrepFFI, CUDA.lean:154-155; replaces ffi/puffercuda.cu:316-335 */
lean_obj_res lean_cuda_mg_prep(lean_obj_arg rew, lean_obj_arg term, lean_obj_arg act, lean_obj_arg logp,
                               lean_obj_arg val, lean_obj_arg boot, size_t N, size_t T, size_t K, lean_obj_arg w);
/* cudaMgColsReadyFFI, CUDA.lean:361-362; replaces ffi/puffercuda.cu:305-309 */
lean_obj_res lean_cuda_mg_cols_ready(size_t N, size_t T, lean_obj_arg w);
/* cudaMgVtraceFFI, CUDA.lean:159-160; replaces ffi/puffercuda.cu:389-399 */
/* cudaMgChainReadyFFI, CUDA.lean:338; replaces ffi/puffercuda.cu:284-289 (IO Bool). */
lean_obj_res lean_cuda_mg_chain_ready(size_t N, size_t D, size_t LH, lean_obj_arg w);
lean_obj_res lean_cuda_mg_vtrace(size_t N, size_t T, double gamma, double lam, double rhoClip, double cClip,
                                 lean_obj_arg w);
/* cudaMgVtracePrioFFI, CUDA.lean:369-371; replaces ffi/puffercuda.cu:443-470 */
lean_obj_res lean_cuda_mg_vtrace_prio(size_t N, size_t T, double gamma, double lam, double rhoClip, double cClip,
                                      size_t mbSegs, double prioAlpha, double annealBeta, uint64_t rng,
                                      lean_obj_arg w);
/* cudaMinGRUPpoGradFFI, CUDA.lean:126-129; replaces ffi/puffercuda.cu:5206-5622 */
lean_obj_res lean_cuda_mingru_ppo_grad(lean_obj_arg params, lean_obj_arg obs, lean_obj_arg scal, size_t B, size_t T,
                                       size_t H, size_t D, size_t L, size_t A, size_t K, lean_obj_arg hs,
                                       double vfCoef, double entCoef, double clipEps, double vfClip,
                                       lean_obj_arg segIdx, lean_obj_arg mbPrio, lean_obj_arg w);
/* cudaMinGRUMuonResidentFFI, CUDA.lean:354-356; replaces ffi/puffercuda.cu:5727-5976 */
lean_obj_res lean_cuda_mingru_muon_resident(size_t handle, lean_obj_arg gClip, size_t H, size_t D, size_t L,
                                            size_t A, double lr, double wd, double mu, double eps,
                                            double maxGradNorm, double gscale, lean_obj_arg w);
/* No reference counterpart: the pl_mg session behind the MinGRU symbols (NULL before the first
 * lean_cuda_mg_prep); the rollout passes its device obs trajectory to pl_mg_set_obs_dev on it. */
pl_mg* pl_lean_mg_session(void);
/* prioSampleFFI / gatherSeqMinibatchFFI, Puffer/Float/FFI.lean:113-125; replace ffi/pufferffi.c:1094-1125
 * and :1137-1176 */
lean_obj_res lean_ffi_prio_sample(lean_obj_arg advL1, size_t N, size_t T, size_t mbSegs, double prioAlpha,
                                  double annealBeta, uint64_t rng);
lean_obj_res lean_ffi_gather_seq_minibatch(lean_obj_arg obsCol, lean_obj_arg actCol, lean_obj_arg logpCol,
                                           lean_obj_arg termCol, lean_obj_arg advFlat, lean_obj_arg valueBuf,
                                           lean_obj_arg segIdx, lean_obj_arg mbPrio, size_t T, size_t Bmb, size_t D,
                                           size_t N);

#ifdef __cplusplus
}
#endif
#endif
