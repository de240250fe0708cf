/* pufferlean_b200 -- B200 (sm_100a) implementation of pufferlean's PPO+Muon training update.
 *
 * Plain C ABI: host or device pointers, sizes, scalars, status codes. No Lean, torch or CUDA
 * types cross it (streams are passed as void*). Each entry point names the reference symbol it
 * replaces (file:line within the reference project). The reference's Lean `@[extern]` symbols
 * (lean_cuda_*, lean_ffi_*) are provided on top of this ABI by the adapter declared in
 * include/pufferlean_lean.h.
 *
 * Conventions shared with the reference:
 *  - f64 host arrays in row-major order; parameter vectors use the flat layout
 *    [W1(H*D) | b1(H) | W2(O*H) | b2(O)], O = A+1 (logits then value), and the policy handle owns
 *    the combined [params(P); mom(P)] buffer (ffi/puffercuda.cu:6100-6116);
 *  - gradients are of the PPO OBJECTIVE and Muon ascends (ffi/pufferblas.c:1397-1398);
 *  - bf16 = 1 selects the bf16 tensor-core tier (fp32 accumulate, f64 master weights and momentum);
 *    bf16 = 0 the tight tier (fp32 GEMMs, f64 Newton-Schulz in the reference's op order).
 *
 * Every function returns PL_OK (0) or a negative status; pl_last_error() describes the failure.
 * There is no CPU fallback: without a usable device, calls fail with PL_ERR_NO_DEVICE.
 */
#ifndef PUFFERLEAN_B200_H
#define PUFFERLEAN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PL_OK 0
#define PL_ERR_INVALID (-1)
#define PL_ERR_CUDA (-2)
#define PL_ERR_NOMEM (-3)
#define PL_ERR_UNSUPPORTED (-4)
#define PL_ERR_DEVICE_TIMEOUT (-5)
#define PL_ERR_NO_DEVICE (-6)
#define PL_ERR_COMM (-7)

/* Message for the calling thread's most recent failure ("" if none). */
const char* pl_last_error(void);
/* Number of CUDA devices visible to this process. */
int pl_device_count(void);
/* Selects the device later calls from this thread use (default 0). */
int pl_set_device(int device);
/* Number of this library's kernels launched since load (all threads, all devices). */
uint64_t pl_kernel_launch_count(void);

/* ------------------------------------------------------------------ advantage scans ----------- */

/* V-trace, vector-delta form, f64, bit-exact with the reference's scan (host buffers, B*T row-major).
 * Replaces lean_cuda_vtrace (ffi/puffercuda.cu:94-136; Puffer/Float/CUDA.lean:20-22). */
int pl_vtrace(const double* rew, const double* val, const double* term, const double* imp, size_t B, size_t T,
              double gamma, double lam, double rhoClip, double cClip, double* adv);

/* V-trace, MinGRU scalar-delta form with bootstrap bootv[B], f64, bit-exact.
 * Replaces lean_cuda_vtrace_mingru (ffi/puffercuda.cu:171-216; Puffer/Float/CUDA.lean:29-31). */
int pl_vtrace_mingru(const double* rew, const double* val, const double* term, const double* imp,
                     const double* bootv, size_t B, size_t T, double gamma, double lam, double rhoClip,
                     double cClip, double* adv);

/* Device-resident scans (all pointers device pointers; stream may be NULL).
 * bootv == NULL selects the vector form (adv[T-1] = 0), else the MinGRU form. adv_l1, if not NULL,
 * receives sum_t |adv[b,t]| per segment (the k_vtrace_mingru + k_adv_l1 pair,
 * ffi/puffercuda.cu:146-167, 311-312). The f32 form is the fast tier (warp per segment,
 * shuffle-based reverse scan); the f64 form keeps the reference's sequential op order. */
int pl_vtrace_f32_dev(const float* rew, const float* val, const float* term, const float* imp, const float* bootv,
                      size_t B, size_t T, double gamma, double lam, double rhoClip, double cClip, float* adv,
                      float* adv_l1, void* stream);
int pl_vtrace_f64_dev(const double* rew, const double* val, const double* term, const double* imp,
                      const double* bootv, size_t B, size_t T, double gamma, double lam, double rhoClip,
                      double cClip, double* adv, double* adv_l1, void* stream);
/* The f64 scan in the fp32 form's warp-parallel order (one warp per segment, coalesced loads, affine
 * maps composed by shuffles): not bit-identical to the sequential order, about 1e-15 relative. The
 * recurrent update's bf16 tier uses it. No separate reference symbol (same semantics as above). */
int pl_vtrace_f64_scan_dev(const double* rew, const double* val, const double* term, const double* imp,
                           const double* bootv, size_t B, size_t T, double gamma, double lam, double rhoClip,
                           double cClip, double* adv, double* adv_l1, void* stream);

/* ------------------------------------------------------------------ host bookkeeping ---------- */

/* out = arr[off, off + len) of an n-element array; the range must lie inside it (PL_ERR_INVALID
 * otherwise). Replaces lean_ffi_slice (ffi/pufferffi.c:13-20; Puffer/Float/FFI.lean:76-77). */
int pl_slice(const double* arr, size_t n, size_t off, size_t len, double* out);
/* Minibatch gather from the SoA columns of NT rows: row k takes column row (size_t)idxs[k] (f64-encoded
 * index, truncated like the reference's cast): mbObs[k*D + j] = obsCol[i*D + j], mbAct/mbAdv/mbRet/
 * mbOlp[k] = the scalar columns at i. Bit-exact; an index that is NaN, negative or >= NT fails with
 * PL_ERR_INVALID before anything is written. Replaces lean_ffi_gather_minibatch
 * (ffi/pufferffi.c:1046-1081; Puffer/Float/FFI.lean:105-107). */
int pl_gather_minibatch(const double* obsCol, const double* actions, const double* advs, const double* rets,
                        const double* olps, size_t NT, const double* idxs, size_t Nmb, size_t D, double* mbObs,
                        double* mbAct, double* mbAdv, double* mbRet, double* mbOlp);
/* Per-epoch Fisher-Yates with splitmix64, f64-encoded, bit-exact.
 * Replaces lean_ffi_shuffle_perm (ffi/pufferffi.c:1017-1041). out has epochs*NT entries. */
int pl_shuffle_perm(size_t NT, size_t epochs, uint64_t rng, double* out);
/* Truncated GAE + returns over env segments (row e*T+t), bit-exact. out = [adv(NT); ret(NT)].
 * Replaces lean_ffi_gae_soa (ffi/pufferffi.c:946-971). */
int pl_gae_soa(const double* vals, const double* rews, const double* terms, size_t N, size_t T, double gamma,
               double lam, double* out);

/* ------------------------------------------------------------------ Muon ---------------------- */

/* One Muon step of one matrix in the tight tier (f64 Newton-Schulz, reference op order, bit-exact).
 * out = [newW(rows*cols); newMom(rows*cols)].
 * Replaces lean_cuda_muon_stepmat (ffi/puffercuda.cu:559-631; Puffer/Float/CUDA.lean:37-39). */
int pl_muon_stepmat(const double* W, const double* G, const double* M, size_t rows, size_t cols, double lr,
                    double wd, double mu, double eps, double* out);

/* Newton-Schulz orthogonalisation of a batch of equally shaped bf16 matrices on the device
 * (tensor cores, fp32 accumulate): X[b] <- NS(X[b] / (||X[b]||_F + eps)) with an iters x 3
 * coefficient table (host, row-major). X is batch x rows x cols, updated in place; rows and cols are
 * multiples of 8. Tall matrices are orthogonalised through their transpose. */
int pl_ns_batched_bf16_dev(void* X, size_t batch, size_t rows, size_t cols, double eps, const double* coeffs,
                           size_t iters, void* stream);

/* Several such batches in one call: group k is batch[k] matrices of rows[k] x cols[k] at X[k], each
 * orthogonalised in place with the same bits pl_ns_batched_bf16_dev gives it alone. The wide groups
 * whose short side exceeds 128 (two steps or more) share one persistent launch, four groups at most
 * per launch, so that one group's short dependent products run while another's tiles fill the SMs;
 * the other groups run as pl_ns_batched_bf16_dev runs them, before those. At most 16 groups. No
 * counterpart in the reference, whose batched Newton-Schulz takes one shape per call. */
int pl_ns_groups_bf16_dev(size_t ngroups, void* const* X, const size_t* batch, const size_t* rows,
                          const size_t* cols, double eps, const double* coeffs, size_t iters, void* stream);

/* The same batched Newton-Schulz over the ranks of a communicator (pl_comm_create): every rank passes
 * the same batch and ends with every result, bit-identical to pl_ns_batched_bf16_dev on one GPU. The
 * batch is cut into `chunks` chunks of world * cs matrices; in each chunk a rank orthogonalises its cs
 * matrices in place and the chunk is all-gathered (ncclAllGather, in place) on a second stream while
 * the next chunk is orthogonalised; the matrices left over (fewer than world * chunks) are
 * orthogonalised on every rank under the last all-gather. A batch of matrices with a short side of at
 * most 128 and a long side of at most 512 runs whole on every rank (its fused one-CTA-per-matrix
 * kernel is latency-bound: sharding would only add the gather).
 * Work is enqueued on `stream`, which waits for the gathers. A collective: every rank calls it with
 * the same shape and chunk count.
 * BASELINE configs[2] at N > 1 ("sharded across 1/2/4/8 GPUs, followed by an all-gather"); no
 * counterpart in the reference, which has no multi-GPU code. */
int pl_ns_batched_bf16_dev_sharded(void* X, size_t batch, size_t rows, size_t cols, double eps,
                                   const double* coeffs, size_t iters, void* comm, size_t chunks, void* stream);
/* The plan pl_ns_batched_bf16_dev_sharded follows: *per_rank matrices per rank and chunk and *used
 * chunks (the request clamped to [1, 16] and lowered until a chunk holds at least one matrix per
 * rank; 0 chunks when the batch has fewer matrices than ranks). Chunk c's rank r matrices are
 * [c world per_rank + r per_rank, c world per_rank + (r + 1) per_rank); the rest of the batch, from
 * used * world * per_rank on, runs on every rank. Host only. */
int pl_ns_shard_chunks(size_t batch, size_t world, size_t chunks, size_t* per_rank, size_t* used);

/* The same batched Newton-Schulz without allocating device memory, for callers that cannot call
 * cudaMalloc: hosts whose device memory belongs to another allocator or to a budget fixed at
 * start-up, and loops that must stay off the driver's allocator (whose calls can block and
 * synchronise the device). No counterpart in the reference. The workspace is a fixed 32 MiB array
 * inside the library, held on every GPU that loads it until exit. A request needs, each region
 * rounded up to 256 bytes: 2*batch*m*n bf16 + 2*batch*m*m bf16 + batch*ceil(m*n/16384) doubles +
 * (3*batch + 1) 32-bit words + 2*batch floats + 256 bytes, with m = min(rows,cols) and
 * n = max(rows,cols); larger requests fail with PL_ERR_INVALID before anything runs. All calls on a
 * device share that array and it keeps the last call's contents, so calls that overlap on the GPU
 * race: serialise them. The call waits for its work on `stream` and returns PL_ERR_DEVICE_TIMEOUT
 * if a device-side bounded wait ran out. The first call on a device looks the array up
 * (cudaGetSymbolAddress) and clears its error word. */
int pl_ns_batched_bf16_dev_noalloc(void* X, size_t batch, size_t rows, size_t cols, double eps,
                                   const double* coeffs, size_t iters, void* stream);

/* ------------------------------------------------------------------ MLP PPO -------------------- */

/* Summed PPO-objective gradient of the one-hidden-layer MLP (host buffers).
 * Replaces lean_cuda_mlp_ppo_grad (ffi/puffercuda.cu:748-816; Puffer/Float/CUDA.lean:45-47). */
int pl_mlp_ppo_grad(const double* params, const double* obs, const double* acts, const double* advs,
                    const double* rets, const double* oldlps, size_t N, size_t H, size_t D, size_t A,
                    double vfCoef, double entCoef, double clipEps, uint8_t bf16, double* g);

/* (adv - mean) / (std + 1e-8), population std.
 * Replaces lean_cuda_adv_normalize (ffi/puffercuda.cu:836-855; Puffer/Float/CUDA.lean:50-52). */
int pl_adv_normalize(const double* adv, size_t n, double* out);

/* One resident step: normalize -> mean gradient -> Muon. pm/pm_out = [params; mom] (2P).
 * Replaces lean_cuda_train_step (ffi/puffercuda.cu:988-1080; Puffer/Float/CUDA.lean:61-63). */
int pl_train_step(const double* pm, const double* obs, const double* acts, const double* advRaw,
                  const double* rets, const double* oldlps, size_t N, size_t H, size_t D, size_t A, double lr,
                  double wd, double mu, double eps, double vfCoef, double entCoef, double clipEps, uint8_t bf16,
                  double* pm_out);

/* Whole update (all epochs x minibatches) with host-threaded [params; mom].
 * Replaces lean_cuda_train_update (ffi/puffercuda.cu:1094-1167; Puffer/Float/CUDA.lean:72-75). */
int pl_train_update(const double* pm, const double* obs, const double* acts, const double* adv,
                    const double* ret, const double* olp, const double* perm, size_t NT, size_t D, size_t H,
                    size_t A, size_t epochs, size_t numMB, double lr, double wd, double mu, double eps,
                    double vfCoef, double entCoef, double clipEps, uint8_t bf16, double* pm_out);

/* Device-resident policy: [params(P); mom(P)] f64 in device memory behind an opaque handle.
 * Replace lean_cuda_policy_load / _download / _free (ffi/puffercuda.cu:6100-6116). */
int pl_policy_load(const double* pm, size_t P, size_t* handle);
int pl_policy_download(size_t handle, size_t P, double* pm_out);
int pl_policy_free(size_t handle);

/* Whole update on the resident policy, updated in place; params0_out receives params[0].
 * oldVal may be NULL / oldValN < NT (value clip off); vfClip <= 0 and maxGradNorm <= 0 select
 * the unclipped arithmetic, as in the reference.
 * Replaces lean_cuda_train_update_resident (ffi/puffercuda.cu:1187-1294; Puffer/Float/CUDA.lean:241-244). */
int pl_train_update_resident(size_t handle, const double* obs, const double* acts, const double* adv,
                             const double* ret, const double* olp, const double* oldVal, size_t oldValN,
                             const double* perm, size_t NT, size_t D, size_t H, size_t A, size_t epochs,
                             size_t numMB, double lr, double wd, double mu, double eps, double vfCoef,
                             double entCoef, double clipEps, double vfClip, double maxGradNorm, uint8_t bf16,
                             double* params0_out);

/* Network shape beyond the reference's single hidden layer. L hidden layers of width H (L = 1 is the
 * reference layout), hidden activation act (0 = ReLU as in the reference, 1 = GELU tanh form,
 * Puffer/Net/Forward.lean:271-273), and the Newton-Schulz coefficient table (NULL = the reference's
 * tuned 5-row table, Puffer/Float/Muon.lean:64-67). Flat layout
 * [W1|b1|W2|b2|...|W_L|b_L|W_out|b_out]. */
typedef struct {
  size_t L;
  int act;
  const double* ns_coeffs; /* iters x 3, row-major; NULL = reference table */
  size_t ns_iters;
} pl_mlp_arch;

/* Parameter count of the flat layout for (D, H, A, L). */
size_t pl_mlp_param_count(size_t D, size_t H, size_t A, size_t L);

/* Deep variant of pl_train_update_resident (no reference symbol: the reference MLP has one hidden
 * layer, ffi/puffercuda.cu:746). Same conventions plus `arch`. */
int pl_train_update_resident_deep(size_t handle, const pl_mlp_arch* arch, const double* obs, const double* acts,
                                  const double* adv, const double* ret, const double* olp, const double* oldVal,
                                  size_t oldValN, const double* perm, size_t NT, size_t D, size_t H, size_t A,
                                  size_t epochs, size_t numMB, double lr, double wd, double mu, double eps,
                                  double vfCoef, double entCoef, double clipEps, double vfClip, double maxGradNorm,
                                  uint8_t bf16, double* params0_out);

/* ------------------------------------------------------------------ update sessions ------------ */
/* A session binds a policy handle to fixed shapes and keeps the rollout columns and every
 * per-minibatch buffer resident, so an update can be run from device memory alone (the form the
 * reference reaches when its rollout leaves the obs trajectory on the device, ffi/puffercuda.cu:1226-1228).
 * pl_train_update_resident(_deep) is a session created on first use plus one host upload per call. */
typedef struct pl_update pl_update;
typedef struct {
  size_t NT, D, H, A, epochs, numMB;
  pl_mlp_arch arch;
  double wd, mu, eps, vfCoef, entCoef, clipEps, vfClip, maxGradNorm;
  uint8_t bf16;
  uint8_t use_old_values; /* value clip needs the old-value column */
  /* data-parallel group: rank/world; comm = a communicator from pl_comm_create, or NULL at world 1 */
  int rank, world;
  void* comm;
} pl_update_desc;

int pl_update_create(size_t handle, const pl_update_desc* desc, pl_update** out);
/* Host columns (f64, the reference ABI's form); uploaded and converted on the device. perm is the
 * epochs*NT f64-encoded shuffle. oldVal may be NULL when desc->use_old_values is 0. */
int pl_update_set_columns(pl_update* u, const double* obs, const double* acts, const double* adv,
                          const double* ret, const double* olp, const double* oldVal, const double* perm,
                          void* stream);
/* Device columns: obs as fp32 [NT x D], the rest f64 [NT] (perm f64 [epochs*NT]). Copied into the
 * session's own layout on the device. adv, ret and oldVal may be NULL when
 * pl_update_set_advantages_dev computes them on the device. */
int pl_update_set_columns_dev(pl_update* u, const float* obs, const double* acts, const double* adv,
                              const double* ret, const double* olp, const double* oldVal, const double* perm,
                              void* stream);
/* Advantages on the device for the session's columns: the fp32 V-trace scan in its vector form
 * over N = NT/T segments of horizon T (row e*T + t, the layout of ffi/pufferffi.c:946), with
 * importance ratios `imp` (NULL = all ones, which is truncated GAE), then ret = adv + val. The old
 * value column of the value clip is set to val. rew/val/term/imp are device fp32 [NT]. */
int pl_update_set_advantages_dev(pl_update* u, const float* rew, const float* val, const float* term,
                                 const float* imp, size_t T, double gamma, double lam, double rhoClip, double cClip,
                                 void* stream);
/* Runs every epoch x minibatch of one update at learning rate lr on `stream`. */
int pl_update_run(pl_update* u, double lr, void* stream);
/* pl_update_set_columns + pl_update_run in one call, with the upload of the reference-shaped update
 * entries (ffi/puffercuda.cu:1187, lean_cuda_train_update_resident): in the bf16 tier, rows of 64 or
 * more observations are read from the host during the call in the first epoch's shuffle order, one
 * minibatch ahead of the kernels that use them, so the upload runs under the compute. The host columns
 * must stay unchanged until the call returns; a first-epoch shuffle entry that is not a row index in
 * [0, NT) fails the call. Results are identical to the two calls. */
int pl_update_run_columns(pl_update* u, const double* obs, const double* acts, const double* adv, const double* ret,
                          const double* olp, const double* oldVal, const double* perm, double lr, void* stream);
/* Kernels launched by the last pl_update_run (this library's own kernels). */
uint64_t pl_update_last_launches(const pl_update* u);
/* Host-to-device bytes the last pl_update_set_columns call (of any session in the process; the
 * reference-shaped update entries call it once per update) copied: observations as bf16 rows where
 * the host threads rounded them and as f64 rows otherwise, plus the scalar columns and the shuffle. */
uint64_t pl_update_last_upload_bytes(void);
/* Per-class kernel timing with CUDA events on the launch stream while `on` (classes: 0 forward GEMM,
 * 1 PPO-head GEMM, 2 data-gradient GEMM, 3 weight-gradient GEMM incl. split-K sum, 4 Newton-Schulz
 * GEMMs, 5 gather/statistics, 6 optimizer elementwise and reductions, 7 data-parallel collectives).
 * pl_update_profile_read
 * synchronizes and returns, per class, total milliseconds, algorithmic flops and launches since
 * profiling was switched on. */
int pl_update_profile(pl_update* u, int on);
int pl_update_profile_read(pl_update* u, double ms[8], double flops[8], double launches[8]);
/* Data parallel: the gradient all-reduces on the session's communication stream since profiling was
 * switched on: their total milliseconds on that stream (class 7 above is the part of it the compute
 * stream had to wait for), bytes reduced per rank and launches. */
int pl_update_comm_profile_read(pl_update* u, double* ms, double* bytes, double* launches);
/* Strong-scaling form of a data-parallel session (no reference counterpart): every rank holds the
 * same columns and the same shuffle, and rank r of R takes rows [lo + n*r/R, lo + n*(r+1)/R) of each
 * minibatch [lo, lo + n), so the R ranks together run exactly the single-GPU update's minibatches
 * (the advantage statistics and the gradient mean are over the whole minibatch). Without it (the
 * default) every rank brings its own rollout. Needs at least R rows per minibatch. */
int pl_update_split_minibatch(pl_update* u, int on);
int pl_update_destroy(pl_update* u);

/* ------------------------------------------------------------------ data parallelism ----------- */
/* One process per GPU over NCCL (no reference counterpart: the reference is single-GPU,
 * docs/KNOWN_GAPS.md:349). Rank 0 draws a 128-byte id, the caller hands it to every rank by any side
 * channel, each rank creates its communicator on its current device and passes it to
 * pl_update_create through pl_update_desc {rank, world, comm}. In a data-parallel update every rank
 * gathers its own rows of each minibatch; the advantage statistics and the summed gradient are
 * all-reduced (the gradient layer by layer on a second stream, each block as soon as the backward pass
 * has finished it); each weight matrix is orthogonalised by one owner rank (pl_muon_shard_plan) and the
 * results are broadcast; every rank then applies the identical step. */
int pl_comm_unique_id(uint8_t id[128]);
/* Creates this rank's communicator non-blocking and polls it with the deadline of pl_comm_set_timeout:
 * a peer that never joins makes it fail with PL_ERR_COMM (the half-made communicator is aborted). */
int pl_comm_create(int rank, int world, const uint8_t id[128], void** comm);
int pl_comm_destroy(void* comm);
/* Deadline of every blocking step of the communicator (creation, an enqueue that answers "in
 * progress", pl_comm_wait), in seconds; 600 by default. Applies to later calls in the process. */
int pl_comm_set_timeout(double seconds);
/* Watchdog of enqueued work: waits until `stream` has finished while polling the communicator's
 * asynchronous error state. An error (a peer that died, a network error) or the deadline aborts the
 * communicator (ncclCommAbort, which also releases NCCL kernels still waiting for a peer) and returns
 * PL_ERR_COMM. Every later call on an aborted communicator, and every update session or MinGRU state
 * that uses it, fails with PL_ERR_COMM before enqueuing anything. */
int pl_comm_wait(void* comm, void* stream);
/* Aborts the communicator (e.g. after the host learned that a peer left); idempotent. */
int pl_comm_abort(void* comm);
/* 1 if the communicator was aborted, 0 if not, -1 if it is not a communicator of this library. */
int pl_comm_aborted(void* comm);
/* Owner rank of each of nmat matrices (rows[i] x cols[i]) for the sharded Newton-Schulz: greedy
 * longest-processing-time by 4 m^2 n + 2 m^3 flops. Deterministic. */
int pl_muon_shard_plan(const size_t* rows, const size_t* cols, size_t nmat, int world, int* owner);

/* ------------------------------------------------------------------ MinGRU (recurrent) path ----- */
/* The network of Puffer/Net/MinGRU.lean:9-17 in the flattenMG layout (Puffer/RL/MinGRUTrain.lean:282-292):
 * [wEnc(H*D) | bEnc(H) | L x layer(K*H x H) | wDec(A*H) | bDec(A) | wVal(H) | bVal(1)].
 * K = 3: [hid | gate | proj] with the highway output (the reference); K = 2: [hid | gate], the output is
 * the scan state. enc_act 0: linear encoder (the reference); 1: GELU after the encoder. */
typedef struct {
  size_t D, H, L, A, K;
  int enc_act;
} pl_mg_net;
size_t pl_mg_param_count(const pl_mg_net* net);

/* Host-buffer BPTT gradient: B sequences of T steps packed time-major (obs [(t*B+b)*D + j], scal =
 * [act | adv | ret | old | term | ov] each [t*B + b]); zero initial state, state reset after a terminal.
 * out = [summed ascent gradient (P); new log-prob (T*B); new value (T*B)].
 * bf16 = 0: fp32 GEMMs and activations; 1: bf16 tensor-core GEMMs (fp32 accumulate), bf16 activations.
 * Replaces the host mode of lean_cuda_mingru_ppo_grad (ffi/puffercuda.cu:5206-5622). */
int pl_mingru_ppo_grad(const double* params, const double* obs, const double* scal, size_t B, size_t T,
                       const pl_mg_net* net, double vfCoef, double entCoef, double clipEps, double vfClip,
                       uint8_t bf16, double* out);

/* The same with W multi-discrete heads of sizes head_sizes (summing to net->A): scal is
 * [act (W per row, [(t*B + b)*W + h]) | adv | ret | old | term | ov], (W + 5)*T*B values; the head is
 * k_mg_ppo_b_md's (joint log-prob in double). W = 1 is pl_mingru_ppo_grad. Replaces the K > 1 host mode
 * of lean_cuda_mingru_ppo_grad (ffi/puffercuda.cu:5204-5221, 5428). */
int pl_mingru_ppo_grad_md(const double* params, const double* obs, const double* scal, size_t B, size_t T,
                          const pl_mg_net* net, size_t W, const double* head_sizes, double vfCoef, double entCoef,
                          double clipEps, double vfClip, uint8_t bf16, double* out);

/* Host bookkeeping twins, bit-exact: prioritised segment sampling (replaces lean_ffi_prio_sample,
 * ffi/pufferffi.c:1094-1125) and the MinGRU minibatch scalar gather (replaces
 * lean_ffi_gather_seq_minibatch, ffi/pufferffi.c:1137-1176; out = 6*T*Bmb, [act|adv|ret|old|term|ov]). */
int pl_prio_sample(const double* advL1, size_t N, size_t mbSegs, double prioAlpha, double annealBeta, uint64_t rng,
                   double* segIdx, double* mbPrio);
int pl_gather_seq_minibatch(const double* actCol, const double* logpCol, const double* termCol,
                            const double* advFlat, const double* valueBuf, const double* segIdx, const double* mbPrio,
                            size_t T, size_t Bmb, double* out);

/* Resident MinGRU state: the rollout's N x T columns (rows e*T + t) on the device, the live value and
 * importance-ratio buffers the replay iterates, the device obs trajectory, the sampled minibatch, the
 * BPTT workspace and the resident gradient. One object replaces the reference's process-global
 * device columns and caches (ffi/puffercuda.cu:225-507, 5132-5622, 5727-5976). */
typedef struct pl_mg pl_mg;
int pl_mg_create(size_t N, size_t T, pl_mg** out);
/* Replaces lean_cuda_mg_prep (ffi/puffercuda.cu:316-335): uploads rew, term, act, logp, val [N*T] and
 * boot [N] (host f64); value := val, ratio := 1. The _dev form takes device f64 pointers. */
int pl_mg_set_columns(pl_mg* s, const double* rew, const double* term, const double* act, const double* logp,
                      const double* val, const double* boot);
int pl_mg_set_columns_dev(pl_mg* s, const double* rew, const double* term, const double* act, const double* logp,
                          const double* val, const double* boot, void* stream);
/* Rollout-side column producer (replaces the reference's device column stamping, ffi/puffercuda.cu:242-309,
 * and its obs-trajectory scatter, :975-983): a rollout stamps each step's device outputs straight into
 * the session's columns, so they never pass through the host. pl_mg_stamp_step writes step `step` of
 * envs [e0, e0 + ne): act [ne x W] (the session's head width), logp and val [ne] (device f64; val also
 * becomes the live value), obs [ne x D] (device f32, may be NULL) into the session's own trajectory.
 * pl_mg_stamp_finish takes the whole update's reward and terminal planes, step-major [T x N] (row
 * s*N + e, the rollout's staging order), and boot [N] (device f64); the columns are then complete.
 * pl_mg_take_stamped reports (once) whether the current columns came from the stamps. */
int pl_mg_stamp_step(pl_mg* s, size_t step, size_t e0, size_t ne, const double* act, const double* logp,
                     const double* val, const float* obs, size_t D, void* stream);
int pl_mg_stamp_finish(pl_mg* s, const double* rew, const double* term, const double* boot, void* stream);
int pl_mg_take_stamped(pl_mg* s, int* stamped);
/* Resident chaining (the reference's g_mgchain protocol, ffi/puffercuda.cu:255-289): a rollout that keeps
 * its observations and recurrent state resident across updates stamps (N envs, obs D, L*H state);
 * N = 0 clears the stamp. pl_mg_chain_ready reports whether the stamp matches a query (the trainer then
 * passes empty obs0 / state0 to that rollout). */
int pl_mg_chain_stamp(pl_mg* s, size_t N, size_t D, size_t LH);
int pl_mg_chain_ready(pl_mg* s, size_t N, size_t D, size_t LH, int* ready);
/* The same scatters on caller-owned columns (the feed-forward path's obs trajectory and columns for
 * pl_update_set_columns_dev): src holds ne rows of `width` values for step `step`, written to rows
 * e*T + step of col [N*T x width]; a plane is step-major [T x N]. */
int pl_stamp_rows_f64(double* col, size_t width, size_t N, size_t T, size_t step, size_t e0, size_t ne,
                      const double* src, void* stream);
int pl_stamp_rows_f32(float* col, size_t width, size_t N, size_t T, size_t step, size_t e0, size_t ne,
                      const float* src, void* stream);
int pl_stamp_plane_f64(double* col, size_t N, size_t T, const double* plane, void* stream);
/* Action heads of the session (the K of lean_cuda_mg_prep / lean_cuda_mingru_ppo_grad,
 * ffi/puffercuda.cu:316-335, 5204-5221): W = 1 one categorical head (the default); W > 1 multi-discrete
 * heads, the act column then holds W actions per row ([(e*T + t)*W + h]) and head_sizes (W values,
 * summing to the network's A) select the heads' logits. Changing W drops the columns (set them again
 * after); head_sizes may be NULL to fix the width first and give the sizes before the gradient. */
int pl_mg_set_heads(pl_mg* s, size_t W, const double* head_sizes);
/* Data parallelism (no reference counterpart; the reference trainer is single-GPU): one process and
 * session per GPU, each with its own rollout columns (weak scaling). With world > 1, pl_mg_grad
 * all-reduces the advantage sums (the normalisation uses the all-rank minibatch) and the summed
 * gradient over `comm` (from pl_comm_create); pl_mg_update scales by the all-rank row count; every
 * rank then takes the identical Muon step. */
int pl_mg_set_comm(pl_mg* s, void* comm, int rank, int world);
/* The obs trajectory [(e*T + t)*D + j]: host f64 (copied to the device as fp32), or a device fp32
 * buffer the caller owns and keeps alive (the rollout's resident trajectory, g_dMGObsTraj in the
 * reference, ffi/puffercuda.cu:2130-2150). */
int pl_mg_set_obs(pl_mg* s, const double* obs, size_t D);
int pl_mg_set_obs_dev(pl_mg* s, const float* traj, size_t D);
/* Replaces lean_cuda_mg_vtrace (ffi/puffercuda.cu:389-399): MinGRU-form V-trace of the columns with the
 * live ratio/value buffers (f64, bit-exact), sum |adv| per segment copied to advL1 (host, N). */
int pl_mg_vtrace(pl_mg* s, double gamma, double lam, double rhoClip, double cClip, double* advL1, void* stream);
/* Replaces lean_cuda_mg_vtrace_prio (ffi/puffercuda.cu:443-470): the same V-trace, then prioritised
 * sampling of mbSegs segments on the device; the sample stays resident for pl_mg_grad. */
int pl_mg_vtrace_prio(pl_mg* s, double gamma, double lam, double rhoClip, double cClip, size_t mbSegs,
                      double prioAlpha, double annealBeta, uint64_t rng, void* stream);
/* Replaces the device-column mode of lean_cuda_mingru_ppo_grad: gathers the sampled minibatch (segIdx
 * and mbPrio host arrays of Bmb entries, or both NULL for the sample pl_mg_vtrace_prio left), runs the
 * BPTT gradient with the weights of `handle` (a pl_policy_load handle; 0 = the host `params` instead),
 * leaves the summed gradient resident, and iterates value/ratio of the sampled segments (the last
 * sampler of a segment writes). */
int pl_mg_grad(pl_mg* s, const pl_mg_net* net, size_t handle, const double* params, const double* segIdx,
               const double* mbPrio, size_t Bmb, double vfCoef, double entCoef, double clipEps, double vfClip,
               uint8_t bf16, void* stream);
/* Copies the last resident gradient (P) and, when non-NULL, the minibatch's new log-prob / value
 * (T*Bmb each, time-major) to host f64. */
int pl_mg_grad_download(pl_mg* s, double* grad, double* newlp, double* newval);
/* Replaces lean_cuda_mingru_muon_resident (ffi/puffercuda.cu:5727-5976): clips the resident gradient
 * (gClip == NULL; gnorm of g*gscale, Puffer/RL/MinGRUTrain.lean:640-648) or takes an already clipped
 * host gradient gClip (P), then one Muon step of every matrix and bias of `handle` in place.
 * coeffs: the Newton-Schulz table (iters rows of a, b, c; NULL = the reference's 5-row table). */
int pl_mg_muon(pl_mg* s, const pl_mg_net* net, size_t handle, const double* gClip, double lr, double wd, double mu,
               double eps, double maxGradNorm, double gscale, const double* coeffs, size_t iters, uint8_t bf16,
               void* stream);
/* Copies value, ratio and the last V-trace advantages (N*T each, may be NULL) to host f64. */
int pl_mg_read_state(pl_mg* s, double* value, double* ratio, double* adv);
typedef struct {
  double gamma, lam, rhoClip, cClip, prioAlpha, annealBeta;
  double wd, mu, eps, vfCoef, entCoef, clipEps, vfClip, maxGradNorm;
  const double* ns_coeffs; /* NULL: the reference table */
  size_t ns_iters;
  uint8_t bf16;
} pl_mg_hyper;
/* One whole update (the minibatch loop of Puffer/RL/MinGRUTrain.lean:800-850): numMB x {V-trace +
 * prioritised sampling of mbSegs segments, BPTT gradient, iterate, clip, Muon}; *rng advances by
 * mbSegs * 0x9E3779B97F4A7C15 per minibatch. */
int pl_mg_update(pl_mg* s, const pl_mg_net* net, size_t handle, const pl_mg_hyper* h, size_t numMB, size_t mbSegs,
                 uint64_t* rng, double lr, void* stream);
uint64_t pl_mg_last_launches(const pl_mg* s);
int pl_mg_destroy(pl_mg* s);

/* ------------------------------------------------------------------ wide action heads --------- */
/* The resident update of the multi-discrete and continuous plugin trainers (one hidden ReLU layer, O
 * outputs): mode 1 = W categorical heads of sizes head_sizes[0..W) (O = sum + 1; joint log-prob, one
 * clip on the joint ratio), mode 2 = W Gaussian dims (O = 2W + 1: means, raw log-stds clamped to
 * [-20, 2], value). acts is NT x W row-major. Replaces lean_cuda_train_update_wide_resident
 * (ffi/puffercuda.cu:1307-1409; heads k_ppo_dout_md :706-727 and k_ppo_dout_cont :1767-1790). */
int pl_train_update_wide_resident(size_t handle, const double* obs, const double* acts, const double* adv,
                                  const double* ret, const double* olp, const double* oldVal, size_t oldValN,
                                  const double* perm, const double* head_sizes, size_t NT, size_t D, size_t H,
                                  size_t O, size_t W, uint32_t mode, size_t epochs, size_t numMB, double lr, double wd,
                                  double mu, double eps, double vfCoef, double entCoef, double clipEps, double vfClip,
                                  double maxGradNorm, uint8_t bf16, double* params0_out);
/* The summed objective gradient of those heads over N rows (no advantage normalisation), as the
 * verify modes check it (the Gaussian form is the reference's lean_ffi_gauss_ppo_grad_batch_vclip,
 * ffi/pufferffi.c:311-360, on the device; oldVal NULL = unclipped value loss). */
int pl_mlp_ppo_grad_wide(const double* params, const double* obs, const double* acts, const double* advs,
                         const double* rets, const double* oldlps, const double* oldVal, size_t N, size_t H, size_t D,
                         size_t O, size_t W, uint32_t mode, const double* head_sizes, double vfCoef, double entCoef,
                         double clipEps, double vfClip, uint8_t bf16, double* g);
/* In-place Muon step of a resident one-hidden-layer policy [W1|b1|W2|b2] from a raw summed gradient
 * (host, P values) scaled by gscale; f64, the reference's table. params_out (may be NULL) receives the
 * new weights. Replaces lean_cuda_muon_step_mlp_resident (ffi/puffercuda.cu:5985-6020). */
int pl_muon_step_mlp_resident(size_t handle, const double* gRaw, size_t H, size_t D, size_t O, double gscale,
                              double lr, double wd, double mu, double eps, double* params_out);
/* Session form: switch a pl_update session to wide heads before pl_update_set_columns (whose acts
 * column is then NT x W; the _dev form takes it as f64 on the device). mode 0 restores one categorical
 * head. */
int pl_update_set_head(pl_update* u, int mode, size_t W, const double* head_sizes);

/* ------------------------------------------------------------------ LSTM (recurrent) path ------- */
/* Batched LSTM + PPO truncated-BPTT gradient: B sequences packed time-major (obs [(t*B + b)*D + d],
 * acts / advs / rets / oldlps / terms [t*B + b], h0s / c0s [b*H + j], the detached initial states);
 * params [Wx(4H x D) | Wh(4H x H) | bih(4H) | Wo(O x H) | bo(O)], O = A + 1, gate rows i, f, g, o; a
 * terminal at step t zeroes the state before step t + 1 and stops the gradient. g[P] = the summed ascent
 * gradient; newlp / newval (may be NULL) the T*B new log-probs and values. tier 0: f64 arithmetic (the
 * reference's f64 BLAS path), 1: f32 (its production tier), 2: its bf16 tier (computed as tier 1 here).
 * H <= 1024. Replaces lean_ffi_lstm_ppo_grad_batch_blas / _f32 / _bf16 (ffi/pufferblas.c:897-1246, device
 * twin ffi/puffercuda.cu:6794-7182). */
int pl_lstm_ppo_grad_batch(const double* params, const double* obs, const double* acts, const double* advs,
                           const double* rets, const double* oldlps, const double* terms, const double* h0s,
                           const double* c0s, size_t B, size_t T, size_t H, size_t D, size_t A, double vfCoef,
                           double entCoef, double clipEps, int tier, double* g, double* newlp, double* newval);
/* on != 0: the next calls reuse the device copies of the previous call's inputs (all but params); the
 * trainer's epochs > 0 of one update. Replaces lean_cuda_lstm_reuse_inputs (ffi/puffercuda.cu:344). */
int pl_lstm_reuse_inputs(int on);
/* Host: per-segment GAE with bootstrap, then advantages normalised over all N*T; time-major [t*N + n];
 * out = [adv(N*T); ret(N*T)]. Bit-exact twin of lean_ffi_lstm_gae_boot_norm (ffi/pufferffi.c:975-1010). */
int pl_lstm_gae_boot_norm(const double* vals, const double* rews, const double* terms, const double* bootV,
                          size_t N, size_t T, double gamma, double lam, double* out);

/* ------------------------------------------------------------------ checkpoints --------------- */
/* The reference's checkpoint file (Puffer/RL/FFITrain.lean:55-90, ckptToBytes / bytesToCkpt): a
 * little-endian u64 parameter count P, then the P weights as little-endian IEEE f64 — byte-compatible,
 * so runs resume across implementations. Host only: pl_ckpt_write writes w[0..P) to path;
 * pl_ckpt_read reads at most cap weights into w and sets *P to the count it holds, bounded by the file
 * size as the reference's parser is (a truncated file yields the doubles it contains). */
int pl_ckpt_write(const char* path, const double* w, size_t P);
int pl_ckpt_read(const char* path, double* w, size_t cap, size_t* P);
/* The same through a policy handle: save writes the handle's first P values (the weights); restore
 * creates a handle holding the file's weights and zero momentum (the reference re-zeros it on load,
 * Puffer/RL/MinGRUTrain.lean:684-700). */
int pl_policy_save(size_t handle, size_t P, const char* path);
int pl_policy_restore(const char* path, size_t* P, size_t* handle);

/* ------------------------------------------------------------------ dashboard losses ----------- */
/* The reference's 7-loss channel [policy, value, entropy, total, old_kl, kl, clipfrac]
 * (ffi/puffercuda.cu:251-262, 336-352). */
int pl_loss_enable(uint8_t on);
int pl_read_losses(double out[7]);

#ifdef __cplusplus
}
#endif
#endif
