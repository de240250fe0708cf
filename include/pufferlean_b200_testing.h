/* Test hooks of pufferlean_b200: direct access to the tcgen05 GEMM and its epilogues on device
 * pointers, so kernel numerics can be checked against a plain fp32 reference. Not part of the
 * reference's interface; no reference counterpart. */
#ifndef PUFFERLEAN_B200_TESTING_H
#define PUFFERLEAN_B200_TESTING_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  /* operands: bf16 device storage, rows x cols with cols contiguous, leading dimension ld */
  const void* a; long a_rows, a_cols, a_ld, a_bstride; int a_mn;
  const void* b; long b_rows, b_cols, b_ld, b_bstride; int b_mn;
  int M, N, K, bn, epi, batch, k_splits;
  /* epilogue (see pl_gemm.cuh EpiArgs) */
  void* out; long ldo, out_bstride; int out_rows, out_cols;
  float alpha, beta;
  const void* aux; long ld_aux, aux_bstride;
  const float* bias;
  void* out2; long ldo2;
  float* colsum; long ld_colsum;
  int act;
  const int* act_idx; const float* adv; const float* ret; const float* olp; const float* ov;
  int A; float vf, ent, clip, vfclip;
  float* newlp; float* newval; float* loss_part;
} pl_test_gemm_args;

int pl_test_gemm(const pl_test_gemm_args* g, void* stream);
/* Selects the GEMM's tile mode for every later launch in this process: 0 = single-CTA tiles only,
 * 1 = CTA pairs (cta_group::2, 256-row tiles) where eligible, 2 = CTA pairs for products whose two
 * operands are MN-major (the weight gradients) only (the default); a negative mode only queries.
 * Returns the previous mode. */
int pl_test_gemm_pair_mode(int mode);
/* Newton-Schulz for matrices with both sides <= 128: 1 = one fused CTA per matrix (the default),
 * 0 = the per-step GEMM chain; a negative mode only queries. Returns the previous mode. */
int pl_test_ns_small_mode(int mode);
/* Newton-Schulz for batches with m = min(rows, cols) > 128: 1 = all steps in one persistent
 * cooperative launch (the default; see pl_test_ns_chain_capture for stream capture), 0 = three GEMM
 * launches per step; a negative mode only queries. Returns the previous mode. */
int pl_test_ns_chain_mode(int mode);
/* While a stream is being captured into a CUDA graph: 1 = the persistent Newton-Schulz chain is recorded
 * as a cooperative kernel node (the default), 0 = the per-step GEMM launches are recorded instead; a
 * negative mode only queries. Returns the previous mode. */
int pl_test_ns_chain_capture(int mode);
/* Host observations in the bf16 tier: 1 = rounded to bf16 on the host threads, a quarter of the bytes
 * copied (the default), 0 = f64 rows copied and converted on the device; a negative mode only
 * queries. Returns the previous mode. */
int pl_test_host_bf16(int mode);
/* The host rounding itself: rows x D f64 values -> Dp-wide bf16 rows (bits), zero padded. */
int pl_test_round_rows_bf16(const double* src, long rows, int D, int Dp, uint16_t* dst);
/* The gather of minibatch (epoch, mb) of an update session, exactly as pl_update_run runs it before
 * that minibatch's forward pass (same row range, same shuffle translation, same kernel), with its
 * outputs copied to the host: rows = Nmb x row_elems observation values (f32 in the tight tier; bf16
 * bits in the bf16 tier, row_elems = D rounded up to 64, zero padded), act (int32), adv, ret, olp and
 * ov (f32; ov only when the session clips values). *nmb receives Nmb (0 for an empty minibatch). Any
 * output pointer may be NULL. Under data parallelism every rank must call it (it all-reduces the
 * advantage statistics as the update does). */
struct pl_update;
int pl_test_update_gather(struct pl_update* u, size_t epoch, size_t mb, void* rows, size_t* row_elems, int* act,
                          float* adv, float* ret, float* olp, float* ov, size_t* nmb, void* stream);
/* Data-parallel sessions created afterwards: 1 = the gradient all-reduced per layer on a second stream
 * while the backward pass continues (the default), 0 = one all-reduce of the whole gradient after the
 * backward pass; a negative mode only queries. Returns the previous mode. */
int pl_test_dp_overlap(int mode);
/* Tight-tier (f64 Muon) sessions created afterwards: 1 = the Muon step of layers small enough for one CTA
 * each runs as one launch (the default), 0 = one launch sequence per matrix and bias; a negative mode
 * only queries. Returns the previous mode. */
int pl_test_exact_group(int mode);
/* bf16-tier update: 1 = the Newton-Schulz chains of all equal-shape layer groups run in one persistent
 * launch per Muon step (the default), 0 = one launch per group; a negative mode only queries. Returns the
 * previous mode. */
int pl_test_ns_group_launch(int mode);
/* LSTM recurrences: 1 = four threads per unit where a sequence's 4H threads fit a CTA and Wh fits
 * shared memory (the default), 0 = one thread per unit; a negative mode only queries. Returns the
 * previous mode. */
int pl_test_lstm_quad(int mode);
/* Replaces NCCL and the stream query used by pl_comm_* with host-side fakes, for failure tests without a
 * GPU: 1 = creation never completes (a peer that never joins), 2 = a peer fails once the communicator
 * is up (asynchronous-error queries report it), 3 = enqueued work never completes, 4 = a healthy
 * communicator; 0 = the real library. A negative mode only queries. Returns the previous mode. */
int pl_test_comm_fake(int mode);
/* Number of communicator aborts the fakes have received. */
int pl_test_comm_fake_aborts(void);
/* Reads and clears the device-side bounded-wait error word (0 = none). */
int pl_test_device_error(unsigned* code);

#ifdef __cplusplus
}
#endif
#endif
