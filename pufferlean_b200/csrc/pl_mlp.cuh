// The MLP PPO+Muon update session: device layout of the rollout columns, the per-minibatch
// activations and the optimizer state, and the launchers of the memory-bound kernels.
#pragma once
#include <vector>

#include "pl_common.cuh"

namespace pl {

// One linear layer of the flat parameter vector: W at params[oW] (out x in, row-major), b at
// params[ob] (out). Padded extents (in_p, out_p: multiples of 64) size the bf16 shadow copies.
struct Layer {
  int in, out, in_p, out_p;
  size_t oW, ob;
};

// Newton-Schulz workspace of the largest matrix (wide layout: m = min(rows,cols) rows of
// n = max(rows,cols) contiguous values).
struct NsWork {
  __nv_bfloat16 *X0 = nullptr, *X1 = nullptr, *G = nullptr, *B = nullptr;
  float* Xf = nullptr;
  double* U = nullptr;
  double* part = nullptr;
  long ldx = 0, ldg = 0;
  unsigned* err = nullptr;  // bounded-wait error word for the GEMMs (NULL = the per-device default)
  unsigned* cnt = nullptr;  // ns_chain_counter_words(batch) words: enables the persistent chain kernel
};

// 0 = every batch takes the per-step GEMM chain, 1 = matrices with m, n <= 128 run fused in one CTA
// each (default); a negative mode only queries. Returns the previous mode.
int ns_set_small_mode(int mode);
// 0 = every batch takes the per-step GEMM launches, 1 = batches with m > 128 run as one persistent
// cooperative launch when the workspace has counters (default); a negative mode only queries.
int ns_set_chain_mode(int mode);
int ns_set_chain_capture(int mode);
long ns_chain_counter_words(long batch);
// One group of same-shape wide matrices for the persistent chain: iterate 0 is X, later iterates
// alternate between xbuf[1] and xbuf[0]; G / B the m x m workspaces; the last step writes out_f32,
// final_bf16 or xbuf[iters & 1]; scale0 (optional) is the first step's per-matrix factor; cnt holds
// 3 * batch zeroed counters.
struct NsChainGroupHost {
  int m, n, batch;
  __nv_bfloat16 *X, *xbuf[2];
  long ldx, xbs;
  __nv_bfloat16 *G, *B;
  long ldg;
  float* out_f32;
  long ld_out, obs;
  __nv_bfloat16* final_bf16;
  float* scale0;
  double fold_eps;  // >= 0: scale0 is written by the first step (see ns_run_batched)
  unsigned* cnt;
};
// Up to kNsChainMaxGroups groups in one persistent cooperative launch (sets *used; nothing is launched
// when a group cannot take the chain, the stream is being captured or the chain is switched off).
// abort_word: one zeroed word.
constexpr int kNsChainMaxGroups = 4;
int ns_chain_launch(int ngroups, const NsChainGroupHost* groups, const double* coeffs, int iters,
                    unsigned* abort_word, unsigned* err, cudaStream_t st, bool* used);
// Runs the whole chain as one persistent launch when eligible (sets *used); the result then lies in
// *result (the final bf16 buffer, or the iterate buffer that holds it; NULL for fp32 output).
int ns_chain_try(int m, int n, int batch, const double* coeffs, int iters, NsWork& w, __nv_bfloat16* X, long ldx,
                 long xbs, __nv_bfloat16* const xbuf[2], float* out_f32, long ld_out, long obs,
                 __nv_bfloat16* final_bf16, float* scale0, cudaStream_t st, __nv_bfloat16** result, bool* used,
                 double fold_eps = -1.0);
// final_bf16 (optional): the last step's bf16 output goes there (not an iterate buffer) instead of
// back into X; result_at (optional): receives the iterate buffer that holds the bf16 result, and X
// is then left as it is. Iterate 0 is X; iterate s >= 1 lives in w.X0 / w.X1 (X itself when X is one
// of them). scale0 (optional; not for batches the fused short-matrix kernel takes, see
// ns_small_eligible): X is not yet normalised, and scale0[b] (with scale0[b]^2 at
// scale0[batch + b]) is the per-matrix factor the first step's G and X' epilogues apply; final_bf16
// may then be X itself (X is read by the first step only; iters >= 2). With fold_eps >= 0 scale0 is
// an output instead: the first step's G is X X^T of the raw X, and its polynomial's epilogue takes
// s = 1 / (sqrt(trace G) + fold_eps) from G's diagonal, applies s^2 and s^4 there and writes s to
// scale0[b] for the first X' (no separate normalisation pass over X).
int ns_run_batched(int m, int n, int batch, const double* coeffs, int iters, NsWork& w, __nv_bfloat16* X, long ldx,
                   long xbs, float* out_f32, long ld_out, long obs, cudaStream_t st,
                   __nv_bfloat16* final_bf16 = nullptr, __nv_bfloat16** result_at = nullptr,
                   float* scale0 = nullptr, double fold_eps = -1.0);
// True when ns_run_batched takes the fused one-CTA kernel for this batch (which normalises in the kernel
// when given fold_eps >= 0 and no scale0).
bool ns_small_eligible(int m, int n, int batch, int iters);
// Per-matrix 1 / (||X||_F + eps) and its square into scale[0, batch) and scale[batch, 2 batch): the
// sum-of-squares pass of launch_ns_prepare without the scaled copy.
int launch_ns_scale_factors(const __nv_bfloat16* X, long batch, int rows, int cols, double eps, double* part,
                            float* scale, cudaStream_t st);
// Normalised wide-layout copy of a batch of row-major bf16 matrices (pl_ns.cu).
long ns_prepare_parts(long per);
int launch_ns_prepare(const __nv_bfloat16* X, long batch, int rows, int cols, double eps, double* part,
                      __nv_bfloat16* dst, cudaStream_t st);
int ns_run(int m, int n, const double* coeffs, int iters, NsWork& w, __nv_bfloat16* X, long ldx, float* out_f32,
           long ld_out, cudaStream_t st);

// The shared 7-loss dashboard channel (pl_mlp_update.cu).
bool loss_channel_on();
void loss_channel_store(const double v[7]);

// launchers (pl_mlp_kernels.cu)
int launch_obs_to_bf16_f64(const double* src, long NT, int D, int Dp, __nv_bfloat16* dst, cudaStream_t st);
int launch_obs_to_bf16_f32(const float* src, long NT, int D, int Dp, __nv_bfloat16* dst, cudaStream_t st);
int launch_obs_to_f32_f64(const double* src, long n, float* dst, cudaStream_t st);
int launch_columns(const double* act, const double* ret, const double* olp, const double* ov, long NT, int* act_i,
                   float* ret_f, float* olp_f, float* ov_f, cudaStream_t st);
int launch_perm(const double* perm, long n, int* out, cudaStream_t st);
// For observations stored in the first epoch's order: pos = inverse of perm[0, NT) (scratch, NT ints)
// and out[i] = pos[perm[i]] for i < n, each row id translated into its first-epoch position.
int launch_perm_positions(const int* perm, long NT, long n, int* pos, int* out, cudaStream_t st);
int launch_gather(bool bf16, const int* idx, int Nmb, const void* obs, int rowElems, void* X, const int* act_c,
                  const double* adv_c, const float* ret_c, const float* olp_c, const float* ov_c, int* mb_act,
                  float* mb_adv, float* mb_ret, float* mb_olp, float* mb_ov, double* part, double* ms,
                  cudaStream_t st, double* sums = nullptr, const int* oidx = nullptr);
int launch_adv_ms_from_sums(const double* sums, double* ms, cudaStream_t st);
// Column sums of `tiles` rows of ld floats in `part`; part must have colsum_scratch_elems(tiles, ld)
// floats (the second reduction level lives after the partials).
// rollout-side column producer (pl_columns.cu)
int launch_stamp_rows_f64(double* col, long width, long T, long step, long e0, long ne, const double* src,
                          cudaStream_t st);
int launch_stamp_rows_f32(float* col, long width, long T, long step, long e0, long ne, const float* src,
                          cudaStream_t st);
int launch_stamp_plane(double* col, long N, long T, const double* plane, cudaStream_t st);
long colsum_scratch_elems(int tiles, long ld);
int launch_colsum_reduce(const float* part, int tiles, long ld, int ncols, float* out, cudaStream_t st);
int launch_splitk_reduce(const float* part, int S, long n, float* out, cudaStream_t st);
int launch_gradnorm(const float* g, long P, double sc, double maxNorm, double* part, double* cc, cudaStream_t st);
int launch_nesterov(const float* g, const double* cc, double* mom, double* u, double mu, long n, double* part,
                    int* nparts, cudaStream_t st);
int launch_ns_input(const double* u, const double* part, int nparts, int rows, int cols, double eps,
                    __nv_bfloat16* X, long ldx, cudaStream_t st);
int launch_ns_finalize(const float* Xf, long ldx, int rows, int cols, double c1, double c2, double* W,
                       __nv_bfloat16* Wb, long ldw, cudaStream_t st);
// Muon around Newton-Schulz for one group of equal-shape layers of the bf16 tier, one launch per phase
// (blockIdx.y = layer of the group). X and Xf are the wide layout (min(rows, cols) x max(rows, cols),
// ld ldx; transposed when rows > cols).
constexpr int kMuonGroupMax = 8;
struct MuonGroupArgs {
  int nb = 0, rows = 0, cols = 0;  // layers in this launch; each weight is rows x cols (row-major)
  long ldx = 0;                    // leading dimension of X and Xf
  long ldw = 0;                    // leading dimension of the bf16 shadow weights
  const float* gW[kMuonGroupMax];  // weight gradient
  double* mW[kMuonGroupMax];       // weight momentum (f64)
  __nv_bfloat16* X[kMuonGroupMax]; // Newton-Schulz input; NULL: this rank does not orthogonalise the layer
  const float* Xf[kMuonGroupMax];  // Newton-Schulz result (fp32)
  double* W[kMuonGroupMax];        // f64 master weights
  __nv_bfloat16* Wb[kMuonGroupMax];  // bf16 shadow weights (NULL: none)
  const float* gb[kMuonGroupMax];  // bias gradient (rows values)
  double* b[kMuonGroupMax];        // f64 bias
  double* mb[kMuonGroupMax];       // bias momentum
  float* bf[kMuonGroupMax];        // fp32 bias shadow (NULL: none)
};
// Blocks per layer of the group launches: a function of the shape and the whole group's size only, so
// that the partial sums (and the scale folded from them) do not depend on how the group is chunked;
// nb_total times it is at most max(kMuonBlocksMax, nb_total).
constexpr int kMuonBlocksMax = 1184;  // 8 x 148 SMs
int muon_group_blocks(int rows, int cols, int nb_total);
// Nesterov momentum of each weight (m <- mu m + g cc, u = g cc + mu m, f64 as nesterov_kernel) and
// X = bf16(u) unscaled; with part non-NULL, per-block sums of u^2 into part[q * blocks + block].
int launch_muon_x0(const MuonGroupArgs& a, int blocks, const double* cc, double mu, double* part, cudaStream_t st);
// scale[q] = 1 / (sqrt(sum of layer q's partials) + eps) and scale[nb + q] = its square: the first
// Newton-Schulz step's factors for an unnormalised input (ns_run_batched's scale0).
int launch_muon_scale(const double* part, int blocks, int nb, double eps, float* scale, cudaStream_t st);
// W <- (1 - lr wd) W + lr s Xf with the bf16 shadow, and the bias step (Nesterov on the bias gradient
// times cc, same operation order as the f64 reference) with its fp32 shadow.
int launch_muon_finalize(const MuonGroupArgs& a, int blocks, double lr, double wd, double mu, double s,
                         const double* cc, cudaStream_t st);
int launch_w_to_bf16(const double* W, int rows, int cols, __nv_bfloat16* Wb, long ldw, cudaStream_t st);
int launch_f64_to_f32(const double* s, long n, float* d, cudaStream_t st);
int launch_f32_to_f64(const float* s, long n, double* d, cudaStream_t st);
int launch_sgemm(int M, int N, int K, const float* A, long ars, long acs, const float* B, long brs, long bcs, float* C,
                 long ldc, float alpha, cudaStream_t st);
int launch_sgemm_splitk(int M, int N, int K, const float* A, long ars, long acs, const float* B, long brs, long bcs,
                        float* C, long ldc, float* ws, long ws_elems, cudaStream_t st);
// Z = A W^T + b (A: M x K rows of lda floats, W: N x K dense), H = act(Z); both M x N dense.
int launch_sgemm_bias_act(int M, int N, int K, const float* A, long lda, const float* W, const float* b, float* Z,
                          float* H, int act, cudaStream_t st);
// dH = (dZ W) * act'(Z) (dZ: M x K rows of lda floats, W: K x N dense, Z and dH: M x N dense).
int launch_sgemm_act_grad(int M, int N, int K, const float* A, long lda, const float* W, const float* Z, float* dH,
                          int act, cudaStream_t st);
// Out = H W^T + b for O <= 8 outputs and K <= 1024 (a multiple of 4): one warp per row.
bool skinny_rows_ok(int K, int O);
int launch_skinny_rows(const float* H, int rows, int K, const float* W, const float* b, int O, float* Out,
                       cudaStream_t st);
// Weight and bias gradient of one layer: dW[out x in] = dZ^T Hin, db[out] = column sums of dZ (dZ: K rows of
// ldz floats, Hin: K rows of ldh floats), split over K into ws (splitk_wb_elems floats) and summed in a
// fixed order.
long splitk_wb_elems(int K, int out, int in);
int launch_wgrad_bias_f32(int out, int in, int K, const float* dZ, long ldz, const float* Hin, long ldh, float* dW,
                          float* db, float* ws, long ws_elems, cudaStream_t st);
int launch_bias_act_f32(float* Z, float* H, const float* b, long M, int N, int act, cudaStream_t st);
int launch_act_grad_f32(float* dH, const float* Z, long n, int act, cudaStream_t st);
int launch_ppo_rows_f32(const float* Out, int M, int A, const int* act, const float* adv, const double* ms,
                        const float* ret, const float* olp, const float* ov, float vf, float ent, float clip,
                        float vfclip, float* dOut, float* newlp, float* newval, cudaStream_t st);
int launch_colsum_f32(const float* Mx, long rows, int N, float* out, float* ws, long ws_elems, cudaStream_t st);
// Wide action heads (multi-discrete mode 1, Gaussian mode 2): per-row PPO objective gradient,
// per-128-row column sums (colpart) and loss sums (loss_part); see pl_mlp_kernels.cu.
int launch_ppo_rows_wide(bool bf16_out, const float* Out, int ldo, const float* bias, int M, int O, int ldd, int mode,
                        int W, const int* hs, const float* actw, const float* adv, const double* ms, const float* ret,
                        const float* olp, const float* ov, float vf, float ent, float clip, float vfclip, float lslo,
                        float lshi, void* dOut, float* colpart, float* loss_part, cudaStream_t st);
int launch_gather_rows_f32(const int* idx, int Nmb, const float* src, int W, float* dst, cudaStream_t st);
int launch_f64_to_f32_rows(const double* s, long n, float* d, cudaStream_t st);

}  // namespace pl
