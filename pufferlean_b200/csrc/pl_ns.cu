// Newton-Schulz orthogonalisation on the tensor cores (bf16 operands, fp32 accumulate).
//
// For a wide matrix X (m x n, m <= n; tall matrices are transposed on the way in and out), one
// quintic step with coefficients (a, b, c) is three tcgen05 GEMMs:
//     G  = X X^T                          (m x m, both operands K-major)
//     Bm = b G + c G G                    (G is symmetric, so G's rows serve as its columns)
//     X' = a X + Bm X                     (X read MN-major where it lies)
// which is the reference's a X + b (A X) + c A (A X) (Puffer/Float/Muon.lean:74-90) regrouped as
// (a I + b A + c A^2) X: 4 m^2 n + 2 m^3 flops per step instead of 6 m^2 n. The second GEMM's
// epilogue forms the whole polynomial Pm = a I + b G + c G G (a on the diagonal), so the third is
// a plain product X' = Pm X with no second read of X. The last step writes fp32 for the finalise,
// or bf16 straight into the caller's buffer.
#include <vector>

#include "pl_gemm.cuh"
#include "pl_mlp.cuh"
#include "pl_runtime.h"

namespace pl {

static inline int pick_bn(int N) { return N <= 128 ? 128 : 256; }

int ns_run(int m, int n, const double* coeffs, int iters, NsWork& w, __nv_bfloat16* X, long ldx, float* out_f32,
           long ld_out, cudaStream_t st) {
  return ns_run_batched(m, n, 1, coeffs, iters, w, X, ldx, 0, out_f32, ld_out, 0, st);
}

int ns_run_batched(int m, int n, int batch, const double* coeffs, int iters, NsWork& w, __nv_bfloat16* X, long ldx,
                   long xbs, float* out_f32, long ld_out, long obs, cudaStream_t st, __nv_bfloat16* final_bf16,
                   __nv_bfloat16** result_at) {
  PL_REQUIRE(!final_bf16 || (final_bf16 != w.X0 && final_bf16 != w.X1 && final_bf16 != X), PL_ERR_INVALID,
             "Newton-Schulz: the final output may not alias the iterates");
  PL_REQUIRE(m <= n, PL_ERR_INVALID, "Newton-Schulz expects the wide layout (m=%d > n=%d)", m, n);
  const long gbs = (long)w.ldg * m;
  __nv_bfloat16* cur = X;
  __nv_bfloat16* nxt = (X == w.X0) ? w.X1 : w.X0;
  const long xbs_eff = batch > 1 ? xbs : (long)ldx * m;
  for (int it = 0; it < iters; it++) {
    const float a = (float)coeffs[3 * it], b = (float)coeffs[3 * it + 1], c = (float)coeffs[3 * it + 2];
    Operand opX{cur, m, n, ldx, batch, xbs_eff};
    Operand opG{w.G, m, m, w.ldg, batch, gbs};
    Operand opB{w.B, m, m, w.ldg, batch, gbs};
    EpiArgs e{};
    e.err = w.err;
    // G = X X^T
    e.out = w.G;
    e.ldo = w.ldg;
    e.out_bstride = gbs;
    e.out_rows = m;
    e.out_cols = m;
    e.alpha = 1.f;
    int rc = gemm_launch(pick_bn(m), EPI_BF16, false, false, opX, opX, m, m, n, batch, e, st);
    if (rc) return rc;
    // Pm = a I + b G + c G G
    e.out = w.B;
    e.alpha = c;
    e.beta = b;
    e.diag = a;
    e.aux = w.G;
    e.ld_aux = w.ldg;
    e.aux_bstride = gbs;
    rc = gemm_launch(pick_bn(m), EPI_BF16, false, false, opG, opG, m, m, m, batch, e, st);
    if (rc) return rc;
    // X' = Pm X
    EpiArgs u{};
    u.err = w.err;
    u.ldo = ldx;
    u.out_bstride = xbs_eff;
    u.out_rows = m;
    u.out_cols = n;
    u.alpha = 1.f;
    const bool last = (it + 1 == iters);
    if (last && out_f32) {
      u.out = out_f32;
      u.ldo = ld_out;
      u.out_bstride = batch > 1 ? obs : (long)ld_out * m;
      rc = gemm_launch(pick_bn(n), EPI_F32, false, true, opB, opX, m, n, m, batch, u, st);
      if (rc) return rc;
    } else {
      u.out = (last && final_bf16) ? final_bf16 : nxt;
      rc = gemm_launch(pick_bn(n), EPI_BF16, false, true, opB, opX, m, n, m, batch, u, st);
      if (rc) return rc;
      if (last && final_bf16) return PL_OK;
      std::swap(cur, nxt);
    }
  }
  if (result_at) {
    *result_at = cur;
    return PL_OK;
  }
  if (!out_f32 && cur != X) {
    // result must end where it started
    PL_CUDA(cudaMemcpy2DAsync(X, ldx * 2, cur, ldx * 2, (size_t)n * 2, (size_t)m * batch, cudaMemcpyDeviceToDevice, st));
  }
  return PL_OK;
}

// ---------------------------------------------------------------- batched public entry
// Per-matrix Frobenius normalisation X / (||X||_F + eps) in two passes: sums of squares of
// fixed 16384-element chunks (f64, fixed order inside each block), then a pass in which every block
// folds its matrix's chunk sums in chunk order and scales its own piece. The result does not depend
// on the launch shape's timing.
constexpr long kNsChunk = 16384;
static inline long ns_chunks(long per) { return (per + kNsChunk - 1) / kNsChunk; }

template <bool VEC>
__global__ void __launch_bounds__(256) ns_sumsq_kernel(const __nv_bfloat16* __restrict__ X, long per,
                                                       double* __restrict__ part) {
  __shared__ double sh[8];
  const long chunks = gridDim.x;
  const __nv_bfloat16* x = X + (long)blockIdx.y * per;
  const long lo = (long)blockIdx.x * kNsChunk, hi = min(per, lo + kNsChunk);
  double s = 0.0;
  if (VEC) {
    for (long i = lo + 8 * (long)threadIdx.x; i < hi; i += 8 * 256) {
      const uint4 q = *reinterpret_cast<const uint4*>(x + i);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
      float f = 0.f;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 v = __bfloat1622float2(h[j]);
        f = fmaf(v.x, v.x, f);
        f = fmaf(v.y, v.y, f);
      }
      s += (double)f;
    }
  } else {
    for (long i = lo + threadIdx.x; i < hi; i += 256) {
      const double v = (double)__bfloat162float(x[i]);
      s += v * v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; w++) t += sh[w];
    part[(long)blockIdx.y * chunks + blockIdx.x] = t;
  }
}
__device__ __forceinline__ float ns_inv_norm(const double* part, long chunks, double eps) {
  double t = 0.0;
  for (long c = 0; c < chunks; c++) t += part[c];
  return (float)(1.0 / (sqrt(t) + eps));
}
// dst = src * inv for the block's chunk (same layout)
template <bool VEC>
__global__ void __launch_bounds__(256) ns_scale_kernel(const __nv_bfloat16* __restrict__ src, long per,
                                                       const double* __restrict__ part, double eps,
                                                       __nv_bfloat16* __restrict__ dst) {
  __shared__ float inv_s;
  const long chunks = gridDim.x;
  if (threadIdx.x == 0) inv_s = ns_inv_norm(part + (long)blockIdx.y * chunks, chunks, eps);
  __syncthreads();
  const float inv = inv_s;
  const long off = (long)blockIdx.y * per;
  const long lo = (long)blockIdx.x * kNsChunk, hi = min(per, lo + kNsChunk);
  if (VEC) {
    for (long i = lo + 8 * (long)threadIdx.x; i < hi; i += 8 * 256) {
      uint4 q = *reinterpret_cast<const uint4*>(src + off + i);
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&q);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float2 v = __bfloat1622float2(h[j]);
        h[j] = __floats2bfloat162_rn(v.x * inv, v.y * inv);
      }
      *reinterpret_cast<uint4*>(dst + off + i) = q;
    }
  } else {
    for (long i = lo + threadIdx.x; i < hi; i += 256) dst[off + i] = __float2bfloat16_rn(__bfloat162float(src[off + i]) * inv);
  }
}
// dst (cols x rows) = src (rows x cols)^T * inv, per matrix
__global__ void transpose_scale_bf16_kernel(const __nv_bfloat16* __restrict__ src, int rows, int cols,
                                            const double* __restrict__ part, long chunks, double eps,
                                            __nv_bfloat16* __restrict__ dst) {
  __shared__ __nv_bfloat16 t[32][33];
  __shared__ float inv_s;
  if (threadIdx.x == 0 && threadIdx.y == 0) inv_s = ns_inv_norm(part + (long)blockIdx.z * chunks, chunks, eps);
  const long bo = (long)blockIdx.z * rows * cols;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[i][threadIdx.x] = src[bo + (long)r * cols + c];
  }
  __syncthreads();
  const float inv = inv_s;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[bo + (long)c * rows + r] = __float2bfloat16_rn(__bfloat162float(t[threadIdx.x][i]) * inv);
  }
}
// batched transpose (rows x cols -> cols x rows), bf16
__global__ void transpose_bf16_kernel(const __nv_bfloat16* __restrict__ src, int rows, int cols, __nv_bfloat16* dst) {
  __shared__ __nv_bfloat16 t[32][33];
  const long bo = (long)blockIdx.z * rows * cols;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[i][threadIdx.x] = src[bo + (long)r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[bo + (long)c * rows + r] = t[threadIdx.x][i];
  }
}

// Normalised wide-layout copy of the caller's batch: dst (m x n per matrix, m <= n) =
// X / (||X||_F + eps), transposed when rows > cols. part holds batch * ns_prepare_parts(rows*cols)
// doubles.
long ns_prepare_parts(long per) { return ns_chunks(per); }
int launch_ns_prepare(const __nv_bfloat16* X, long batch, int rows, int cols, double eps, double* part,
                      __nv_bfloat16* dst, cudaStream_t st) {
  const long per = (long)rows * cols, chunks = ns_chunks(per);
  PL_REQUIRE(batch <= 65535, PL_ERR_UNSUPPORTED, "batched Newton-Schulz: at most 65535 matrices per call");
  const bool vec = (per % 8) == 0 && ((uintptr_t)X % 16) == 0 && ((uintptr_t)dst % 16) == 0;
  dim3 grid((unsigned)chunks, (unsigned)batch);
  if (vec)
    ns_sumsq_kernel<true><<<grid, 256, 0, st>>>(X, per, part);
  else
    ns_sumsq_kernel<false><<<grid, 256, 0, st>>>(X, per, part);
  count_launch();
  PL_LAUNCH("ns_sumsq_kernel");
  if (rows > cols) {
    dim3 tg((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32), (unsigned)batch);
    transpose_scale_bf16_kernel<<<tg, dim3(32, 8), 0, st>>>(X, rows, cols, part, chunks, eps, dst);
    count_launch();
    PL_LAUNCH("transpose_scale_bf16_kernel");
  } else {
    if (vec)
      ns_scale_kernel<true><<<grid, 256, 0, st>>>(X, per, part, eps, dst);
    else
      ns_scale_kernel<false><<<grid, 256, 0, st>>>(X, per, part, eps, dst);
    count_launch();
    PL_LAUNCH("ns_scale_kernel");
  }
  return PL_OK;
}
int launch_transpose_bf16(const __nv_bfloat16* src, long batch, int rows, int cols, __nv_bfloat16* dst,
                          cudaStream_t st) {
  dim3 grid((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32), (unsigned)batch);
  transpose_bf16_kernel<<<grid, dim3(32, 8), 0, st>>>(src, rows, cols, dst);
  count_launch();
  PL_LAUNCH("transpose_bf16_kernel");
  return PL_OK;
}

}  // namespace pl

extern "C" int pl_ns_batched_bf16_dev(void* Xv, size_t batch, size_t rows, size_t cols, double eps,
                                      const double* coeffs, size_t iters, void* stream) {
  using namespace pl;
  if (batch == 0 || rows == 0 || cols == 0) return PL_OK;
  PL_REQUIRE(coeffs && iters > 0 && iters <= 64, PL_ERR_INVALID, "Newton-Schulz needs a coefficient table");
  PL_REQUIRE(rows % 8 == 0 && cols % 8 == 0, PL_ERR_INVALID, "batched NS needs rows and cols multiples of 8");
  cudaStream_t st = (cudaStream_t)stream;
  __nv_bfloat16* X = (__nv_bfloat16*)Xv;
  const int m = (int)(rows < cols ? rows : cols), n = (int)(rows < cols ? cols : rows);
  const bool tall = rows > cols;
  const long per = (long)m * n;
  NsWork w;
  w.ldx = n;
  w.ldg = m;
  const size_t xbytes = (size_t)per * batch * 2, gbytes = (size_t)m * m * batch * 2;
  w.X0 = (__nv_bfloat16*)scratch(10, xbytes);
  w.X1 = (__nv_bfloat16*)scratch(11, xbytes);
  w.G = (__nv_bfloat16*)scratch(12, gbytes);
  w.B = (__nv_bfloat16*)scratch(13, gbytes);
  double* part = (double*)scratch(14, (size_t)batch * ns_prepare_parts(per) * sizeof(double));
  if (!w.X0 || !w.X1 || !w.G || !w.B || !part) return PL_ERR_NOMEM;
  int rc = launch_ns_prepare(X, (long)batch, (int)rows, (int)cols, eps, part, w.X0, st);
  if (rc) return rc;
  // a wide batch ends in the caller's buffer; a tall one in the workspace, transposed back after
  __nv_bfloat16* res = nullptr;
  rc = ns_run_batched(m, n, (int)batch, coeffs, (int)iters, w, w.X0, n, per, nullptr, 0, 0, st, tall ? nullptr : X,
                      &res);
  if (rc) return rc;
  if (tall) {
    dim3 grid((unsigned)ceil_div(rows, 32), (unsigned)ceil_div(cols, 32), (unsigned)batch);
    transpose_bf16_kernel<<<grid, dim3(32, 8), 0, st>>>(res, (int)cols, (int)rows, X);
    count_launch();
    PL_LAUNCH("transpose_bf16_kernel");
  }
  return PL_OK;
}
