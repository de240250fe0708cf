// Newton-Schulz orthogonalisation on the tensor cores (bf16 operands, fp32 accumulate).
//
// For a wide matrix X (m x n, m <= n; tall matrices are transposed on the way in and out), one
// quintic step with coefficients (a, b, c) is three tcgen05 GEMMs:
//     G  = X X^T                          (m x m, both operands K-major)
//     Bm = b G + c G G                    (G is symmetric, so G's rows serve as its columns)
//     X' = a X + Bm X                     (X read MN-major where it lies)
// which is the reference's a X + b (A X) + c A (A X) (Puffer/Float/Muon.lean:74-90) regrouped as
// (a I + b A + c A^2) X: 4 m^2 n + 2 m^3 flops per step instead of 6 m^2 n. The fused epilogues
// do the axpby; the last step writes fp32 for the finalise.
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
                   long xbs, float* out_f32, long ld_out, long obs, cudaStream_t st) {
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
    // Bm = b G + c G G
    e.out = w.B;
    e.alpha = c;
    e.beta = b;
    e.aux = w.G;
    e.ld_aux = w.ldg;
    e.aux_bstride = gbs;
    rc = gemm_launch(pick_bn(m), EPI_BF16, false, false, opG, opG, m, m, m, batch, e, st);
    if (rc) return rc;
    // X' = a X + Bm X
    EpiArgs u{};
    u.err = w.err;
    u.ldo = ldx;
    u.out_bstride = xbs_eff;
    u.out_rows = m;
    u.out_cols = n;
    u.alpha = 1.f;
    u.beta = a;
    u.aux = cur;
    u.ld_aux = ldx;
    u.aux_bstride = xbs_eff;
    const bool last = (it + 1 == iters);
    if (last && out_f32) {
      u.out = out_f32;
      u.ldo = ld_out;
      u.out_bstride = batch > 1 ? obs : (long)ld_out * m;
      rc = gemm_launch(pick_bn(n), EPI_F32, false, true, opB, opX, m, n, m, batch, u, st);
      if (rc) return rc;
    } else {
      u.out = nxt;
      rc = gemm_launch(pick_bn(n), EPI_BF16, false, true, opB, opX, m, n, m, batch, u, st);
      if (rc) return rc;
      std::swap(cur, nxt);
    }
  }
  if (!out_f32 && cur != X) {
    // result must end where it started
    PL_CUDA(cudaMemcpy2DAsync(X, ldx * 2, cur, ldx * 2, (size_t)n * 2, (size_t)m * batch, cudaMemcpyDeviceToDevice, st));
  }
  return PL_OK;
}

// ---------------------------------------------------------------- batched public entry
// per-matrix X <- X / (||X||_F + eps), fixed-order block reduction, in place (bf16)
__global__ void __launch_bounds__(256) ns_batch_normalize_kernel(__nv_bfloat16* X, long per, long bs, double eps) {
  __shared__ double sh[256];
  __nv_bfloat16* x = X + (long)blockIdx.x * bs;
  double s = 0.0;
  for (long i = threadIdx.x; i < per; i += 256) {
    const double v = (double)__bfloat162float(x[i]);
    s += v * v;
  }
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int k = 128; k > 0; k >>= 1) {
    if ((int)threadIdx.x < k) sh[threadIdx.x] += sh[threadIdx.x + k];
    __syncthreads();
  }
  const float inv = (float)(1.0 / (sqrt(sh[0]) + eps));
  for (long i = threadIdx.x; i < per; i += 256) x[i] = __float2bfloat16_rn(__bfloat162float(x[i]) * inv);
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

int launch_ns_normalize(__nv_bfloat16* X, long batch, long per, double eps, cudaStream_t st) {
  ns_batch_normalize_kernel<<<(unsigned)batch, 256, 0, st>>>(X, per, per, eps);
  count_launch();
  PL_LAUNCH("ns_batch_normalize_kernel");
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
  if (!w.X0 || !w.X1 || !w.G || !w.B) return PL_ERR_NOMEM;
  if (tall) {
    dim3 grid((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32), (unsigned)batch);
    transpose_bf16_kernel<<<grid, dim3(32, 8), 0, st>>>(X, (int)rows, (int)cols, w.X0);
  } else {
    PL_CUDA(cudaMemcpyAsync(w.X0, X, xbytes, cudaMemcpyDeviceToDevice, st));
  }
  ns_batch_normalize_kernel<<<(unsigned)batch, 256, 0, st>>>(w.X0, per, per, eps);
  count_launch(2);
  PL_LAUNCH("ns_batch_normalize_kernel");
  int rc = ns_run_batched(m, n, (int)batch, coeffs, (int)iters, w, w.X0, n, per, nullptr, 0, 0, st);
  if (rc) return rc;
  if (tall) {
    dim3 grid((unsigned)ceil_div(rows, 32), (unsigned)ceil_div(cols, 32), (unsigned)batch);
    transpose_bf16_kernel<<<grid, dim3(32, 8), 0, st>>>(w.X0, (int)cols, (int)rows, X);
    count_launch();
    PL_LAUNCH("transpose_bf16_kernel");
  } else {
    PL_CUDA(cudaMemcpyAsync(X, w.X0, xbytes, cudaMemcpyDeviceToDevice, st));
  }
  return PL_OK;
}
