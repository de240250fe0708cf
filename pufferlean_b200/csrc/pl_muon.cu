// Muon, tight tier: f64 Nesterov -> Frobenius normalise -> Newton-Schulz -> decoupled decay,
// every arithmetic step rounded on its own (no fused multiply-add) and folded in the order of the
// reference's executable oracle (Puffer/Float/Muon.lean:19-108, whose C twin is
// ffi/pufferblas.c:1369-1406), so the step is bit-identical to it. Used for parity and for the
// bf16 = 0 training tier; the bf16 tier orthogonalises on the tensor cores (pl_ns.cu).
#include "pl_common.cuh"
#include "pl_muon.cuh"
#include "pl_runtime.h"

namespace pl {

__constant__ double c_ns_coeffs[64][3];
constexpr size_t kSmallMuonBytes = 160 * 1024;  // shared memory of the one-CTA exact step

// newMom = mu*mom + g ; upd = g + mu*newMom   (gs scales g first when != 1: g*gs; gs is read from gsp when
// that is not NULL, the device-side clip scale of the update)
__global__ void nesterov_f64_kernel(const double* __restrict__ g, const double* __restrict__ m, double* nm,
                                    double* u, double mu, double gs_val, const double* gsp, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double gs = gsp ? *gsp : gs_val;
  const double gi = gs == 1.0 ? g[i] : __dmul_rn(g[i], gs);
  const double newm = __dadd_rn(__dmul_rn(mu, m[i]), gi);
  nm[i] = newm;
  u[i] = __dadd_rn(gi, __dmul_rn(mu, newm));
}

// Two-level Frobenius fold: per-row sums (one thread per row, sequential in the column), then a
// single thread folds the rows in order; out = 1 / (sqrt(total) + eps).
__global__ void frob_rows_f64_kernel(const double* __restrict__ x, int rows, int cols, double* rowsum) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  const double* r = x + (long)i * cols;
  double s = 0.0;
  for (int j = 0; j < cols; j++) s = __dadd_rn(s, __dmul_rn(r[j], r[j]));
  rowsum[i] = s;
}
__global__ void frob_fold_f64_kernel(const double* __restrict__ rowsum, int rows, double eps, double* inv) {
  if (threadIdx.x || blockIdx.x) return;
  double s = 0.0;
  for (int i = 0; i < rows; i++) s = __dadd_rn(s, rowsum[i]);
  inv[0] = __ddiv_rn(1.0, __dadd_rn(__dsqrt_rn(s), eps));
}
__global__ void scale_f64_kernel(const double* __restrict__ u, const double* __restrict__ inv, double* x, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __dmul_rn(inv[0], u[i]);
}
__global__ void transpose_f64_kernel(const double* __restrict__ X, int rows, int cols, double* Xt) {
  long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)rows * cols) return;
  int i = (int)(idx / cols), j = (int)(idx % cols);
  Xt[(long)j * rows + i] = X[idx];
}
// C[m x n] = A[m x k] B[k x n], s = s + A[i][l]*B[l][j] from 0 (Puffer/Float/Muon.lean:19-31)
__global__ void matmul_f64_kernel(const double* __restrict__ A, const double* __restrict__ B, int m, int k, int n,
                                  double* C) {
  long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)m * n) return;
  int i = (int)(idx / n), j = (int)(idx % n);
  double s = 0.0;
  for (int l = 0; l < k; l++) s = __dadd_rn(s, __dmul_rn(A[(long)i * k + l], B[(long)l * n + j]));
  C[idx] = s;
}
__global__ void lincomb3_f64_kernel(double* X, const double* __restrict__ P, const double* __restrict__ Q, int it,
                                    long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double a = c_ns_coeffs[it][0], b = c_ns_coeffs[it][1], c = c_ns_coeffs[it][2];
  X[i] = __dadd_rn(__dadd_rn(__dmul_rn(a, X[i]), __dmul_rn(b, P[i])), __dmul_rn(c, Q[i]));
}
__global__ void finalize_f64_kernel(const double* __restrict__ W, const double* __restrict__ X, double c1, double c2,
                                    double* nW, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) nW[i] = __dadd_rn(__dmul_rn(c1, W[i]), __dmul_rn(c2, X[i]));
}
// stepVec (Puffer/Float/Muon.lean:105-108); g pre-scaled by gs when gs != 1.
__global__ void stepvec_f64_kernel(double* b, double* m, const double* __restrict__ g, double lr, double wd,
                                   double mu, double gs_val, const double* gsp, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double gs = gsp ? *gsp : gs_val;
  const double gi = gs == 1.0 ? g[i] : __dmul_rn(g[i], gs);
  const double newm = __dadd_rn(__dmul_rn(mu, m[i]), gi);
  const double upd = __dadd_rn(gi, __dmul_rn(mu, newm));
  b[i] = __dadd_rn(__dmul_rn(b[i], __dsub_rn(1.0, __dmul_rn(lr, wd))), __dmul_rn(lr, upd));
  m[i] = newm;
}

// The whole exact step of one matrix small enough for shared memory, in one CTA: every element goes
// through the same sequence of rounded operations as in the kernels above (Nesterov, per-row sums of
// squares folded in row order, the scale, iters x (transpose, three matmuls with their sums from 0 in
// l order, lincomb3), finalize), so the result is the same bits, in one launch instead of 5 iters + 5.
// G is the f64 gradient or the f32 one (widened exactly on load); Wf, when set, receives (float) W.
template <typename GT>
__device__ void exact_small_cta(int rows, int cols, double* W, double* M, const GT* __restrict__ G, double gs,
                                double mu, double eps, int iters, double c1, double c2, double* sm, float* Wf) {
  const int n = rows * cols, mn = rows < cols ? rows : cols;
  double *U = sm, *X = U + n, *Xt = X + n, *P = Xt + n, *Q = P + n, *Am = Q + n, *rs = Am + mn * mn,
         *inv = rs + rows;
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int i = tid; i < n; i += nt) {
    const double g = (double)G[i];
    const double gi = gs == 1.0 ? g : __dmul_rn(g, gs);
    const double newm = __dadd_rn(__dmul_rn(mu, M[i]), gi);
    M[i] = newm;
    U[i] = __dadd_rn(gi, __dmul_rn(mu, newm));
  }
  __syncthreads();
  for (int r = tid; r < rows; r += nt) {
    double acc = 0.0;
#pragma unroll 4
    for (int j = 0; j < cols; j++) acc = __dadd_rn(acc, __dmul_rn(U[r * cols + j], U[r * cols + j]));
    rs[r] = acc;
  }
  __syncthreads();
  if (tid == 0) {
    double acc = 0.0;
#pragma unroll 8
    for (int i = 0; i < rows; i++) acc = __dadd_rn(acc, rs[i]);
    inv[0] = __ddiv_rn(1.0, __dadd_rn(__dsqrt_rn(acc), eps));
  }
  __syncthreads();
  for (int i = tid; i < n; i += nt) X[i] = __dmul_rn(inv[0], U[i]);
  __syncthreads();
  // C[m x q] = A[m x k] B[k x q], each output's sum from 0 in l order (matmul_f64_kernel's order)
  auto matmul = [&](const double* A, const double* B, int m, int k, int q, double* Cm) {
    for (int idx = tid; idx < m * q; idx += nt) {
      const int i = idx / q, j = idx % q;
      double acc = 0.0;
#pragma unroll 8
      for (int l = 0; l < k; l++) acc = __dadd_rn(acc, __dmul_rn(A[i * k + l], B[l * q + j]));
      Cm[idx] = acc;
    }
    __syncthreads();
  };
  for (int it = 0; it < iters; it++) {
    for (int idx = tid; idx < n; idx += nt) {
      const int i = idx / cols, j = idx % cols;
      Xt[j * rows + i] = X[idx];
    }
    __syncthreads();
    if (rows <= cols) {
      matmul(X, Xt, rows, cols, rows, Am);
      matmul(Am, X, rows, rows, cols, P);
      matmul(Am, P, rows, rows, cols, Q);
    } else {
      matmul(Xt, X, cols, rows, cols, Am);
      matmul(X, Am, rows, cols, cols, P);
      matmul(P, Am, rows, cols, cols, Q);
    }
    const double a = c_ns_coeffs[it][0], b = c_ns_coeffs[it][1], c = c_ns_coeffs[it][2];
    for (int i = tid; i < n; i += nt) X[i] = __dadd_rn(__dadd_rn(__dmul_rn(a, X[i]), __dmul_rn(b, P[i])), __dmul_rn(c, Q[i]));
    __syncthreads();
  }
  for (int i = tid; i < n; i += nt) {
    const double w = __dadd_rn(__dmul_rn(c1, W[i]), __dmul_rn(c2, X[i]));
    W[i] = w;
    if (Wf) Wf[i] = (float)w;
  }
}
__global__ void __launch_bounds__(256) muon_exact_small_kernel(int rows, int cols, double* W, double* M,
                                                               const double* __restrict__ G, double gs_val,
                                                               const double* gsp, double mu, double eps,
                                                               int iters, double c1, double c2) {
  extern __shared__ double sm[];
  exact_small_cta<double>(rows, cols, W, M, G, gsp ? *gsp : gs_val, mu, eps, iters, c1, c2, sm, nullptr);
}

// Every layer's tight-tier step in one launch, one CTA per job: a matrix job is exact_small_cta on the
// f32 gradient, a bias job (cols == 0) is stepVec (stepvec_f64_kernel's arithmetic); both also write the
// f32 copies the next forward reads. The gradient scale is read on the device.
struct ExactJob {
  double* W;
  double* M;
  const float* G;
  float* Wf;
  int rows, cols;
  double c1, c2;
};
constexpr int kMaxExactJobs = 32;
struct ExactJobs {
  ExactJob j[kMaxExactJobs];
};
__global__ void __launch_bounds__(256) muon_exact_group_kernel(const ExactJobs jobs, const double* __restrict__ gsp,
                                                               double mu, double eps, int iters, double lr, double wd) {
  extern __shared__ double sm[];
  const ExactJob jb = jobs.j[blockIdx.x];
  const double gs = *gsp;
  if (jb.cols > 0) {
    exact_small_cta<float>(jb.rows, jb.cols, jb.W, jb.M, jb.G, gs, mu, eps, iters, jb.c1, jb.c2, sm, jb.Wf);
    return;
  }
  for (int i = threadIdx.x; i < jb.rows; i += blockDim.x) {
    const double g = (double)jb.G[i];
    const double gi = gs == 1.0 ? g : __dmul_rn(g, gs);
    const double newm = __dadd_rn(__dmul_rn(mu, jb.M[i]), gi);
    const double upd = __dadd_rn(gi, __dmul_rn(mu, newm));
    const double b = __dadd_rn(__dmul_rn(jb.W[i], __dsub_rn(1.0, __dmul_rn(lr, wd))), __dmul_rn(lr, upd));
    jb.W[i] = b;
    jb.M[i] = newm;
    jb.Wf[i] = (float)b;
  }
}

int set_ns_coeffs(const double* coeffs, int iters, cudaStream_t st) {
  PL_REQUIRE(iters >= 0 && iters <= 64, PL_ERR_INVALID, "Newton-Schulz iterations %d out of range", iters);
  if (iters) PL_CUDA(cudaMemcpyToSymbolAsync(c_ns_coeffs, coeffs, sizeof(double) * 3 * iters, 0,
                                             cudaMemcpyHostToDevice, st));
  return PL_OK;
}

const double kMuonCoeffs[5][3] = {{4.0848, -6.8946, 2.9270}, {3.9505, -6.3029, 2.6377}, {3.7418, -5.5913, 2.3037},
                                  {2.8769, -3.1427, 1.2046}, {2.8366, -3.0525, 1.2012}};

size_t exact_ws_doubles(int rows, int cols) {
  long n = (long)rows * cols;
  int mn = rows < cols ? rows : cols;
  return (size_t)(5 * n + (long)mn * mn + rows + 8);
}

// In place on (W, M): W <- stepMat(W, g*gs, M) (gs read on the device from gsp when that is not NULL). ws
// holds exact_ws_doubles(rows, cols) doubles. A matrix whose working set fits in shared memory runs in one
// CTA (muon_exact_small_kernel), otherwise one launch per operation.
int muon_mat_exact(int rows, int cols, double* W, double* M, const double* G, double gs, double lr, double wd,
                   double mu, double eps, int iters, double* ws, cudaStream_t st, const double* gsp) {
  const long n = (long)rows * cols;
  const int mn = rows < cols ? rows : cols;
  const double r = (double)rows / (double)cols;
  const double scale = sqrt(1.0 <= r ? r : 1.0);
  volatile double lrwd = lr * wd;
  const double c1 = 1.0 - lrwd, c2 = lr * scale;
  const size_t small_bytes = sizeof(double) * (size_t)(5 * n + (long)mn * mn + rows + 8);
  if (small_bytes <= kSmallMuonBytes && iters <= 64) {
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      PL_CUDA(cudaFuncSetAttribute((const void*)muon_exact_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kSmallMuonBytes));
      attr_set[dev] = true;
    }
    muon_exact_small_kernel<<<1, 256, small_bytes, st>>>(rows, cols, W, M, G, gs, gsp, mu, eps, iters, c1, c2);
    count_launch();
    PL_LAUNCH("muon_exact_small_kernel");
    return PL_OK;
  }
  double *U = ws, *X = U + n, *Xt = X + n, *P = Xt + n, *Q = P + n, *Am = Q + n, *rs = Am + (long)mn * mn,
         *inv = rs + rows;
  const int B = 256;
  const unsigned gN = (unsigned)ceil_div(n, B);
  nesterov_f64_kernel<<<gN, B, 0, st>>>(G, M, M, U, mu, gs, gsp, n);
  frob_rows_f64_kernel<<<(unsigned)ceil_div(rows, 128), 128, 0, st>>>(U, rows, cols, rs);
  frob_fold_f64_kernel<<<1, 32, 0, st>>>(rs, rows, eps, inv);
  scale_f64_kernel<<<gN, B, 0, st>>>(U, inv, X, n);
  count_launch(4);
  for (int it = 0; it < iters; it++) {
    transpose_f64_kernel<<<gN, B, 0, st>>>(X, rows, cols, Xt);
    if (rows <= cols) {
      matmul_f64_kernel<<<(unsigned)ceil_div((long)rows * rows, B), B, 0, st>>>(X, Xt, rows, cols, rows, Am);
      matmul_f64_kernel<<<gN, B, 0, st>>>(Am, X, rows, rows, cols, P);
      matmul_f64_kernel<<<gN, B, 0, st>>>(Am, P, rows, rows, cols, Q);
    } else {
      matmul_f64_kernel<<<(unsigned)ceil_div((long)cols * cols, B), B, 0, st>>>(Xt, X, cols, rows, cols, Am);
      matmul_f64_kernel<<<gN, B, 0, st>>>(X, Am, rows, cols, cols, P);
      matmul_f64_kernel<<<gN, B, 0, st>>>(P, Am, rows, cols, cols, Q);
    }
    lincomb3_f64_kernel<<<gN, B, 0, st>>>(X, P, Q, it, n);
    count_launch(5);
  }
  finalize_f64_kernel<<<gN, B, 0, st>>>(W, X, c1, c2, W, n);
  count_launch();
  PL_LAUNCH("muon_mat_exact");
  return PL_OK;
}

static size_t small_bytes_of(int rows, int cols) {
  const long n = (long)rows * cols;
  const int mn = rows < cols ? rows : cols;
  return sizeof(double) * (size_t)(5 * n + (long)mn * mn + rows + 8);
}
bool muon_group_fits(const ExactLayer* ls, int n, int iters) {
  if (n <= 0 || 2 * n > kMaxExactJobs || iters > 64) return false;
  for (int i = 0; i < n; i++)
    if (small_bytes_of(ls[i].rows, ls[i].cols) > kSmallMuonBytes) return false;
  return true;
}
int muon_group_exact(const ExactLayer* ls, int n, double* pm, long P, const float* g, double lr, double wd, double mu,
                     double eps, int iters, const double* gsp, cudaStream_t st) {
  PL_REQUIRE(muon_group_fits(ls, n, iters), PL_ERR_INVALID, "exact Muon group does not fit one CTA per matrix");
  ExactJobs jobs{};
  size_t smem = 0;
  volatile double lrwd = lr * wd;  // rounded on its own, as in muon_mat_exact
  for (int i = 0; i < n; i++) {
    const ExactLayer& l = ls[i];
    const double r = (double)l.rows / (double)l.cols;
    const double scale = sqrt(1.0 <= r ? r : 1.0);
    jobs.j[2 * i] = ExactJob{pm + l.oW, pm + P + l.oW, g + l.oW, l.Wf, l.rows, l.cols, 1.0 - lrwd, lr * scale};
    jobs.j[2 * i + 1] = ExactJob{pm + l.ob, pm + P + l.ob, g + l.ob, l.bf, l.rows, 0, 0.0, 0.0};
    smem = std::max(smem, small_bytes_of(l.rows, l.cols));
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    PL_CUDA(cudaFuncSetAttribute((const void*)muon_exact_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSmallMuonBytes));
    attr_set[dev] = true;
  }
  muon_exact_group_kernel<<<2 * n, 256, smem, st>>>(jobs, gsp, mu, eps, iters, lr, wd);
  count_launch();
  PL_LAUNCH("muon_exact_group_kernel");
  return PL_OK;
}

int stepvec_launch(double* b, double* m, const double* g, double lr, double wd, double mu, double gs, long n,
                   cudaStream_t st, const double* gsp) {
  if (n <= 0) return PL_OK;
  stepvec_f64_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(b, m, g, lr, wd, mu, gs, gsp, n);
  count_launch();
  PL_LAUNCH("stepvec_f64_kernel");
  return PL_OK;
}

}  // namespace pl

extern "C" int pl_muon_stepmat(const double* W, const double* G, const double* M, size_t rows, size_t cols, double lr,
                               double wd, double mu, double eps, double* out) {
  int rc = pl::require_device();
  if (rc) return rc;
  PL_REQUIRE(W && G && M && out, PL_ERR_INVALID, "pl_muon_stepmat: NULL buffer");
  const size_t n = rows * cols;
  if (n == 0) return PL_OK;
  const size_t wsd = pl::exact_ws_doubles((int)rows, (int)cols);
  double* d = (double*)pl::scratch(1, sizeof(double) * (3 * n + wsd));
  if (!d) return PL_ERR_NOMEM;
  double *dW = d, *dM = d + n, *dG = d + 2 * n, *ws = d + 3 * n;
  PL_CUDA(cudaMemcpy(dW, W, 8 * n, cudaMemcpyHostToDevice));
  PL_CUDA(cudaMemcpy(dM, M, 8 * n, cudaMemcpyHostToDevice));
  PL_CUDA(cudaMemcpy(dG, G, 8 * n, cudaMemcpyHostToDevice));
  rc = pl::set_ns_coeffs(&pl::kMuonCoeffs[0][0], 5, 0);
  if (rc) return rc;
  rc = pl::muon_mat_exact((int)rows, (int)cols, dW, dM, dG, 1.0, lr, wd, mu, eps, 5, ws, 0);
  if (rc) return rc;
  PL_CUDA(cudaMemcpy(out, dW, 8 * n, cudaMemcpyDeviceToHost));
  PL_CUDA(cudaMemcpy(out + n, dM, 8 * n, cudaMemcpyDeviceToHost));
  return PL_OK;
}
