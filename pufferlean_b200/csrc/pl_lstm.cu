// LSTM + PPO truncated-BPTT gradient, batched over B sequences packed time-major (row r = t*B + b):
// the device form of the reference's batched LSTM gradient (ffi/pufferblas.c:897-1018 and its f32 /
// bf16 tiers, ffi/puffercuda.cu:6794-7182). params [Wx(4H x D) | Wh(4H x H) | bih(4H) | Wo(O x H) | bo(O)],
// O = A + 1, gate rows i, f, g, o.
//
// Only the recurrence is sequential. Everything else is one product over all T*B rows: the input
// projection X Wx^T, the head H Wo^T and its data gradient dOut Wo, and the weight gradients
// dG^T X, dG^T Hprev, dOut^T H (split over fixed row slices, summed in slice order) and the bias
// column sums. The recurrence runs as two persistent kernels, forward and reverse: a CTA owns `rows`
// sequences for all T steps, thread (r, j) carries unit j of sequence r (h, c, and in reverse dh, dc)
// in registers, Wh sits in shared memory with a padded row stride (H + 1, so the forward's row reads
// and the reverse's column reads both hit distinct banks), and a terminal at step t zeroes the state
// before step t + 1 and stops the gradient there. Tiers: 0 = f64 arithmetic throughout, 1 = f32; tier 2
// (the reference's bf16 tier) is the f32 computation with every product's operands rounded to bf16 before
// the multiply-add and f32 accumulation, as cuBLAS's CUBLAS_COMPUTE_32F_FAST_16BF does for the
// reference's GEMMs; the gate, cell and head arithmetic stays f32.
#include <mutex>

#include "../../include/pufferlean_b200.h"
#include "pl_common.cuh"
#include "pl_gemm.cuh"
#include "pl_mlp.cuh"
#include "pl_runtime.h"

namespace pl {
namespace {

__device__ __forceinline__ float lexp(float x) { return expf(x); }
__device__ __forceinline__ double lexp(double x) { return exp(x); }
__device__ __forceinline__ float ltanh(float x) { return tanhf(x); }
__device__ __forceinline__ double ltanh(double x) { return tanh(x); }
__device__ __forceinline__ float llog(float x) { return logf(x); }
__device__ __forceinline__ double llog(double x) { return log(x); }
template <typename R>
__device__ __forceinline__ R lsig(R x) {
  return R(1) / (R(1) + lexp(-x));
}

// An operand of a product: as is, or (RB, the bf16 tier) rounded to bf16 to nearest even.
template <bool RB, typename R>
__device__ __forceinline__ R lop(R x) {
  if constexpr (RB) return (R)__bfloat162float(__float2bfloat16_rn((float)x));
  return x;
}

// C[z][m, n] = sum_{k in slice z} A[m*ars + k*acs] * B[n*brs + k*bcs], k ascending; 64 x 64 tiles,
// 16-deep k steps through shared memory, 4 x 4 outputs per thread. gridDim.z slices of kc rows of K.
template <typename R, bool RB>
__global__ void __launch_bounds__(256) lstm_gemm_kernel(int M, int N, int K, int kc, const R* __restrict__ A,
                                                        long ars, long acs, const R* __restrict__ B, long brs,
                                                        long bcs, R* C, long ldc, long zs) {
  __shared__ R sA[16][65];
  __shared__ R sB[16][65];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int k0 = blockIdx.z * kc, k1 = min(K, k0 + kc);
  R acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = R(0);
  for (int kb = k0; kb < k1; kb += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      const int kk = e / 64, mm = e - kk * 64;
      const int k = kb + kk;
      sA[kk][mm] = (k < k1 && m0 + mm < M) ? lop<RB>(A[(long)(m0 + mm) * ars + (long)k * acs]) : R(0);
      sB[kk][mm] = (k < k1 && n0 + mm < N) ? lop<RB>(B[(long)(n0 + mm) * brs + (long)k * bcs]) : R(0);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; kk++) {
      R a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = sA[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = sB[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] += a[i] * b[j];
    }
    __syncthreads();
  }
  R* Cz = C + (long)blockIdx.z * zs;
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < M && n < N) Cz[(long)m * ldc + n] = acc[i][j];
    }
}
// out[i] = (double) sum_z part[z*n + i], z ascending. Sixteen slices' loads go out before their sums,
// which are still taken one by one in slice order (the loads, not the adds, are what the sum waits on).
template <typename R>
__global__ void lstm_slice_sum_kernel(const R* __restrict__ part, int nz, long n, double* out) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    R s = R(0);
    int z = 0;
    for (; z + 16 <= nz; z += 16) {
      R v[16];
#pragma unroll
      for (int k = 0; k < 16; k++) v[k] = part[(long)(z + k) * n + i];
#pragma unroll
      for (int k = 0; k < 16; k++) s += v[k];
    }
    for (; z < nz; z++) s += part[(long)z * n + i];
    out[i] = (double)s;
  }
}
// part[chunk][c] = sum of rows [chunk*rows_per, ...) of column c, in row order (sixteen rows' loads
// ahead of their sums); then out[c] = sum over chunks in order
template <typename R>
__global__ void lstm_colsum_part_kernel(const R* __restrict__ M, long rows, int N, int rows_per, R* part) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= N) return;
  const long r0 = (long)blockIdx.y * rows_per, r1 = min(rows, r0 + (long)rows_per);
  R s = R(0);
  long r = r0;
  for (; r + 16 <= r1; r += 16) {
    R v[16];
#pragma unroll
    for (int k = 0; k < 16; k++) v[k] = M[(r + k) * N + c];
#pragma unroll
    for (int k = 0; k < 16; k++) s += v[k];
  }
  for (; r < r1; r++) s += M[r * N + c];
  part[(long)blockIdx.y * N + c] = s;
}
template <typename V>
__global__ void lstm_cast_kernel(const double* __restrict__ s, long n, V* d) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) d[i] = (V)s[i];
}
__global__ void lstm_act_kernel(const double* __restrict__ s, long n, int A, int* d) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    int a = (int)(unsigned long long)s[i];
    d[i] = a < 0 ? 0 : (a >= A ? A - 1 : a);  // a malformed action column cannot index past the logits
  }
}

// Forward recurrence. Gin [R x 4H] = X Wx^T (no bias); per step g = (bih + Gin) + h_prev Wh^T. WS: Wh
// staged in shared memory (it fits up to H ~ 64 in f32); otherwise it is read through L1 / L2.
template <typename R, bool WS, bool RB>
__global__ void lstm_fwd_kernel(const R* __restrict__ Gin, const R* __restrict__ Wh, const R* __restrict__ bih,
                                const double* __restrict__ term, const R* __restrict__ h0,
                                const R* __restrict__ c0, R* II, R* FF, R* GG, R* OO, R* TC, R* HT, R* HP, R* CP,
                                int B, int T, int H, int rows) {
  extern __shared__ __align__(16) unsigned char lstm_smem[];
  const int H4 = 4 * H, SW = H + 1;
  R* sWh = (R*)lstm_smem;                    // [4H][H + 1] when WS
  R* sh = sWh + (WS ? (long)H4 * SW : 0L);   // [rows][H]
  const int tid = threadIdx.x, r = tid / H, j = tid - r * H;
  const int b = blockIdx.x * rows + r;
  const bool ok = r < rows && b < B;
  if (WS)
    for (int i = tid; i < H4 * H; i += blockDim.x) {
      const int m = i / H, k = i - m * H;
      sWh[(long)m * SW + k] = lop<RB>(Wh[i]);
    }
  const R* Wm = WS ? sWh : Wh;
  const int ws = WS ? SW : H;
  R c = ok ? c0[(long)b * H + j] : R(0);
  if (r < rows) sh[r * H + j] = ok ? h0[(long)b * H + j] : R(0);
  const R bi = bih[j], bf = bih[H + j], bg = bih[2 * H + j], bo = bih[3 * H + j];
  // this step's input projections and the previous step's terminal flag are loaded one step ahead, so
  // their latency hides under the step before
  R gi = R(0), gf = R(0), gg = R(0), go = R(0);
  double tprev = 0.0;
  if (ok) {
    const R* g = Gin + (long)b * H4;
    gi = g[j];
    gf = g[H + j];
    gg = g[2 * H + j];
    go = g[3 * H + j];
  }
  __syncthreads();
  for (int t = 0; t < T; t++) {
    if (t > 0 && ok && tprev != 0.0) {
      sh[r * H + j] = R(0);
      c = R(0);
    }
    const R ci = gi, cf = gf, cg = gg, co = go;
    if (ok && t + 1 < T) {
      const R* g = Gin + ((long)(t + 1) * B + b) * H4;
      gi = g[j];
      gf = g[H + j];
      gg = g[2 * H + j];
      go = g[3 * H + j];
      tprev = term[(long)t * B + b];
    }
    __syncthreads();
    R a0 = R(0), a1 = R(0), a2 = R(0), a3 = R(0), hold = R(0);
    if (r < rows) {
      const R* hr = sh + r * H;
      const R* w0 = Wm + (long)j * ws;
      const R* w1 = Wm + (long)(H + j) * ws;
      const R* w2 = Wm + (long)(2 * H + j) * ws;
      const R* w3 = Wm + (long)(3 * H + j) * ws;
#pragma unroll 8
      for (int k = 0; k < H; k++) {
        const R hv = lop<RB>(hr[k]);
        if (WS) {  // staged already rounded
          a0 += w0[k] * hv;
          a1 += w1[k] * hv;
          a2 += w2[k] * hv;
          a3 += w3[k] * hv;
        } else {
          a0 += lop<RB>(w0[k]) * hv;
          a1 += lop<RB>(w1[k]) * hv;
          a2 += lop<RB>(w2[k]) * hv;
          a3 += lop<RB>(w3[k]) * hv;
        }
      }
      hold = hr[j];
    }
    __syncthreads();  // every read of the step's h is done before it is overwritten
    if (ok) {
      const long row = (long)t * B + b;
      const R iv = lsig((bi + ci) + a0), fv = lsig((bf + cf) + a1);
      const R gv = ltanh((bg + cg) + a2), ov = lsig((bo + co) + a3);
      const R cn = fv * c + iv * gv, tcv = ltanh(cn), hv = ov * tcv;
      const long o = row * H + j;
      II[o] = iv;
      FF[o] = fv;
      GG[o] = gv;
      OO[o] = ov;
      TC[o] = tcv;
      HT[o] = hv;
      HP[o] = hold;
      CP[o] = c;
      c = cn;
      sh[r * H + j] = hv;
    }
  }
}

// Reverse recurrence. dHo [R x H] = dOut Wo (the head's share of dh); writes dG [R x 4H].
template <typename R, bool WS, bool RB>
__global__ void lstm_bwd_kernel(const R* __restrict__ II, const R* __restrict__ FF, const R* __restrict__ GG,
                                const R* __restrict__ OO, const R* __restrict__ TC, const R* __restrict__ CP,
                                const R* __restrict__ dHo, const R* __restrict__ Wh, const double* __restrict__ term,
                                R* dG, int B, int T, int H, int rows) {
  extern __shared__ __align__(16) unsigned char lstm_smem[];
  const int H4 = 4 * H, SW = H + 1;
  R* sWh = (R*)lstm_smem;                    // [4H][H + 1] when WS
  R* sdg = sWh + (WS ? (long)H4 * SW : 0L);  // [rows][4H]
  const int tid = threadIdx.x, r = tid / H, j = tid - r * H;
  const int b = blockIdx.x * rows + r;
  const bool ok = r < rows && b < B;
  if (WS)
    for (int i = tid; i < H4 * H; i += blockDim.x) {
      const int m = i / H, k = i - m * H;
      sWh[(long)m * SW + k] = lop<RB>(Wh[i]);
    }
  const R* Wm = WS ? sWh : Wh;
  const int ws = WS ? SW : H;
  R dhn = R(0), dcn = R(0);
  // the step's saved activations (and the next step's terminal flag) are loaded one step ahead
  R nho = R(0), ntc = R(0), nov = R(0), niv = R(0), nfv = R(0), ngv = R(0), ncp = R(0);
  double nterm = 0.0;
  if (ok) {
    const long o = ((long)(T - 1) * B + b) * H + j;
    nho = dHo[o];
    ntc = TC[o];
    nov = OO[o];
    niv = II[o];
    nfv = FF[o];
    ngv = GG[o];
    ncp = CP[o];
    if (T > 1) nterm = term[(long)(T - 2) * B + b];
  }
  __syncthreads();
  for (int t = T - 1; t >= 0; t--) {
    R dcp = R(0);
    const R cho = nho, tcv = ntc, ov = nov, iv = niv, fv = nfv, gv = ngv, cpv = ncp;
    const double cterm = nterm;
    if (ok && t > 0) {
      const long o = ((long)(t - 1) * B + b) * H + j;
      nho = dHo[o];
      ntc = TC[o];
      nov = OO[o];
      niv = II[o];
      nfv = FF[o];
      ngv = GG[o];
      ncp = CP[o];
      if (t > 1) nterm = term[(long)(t - 2) * B + b];
    }
    if (ok) {
      const long row = (long)t * B + b;
      const R dh = cho + dhn;
      const R dc = dcn + dh * ov * (R(1) - tcv * tcv);
      const R dO = dh * tcv, dF = dc * cpv, dI = dc * gv, dGg = dc * iv;
      dcp = dc * fv;
      const R q0 = dI * iv * (R(1) - iv), q1 = dF * fv * (R(1) - fv), q2 = dGg * (R(1) - gv * gv),
              q3 = dO * ov * (R(1) - ov);
      R* dgr = dG + row * H4;
      dgr[j] = q0;
      dgr[H + j] = q1;
      dgr[2 * H + j] = q2;
      dgr[3 * H + j] = q3;
      R* s = sdg + r * H4;  // the product's operand copy (rounded in the bf16 tier)
      s[j] = lop<RB>(q0);
      s[H + j] = lop<RB>(q1);
      s[2 * H + j] = lop<RB>(q2);
      s[3 * H + j] = lop<RB>(q3);
    }
    __syncthreads();
    R dhp = R(0);
    if (ok) {
      const R* s = sdg + r * H4;
      if (WS) {
#pragma unroll 8
        for (int k = 0; k < H4; k++) dhp += s[k] * Wm[(long)k * ws + j];
      } else {
#pragma unroll 8
        for (int k = 0; k < H4; k++) dhp += s[k] * lop<RB>(Wm[(long)k * ws + j]);
      }
      const bool flow = t > 0 && cterm == 0.0;
      dhn = flow ? dhp : R(0);
      dcn = flow ? dcp : R(0);
    }
    __syncthreads();  // the step's dG row is read before the next step overwrites it
  }
}

// Four threads per unit (H a multiple of 8, 4H <= 1024 threads per sequence, Wh staged): lane
// (j % 8) + 8 q of warp j / 8 owns gate q of unit j, so each dot product of a step is one thread's and
// a step's latency is a quarter of the one-thread-per-unit form's. Wh's gate blocks sit 8 elements
// apart in shared memory (gate q's rows from q (H (H + 1) + 8)), so the four gates' lanes of a warp read
// distinct banks.
__device__ __forceinline__ long lstm_q_off(int q, int H) { return (long)q * ((long)H * (H + 1) + 8); }

// Forward, four threads per unit: each lane forms its gate's pre-activation (bias + input projection)
// + h_prev . Wh row in the same order as lstm_fwd_kernel, the unit's four values meet by shuffles, and
// every lane of the unit carries the cell; gate q's lane writes two of the eight saved rows.
template <typename R, bool RB>
__global__ void lstm_fwd4_kernel(const R* __restrict__ Gin, const R* __restrict__ Wh, const R* __restrict__ bih,
                                 const double* __restrict__ term, const R* __restrict__ h0,
                                 const R* __restrict__ c0, R* II, R* FF, R* GG, R* OO, R* TC, R* HT, R* HP, R* CP,
                                 int B, int T, int H, int rows) {
  extern __shared__ __align__(16) unsigned char lstm_smem[];
  const int H4 = 4 * H, SW = H + 1;
  R* sWh = (R*)lstm_smem;
  R* sh = sWh + lstm_q_off(4, H);  // [rows][H]
  const int tid = threadIdx.x, r = tid / H4, l = tid - r * H4;
  const int lane = l & 31, q = lane >> 3, j = 8 * (l >> 5) + (lane & 7);
  const int b = blockIdx.x * rows + r;
  const bool ok = r < rows && b < B;
  for (int i = tid; i < H4 * H; i += blockDim.x) {
    const int m = i / H, k = i - m * H;
    sWh[lstm_q_off(m / H, H) + (long)(m % H) * SW + k] = lop<RB>(Wh[i]);
  }
  R c = ok ? c0[(long)b * H + j] : R(0);
  if (r < rows && q == 0) sh[r * H + j] = ok ? h0[(long)b * H + j] : R(0);
  const R bq = bih[q * H + j];
  const R* wrow = sWh + lstm_q_off(q, H) + (long)j * SW;
  R gq = ok ? Gin[(long)b * H4 + q * H + j] : R(0);
  double tprev = 0.0;
  __syncthreads();
  for (int t = 0; t < T; t++) {
    if (t > 0 && ok && tprev != 0.0) {
      if (q == 0) sh[r * H + j] = R(0);
      c = R(0);
    }
    const R cg = gq;
    if (ok && t + 1 < T) {
      gq = Gin[((long)(t + 1) * B + b) * H4 + q * H + j];
      tprev = term[(long)t * B + b];
    }
    __syncthreads();
    R a = R(0), hold = R(0);
    if (r < rows) {
      const R* hr = sh + r * H;
#pragma unroll 8
      for (int k = 0; k < H; k++) a += wrow[k] * lop<RB>(hr[k]);
      hold = hr[j];
    }
    __syncthreads();  // every read of the step's h is done before it is overwritten
    const R z = (bq + cg) + a;
    const int base = lane & 7;
    const R z0 = __shfl_sync(0xffffffffu, z, base), z1 = __shfl_sync(0xffffffffu, z, base + 8);
    const R z2 = __shfl_sync(0xffffffffu, z, base + 16), z3 = __shfl_sync(0xffffffffu, z, base + 24);
    if (ok) {
      const long o = ((long)t * B + b) * H + j;
      const R iv = lsig(z0), fv = lsig(z1), gv = ltanh(z2), ov = lsig(z3);
      const R cn = fv * c + iv * gv, tcv = ltanh(cn), hv = ov * tcv;
      if (q == 0) {
        II[o] = iv;
        TC[o] = tcv;
        sh[r * H + j] = hv;
      } else if (q == 1) {
        FF[o] = fv;
        HT[o] = hv;
      } else if (q == 2) {
        GG[o] = gv;
        HP[o] = hold;
      } else {
        OO[o] = ov;
        CP[o] = c;
      }
      c = cn;
    }
  }
}

// Reverse, four threads per unit: every lane of the unit carries dh and dc and forms the unit's four gate
// derivatives, gate q's lane stores its own; dh_prev[j] is the sum over the four gate blocks of
// Wh[k][j] s[k], one block per lane, added by a fixed butterfly (a different summation order from
// lstm_bwd_kernel's single pass).
template <typename R, bool RB>
__global__ void lstm_bwd4_kernel(const R* __restrict__ II, const R* __restrict__ FF, const R* __restrict__ GG,
                                 const R* __restrict__ OO, const R* __restrict__ TC, const R* __restrict__ CP,
                                 const R* __restrict__ dHo, const R* __restrict__ Wh,
                                 const double* __restrict__ term, R* dG, int B, int T, int H, int rows) {
  extern __shared__ __align__(16) unsigned char lstm_smem[];
  const int H4 = 4 * H, SW = H + 1, SQ = H + 8;
  R* sWh = (R*)lstm_smem;
  R* sdg = sWh + lstm_q_off(4, H);  // [rows][4 (H + 8)]: gate q's block at q (H + 8)
  const int tid = threadIdx.x, r = tid / H4, l = tid - r * H4;
  const int lane = l & 31, q = lane >> 3, j = 8 * (l >> 5) + (lane & 7);
  const int b = blockIdx.x * rows + r;
  const bool ok = r < rows && b < B;
  for (int i = tid; i < H4 * H; i += blockDim.x) {
    const int m = i / H, k = i - m * H;
    sWh[lstm_q_off(m / H, H) + (long)(m % H) * SW + k] = lop<RB>(Wh[i]);
  }
  R dhn = R(0), dcn = R(0);
  R nho = R(0), ntc = R(0), nov = R(0), niv = R(0), nfv = R(0), ngv = R(0), ncp = R(0);
  double nterm = 0.0;
  if (ok) {
    const long o = ((long)(T - 1) * B + b) * H + j;
    nho = dHo[o];
    ntc = TC[o];
    nov = OO[o];
    niv = II[o];
    nfv = FF[o];
    ngv = GG[o];
    ncp = CP[o];
    if (T > 1) nterm = term[(long)(T - 2) * B + b];
  }
  const R* wcol = sWh + lstm_q_off(q, H) + j;  // column j of gate block q, rows k = 0..H-1 at stride SW
  __syncthreads();
  for (int t = T - 1; t >= 0; t--) {
    R dcp = R(0);
    const R cho = nho, tcv = ntc, ov = nov, iv = niv, fv = nfv, gv = ngv, cpv = ncp;
    const double cterm = nterm;
    if (ok && t > 0) {
      const long o = ((long)(t - 1) * B + b) * H + j;
      nho = dHo[o];
      ntc = TC[o];
      nov = OO[o];
      niv = II[o];
      nfv = FF[o];
      ngv = GG[o];
      ncp = CP[o];
      if (t > 1) nterm = term[(long)(t - 2) * B + b];
    }
    if (ok) {
      const long row = (long)t * B + b;
      const R dh = cho + dhn;
      const R dc = dcn + dh * ov * (R(1) - tcv * tcv);
      const R dO = dh * tcv, dF = dc * cpv, dI = dc * gv, dGg = dc * iv;
      dcp = dc * fv;
      const R qv = q == 0 ? dI * iv * (R(1) - iv)
                          : (q == 1 ? dF * fv * (R(1) - fv) : (q == 2 ? dGg * (R(1) - gv * gv) : dO * ov * (R(1) - ov)));
      dG[row * H4 + q * H + j] = qv;
      sdg[(long)r * 4 * SQ + q * SQ + j] = lop<RB>(qv);
    }
    __syncthreads();
    R p = R(0);
    if (r < rows) {
      const R* sq = sdg + (long)r * 4 * SQ + q * SQ;
#pragma unroll 8
      for (int k = 0; k < H; k++) p += sq[k] * wcol[(long)k * SW];
    }
    // the four gate blocks' partials of unit j (lanes base, base + 8, base + 16, base + 24), fixed order
    p += __shfl_xor_sync(0xffffffffu, p, 8);
    p += __shfl_xor_sync(0xffffffffu, p, 16);
    if (ok) {
      const bool flow = t > 0 && cterm == 0.0;
      dhn = flow ? p : R(0);
      dcn = flow ? dcp : R(0);
    }
    __syncthreads();  // the step's block rows are read before the next step overwrites them
  }
}

// Categorical head per row (the LSTM head: log-softmax without the max subtracted, no value clip);
// Out [R x O] without the bias; dOut [R x O].
template <typename R>
__global__ void lstm_head_kernel(const R* __restrict__ Out, const R* __restrict__ bo, long NR, int A,
                                 const int* __restrict__ act, const R* __restrict__ adv, const R* __restrict__ ret,
                                 const R* __restrict__ olp, R vf, R ent, R clip, R* dOut, double* newlp,
                                 double* newval) {
  const int O = A + 1;
  for (long r = (long)blockIdx.x * blockDim.x + threadIdx.x; r < NR; r += (long)gridDim.x * blockDim.x) {
    const R* o = Out + r * O;
    R se = R(0);
    for (int k = 0; k < A; k++) se += lexp(o[k] + bo[k]);
    const R lse = llog(se);
    R pout = R(0);
    for (int k = 0; k < A; k++) {
      const R l = o[k] + bo[k];
      pout += lexp(l - lse) * l;
    }
    const int a = act[r];
    const R logpA = (o[a] + bo[a]) - lse, ratio = lexp(logpA - olp[r]);
    const R lo = R(1) - clip, hi = R(1) + clip, rc = ratio < lo ? lo : (ratio > hi ? hi : ratio);
    const R ad = adv[r], s1 = ad * ratio, s2 = ad * rc;
    const R dPol = s1 <= s2 ? ad * ratio : ad * ((lo < ratio && ratio < hi) ? R(1) : R(0)) * ratio;
    R* d = dOut + r * O;
    for (int k = 0; k < A; k++) {
      const R l = o[k] + bo[k], p = lexp(l - lse);
      d[k] = dPol * ((k == a ? R(1) : R(0)) - p) + ent * p * (pout - l);
    }
    const R vnew = o[A] + bo[A];
    d[A] = -vf * (vnew - ret[r]);
    if (newlp) newlp[r] = (double)logpA;
    if (newval) newval[r] = (double)vnew;
  }
}

inline unsigned nblk(long n) {
  long g = (n + 255) / 256;
  if (g < 1) g = 1;
  if (g > 148 * 16) g = 148 * 16;
  return (unsigned)g;
}

// C = A B^T-style product with strides (see lstm_gemm_kernel); split into nz slices of K summed in order
// into the f64 output when out64 is given, else written (nz = 1) to C.
template <typename R>
int lstm_gemm(int M, int N, int K, const R* A, long ars, long acs, const R* B, long brs, long bcs, R* C, long ldc,
              int nz, cudaStream_t st, bool rb = false) {
  const int kc = (int)ceil_div(ceil_div(K, nz), 16) * 16;
  dim3 grid((unsigned)ceil_div(N, 64), (unsigned)ceil_div(M, 64), (unsigned)nz);
  if (rb)
    lstm_gemm_kernel<R, true><<<grid, 256, 0, st>>>(M, N, K, kc, A, ars, acs, B, brs, bcs, C, ldc, (long)M * ldc);
  else
    lstm_gemm_kernel<R, false><<<grid, 256, 0, st>>>(M, N, K, kc, A, ars, acs, B, brs, bcs, C, ldc, (long)M * ldc);
  count_launch();
  PL_LAUNCH("lstm_gemm_kernel");
  return PL_OK;
}

bool g_reuse_inputs = false;  // lean_cuda_lstm_reuse_inputs: this call's inputs equal the last call's
bool g_lstm_quad = true;      // four threads per unit in the recurrences where they fit (tests compare)

template <typename R>
int lstm_grad(const double* params, const double* obs, const double* acts, const double* advs, const double* rets,
              const double* olps, const double* terms, const double* h0s, const double* c0s, long B, long T, long H,
              long D, long A, double vf, double ent, double clip, bool tc, double* g, double* newlp,
              double* newval) {
  const long O = A + 1, H4 = 4 * H, NR = T * B;
  const long P = H4 * D + H4 * H + H4 + O * H + O;
  const cudaStream_t st = 0;
  const int rows_per = 256;
  const long nch = ceil_div(NR, rows_per);
  // weight gradients: K = T*B rows split into slices of ~128 rows, so the small M x N products still
  // spread over every SM; the slices are summed in order afterwards
  const int NZ = (int)std::min<long>(256, std::max<long>(1, NR / 128));
  // scratch slots 40..63: inputs, activations, gradients
  auto buf = [&](int slot, size_t bytes) { return scratch(slot, bytes); };
  double* stage = (double*)buf(40, sizeof(double) * std::max<long>(P, NR * std::max<long>(D, 2)));
  R* par = (R*)buf(41, sizeof(R) * P);
  R* X = (R*)buf(42, sizeof(R) * NR * D);
  int* act = (int*)buf(43, sizeof(int) * NR);
  R* col = (R*)buf(44, sizeof(R) * NR * 3);  // adv, ret, olp
  double* term = (double*)buf(45, sizeof(double) * NR);
  R* hc0 = (R*)buf(46, sizeof(R) * B * H * 2);
  R* Gin = (R*)buf(47, sizeof(R) * NR * H4);
  R* acts8 = (R*)buf(48, sizeof(R) * NR * H * 8);  // II FF GG OO TC HT HP CP
  R* Out = (R*)buf(49, sizeof(R) * NR * O);
  R* dOut = (R*)buf(50, sizeof(R) * NR * O);
  R* dHo = (R*)buf(51, sizeof(R) * NR * H);
  R* dG = (R*)buf(52, sizeof(R) * NR * H4);
  R* part = (R*)buf(53, sizeof(R) * (size_t)NZ * std::max<long>(H4 * std::max(D, H), O * H));
  R* cpart = (R*)buf(54, sizeof(R) * nch * std::max<long>(H4, O));
  double* g_d = (double*)buf(55, sizeof(double) * P);
  double* lpv = (double*)buf(56, sizeof(double) * NR * 2);
  if (!stage || !par || !X || !act || !col || !term || !hc0 || !Gin || !acts8 || !Out || !dOut || !dHo || !dG ||
      !part || !cpart || !g_d || !lpv)
    return PL_ERR_NOMEM;
  const R* Wx = par;
  const R* Wh = par + H4 * D;
  const R* bih = Wh + H4 * H;
  const R* Wo = bih + H4;
  const R* bo = Wo + O * H;
  auto cast = [&](const double* host, long n, R* dst) -> int {
    PL_CUDA(cudaMemcpyAsync(stage, host, sizeof(double) * n, cudaMemcpyHostToDevice, st));
    lstm_cast_kernel<R><<<nblk(n), 256, 0, st>>>(stage, n, dst);
    count_launch();
    PL_LAUNCH("lstm_cast_kernel");
    return PL_OK;
  };
  int rc = cast(params, P, par);
  if (!g_reuse_inputs) {
    if (!rc) rc = cast(obs, NR * D, X);
    if (!rc) rc = cast(advs, NR, col);
    if (!rc) rc = cast(rets, NR, col + NR);
    if (!rc) rc = cast(olps, NR, col + 2 * NR);
    if (!rc) rc = cast(h0s, B * H, hc0);
    if (!rc) rc = cast(c0s, B * H, hc0 + B * H);
    if (rc) return rc;
    PL_CUDA(cudaMemcpyAsync(stage, acts, sizeof(double) * NR, cudaMemcpyHostToDevice, st));
    lstm_act_kernel<<<nblk(NR), 256, 0, st>>>(stage, NR, (int)A, act);
    count_launch();
    PL_CUDA(cudaMemcpyAsync(term, terms, sizeof(double) * NR, cudaMemcpyHostToDevice, st));
  }
  if (rc) return rc;
  R* II = acts8;
  R* FF = II + NR * H;
  R* GG = FF + NR * H;
  R* OO = GG + NR * H;
  R* TC = OO + NR * H;
  R* HT = TC + NR * H;
  R* HP = HT + NR * H;
  R* CP = HP + NR * H;
  // ---- products over all rows that do not depend on the recurrence, and the recurrence itself
  auto fwd_products = [&]() -> int {
    return lstm_gemm<R>((int)NR, (int)H4, (int)D, X, D, 1, Wx, D, 1, Gin, H4, 1, st, tc);  // Gin = X Wx^T
  };
  rc = fwd_products();
  if (rc) return rc;
  // Four threads per unit when a sequence's 4H threads fit a CTA and Wh fits shared memory (rows
  // sequences per CTA, one until there are more than ~2 per SM); otherwise one thread per unit.
  const size_t wsm4 = sizeof(R) * (size_t)(4 * (H * (H + 1) + 8));
  const int rows4 = (int)std::max<long>(1, std::min<long>(1024 / H4, B / (2 * 148)));
  const bool Q4 = H % 8 == 0 && H4 <= 1024 && wsm4 + sizeof(R) * (size_t)rows4 * 4 * (H + 8) <= 200 * 1024 &&
                  g_lstm_quad;
  // sequences per CTA of the recurrence: one until there are more than ~2 per SM (each CTA reads Wh from
  // shared memory once per sequence and step, so fewer sequences per CTA means more SMs share that work)
  const int rows = Q4 ? rows4 : (int)std::max<long>(1, std::min<long>(std::min<long>(1024 / H, 8), B / (2 * 148)));
  const size_t wsm = sizeof(R) * (size_t)H4 * (H + 1);
  const bool WS = wsm + sizeof(R) * (size_t)rows * H4 <= 200 * 1024;
  const size_t smem_f = Q4 ? wsm4 + sizeof(R) * (size_t)rows * H : (WS ? wsm : 0) + sizeof(R) * (size_t)rows * H;
  const size_t smem_b =
      Q4 ? wsm4 + sizeof(R) * (size_t)rows * 4 * (H + 8) : (WS ? wsm : 0) + sizeof(R) * (size_t)rows * H4;
  auto kf = Q4 ? (tc ? lstm_fwd4_kernel<R, true> : lstm_fwd4_kernel<R, false>)
               : (WS ? (tc ? lstm_fwd_kernel<R, true, true> : lstm_fwd_kernel<R, true, false>)
                     : (tc ? lstm_fwd_kernel<R, false, true> : lstm_fwd_kernel<R, false, false>));
  auto kb = Q4 ? (tc ? lstm_bwd4_kernel<R, true> : lstm_bwd4_kernel<R, false>)
               : (WS ? (tc ? lstm_bwd_kernel<R, true, true> : lstm_bwd_kernel<R, true, false>)
                     : (tc ? lstm_bwd_kernel<R, false, true> : lstm_bwd_kernel<R, false, false>));
  const int threads = rows * (int)(Q4 ? H4 : H);
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    PL_CUDA(cudaFuncSetAttribute((const void*)kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_f));
    PL_CUDA(cudaFuncSetAttribute((const void*)kb, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_b));
  }
  const unsigned nb = (unsigned)ceil_div(B, rows);
  kf<<<nb, threads, smem_f, st>>>(Gin, Wh, bih, term, hc0, hc0 + B * H, II, FF, GG, OO, TC, HT, HP, CP, (int)B, (int)T,
                                  (int)H, rows);
  count_launch();
  PL_LAUNCH("lstm_fwd_kernel");
  // head: Out = HT Wo^T; row gradient; dHo = dOut Wo
  rc = lstm_gemm<R>((int)NR, (int)O, (int)H, HT, H, 1, Wo, H, 1, Out, O, 1, st, tc);
  if (rc) return rc;
  lstm_head_kernel<R><<<nblk(NR), 256, 0, st>>>(Out, bo, NR, (int)A, act, col, col + NR, col + 2 * NR, (R)vf, (R)ent,
                                                (R)clip, dOut, lpv, lpv + NR);
  count_launch();
  PL_LAUNCH("lstm_head_kernel");
  rc = lstm_gemm<R>((int)NR, (int)H, (int)O, dOut, O, 1, Wo, 1, H, dHo, H, 1, st, tc);
  if (rc) return rc;
  kb<<<nb, threads, smem_b, st>>>(II, FF, GG, OO, TC, CP, dHo, Wh, term, dG, (int)B, (int)T, (int)H, rows);
  count_launch();
  PL_LAUNCH("lstm_bwd_kernel");
  // ---- weight gradients over all rows: fixed row slices, summed in slice order
  double* gWx = g_d;
  double* gWh = gWx + H4 * D;
  double* gbih = gWh + H4 * H;
  double* gWo = gbih + H4;
  double* gbo = gWo + O * H;
  auto wgrad = [&](int M, int N, const R* Am, long acs_, const R* Bm, long bcs_, double* dst) -> int {
    int r2 = lstm_gemm<R>(M, N, (int)NR, Am, 1, acs_, Bm, 1, bcs_, part, N, NZ, st, tc);
    if (r2) return r2;
    lstm_slice_sum_kernel<R><<<nblk((long)M * N), 256, 0, st>>>(part, NZ, (long)M * N, dst);
    count_launch();
    PL_LAUNCH("lstm_slice_sum_kernel");
    return PL_OK;
  };
  rc = wgrad((int)H4, (int)D, dG, H4, X, D, gWx);
  if (!rc) rc = wgrad((int)H4, (int)H, dG, H4, HP, H, gWh);
  if (!rc) rc = wgrad((int)O, (int)H, dOut, O, HT, H, gWo);
  if (rc) return rc;
  auto colsum = [&](const R* Mx, int N, double* dst) -> int {
    dim3 grid((unsigned)ceil_div(N, 128), (unsigned)nch);
    lstm_colsum_part_kernel<R><<<grid, 128, 0, st>>>(Mx, NR, N, rows_per, cpart);
    lstm_slice_sum_kernel<R><<<nblk(N), 256, 0, st>>>(cpart, (int)nch, N, dst);
    count_launch(2);
    PL_LAUNCH("lstm_colsum");
    return PL_OK;
  };
  rc = colsum(dG, (int)H4, gbih);
  if (!rc) rc = colsum(dOut, (int)O, gbo);
  if (rc) return rc;
  PL_CUDA(cudaMemcpyAsync(g, g_d, sizeof(double) * P, cudaMemcpyDeviceToHost, st));
  if (newlp) PL_CUDA(cudaMemcpyAsync(newlp, lpv, sizeof(double) * NR, cudaMemcpyDeviceToHost, st));
  if (newval) PL_CUDA(cudaMemcpyAsync(newval, lpv + NR, sizeof(double) * NR, cudaMemcpyDeviceToHost, st));
  PL_CUDA(cudaStreamSynchronize(st));

  return device_error_check();
}

}  // namespace
}  // namespace pl

extern "C" {

int pl_lstm_ppo_grad_batch(const double* params, const double* obs, const double* acts, const double* advs,
                           const double* rets, const double* oldlps, const double* terms, const double* h0s,
                           const double* c0s, size_t B, size_t T, size_t H, size_t D, size_t A, double vfCoef,
                           double entCoef, double clipEps, int tier, double* g, double* newlp, double* newval) {
  using namespace pl;
  PL_REQUIRE(params && obs && acts && advs && rets && oldlps && terms && h0s && c0s && g, PL_ERR_INVALID,
             "pl_lstm_ppo_grad_batch: NULL argument");
  PL_REQUIRE(B > 0 && T > 0 && H > 0 && D > 0 && A > 0 && B * T < (1u << 28), PL_ERR_INVALID,
             "pl_lstm_ppo_grad_batch: bad extents B=%zu T=%zu H=%zu D=%zu A=%zu", B, T, H, D, A);
  PL_REQUIRE(H <= 1024 && tier >= 0 && tier <= 2, PL_ERR_INVALID, "pl_lstm_ppo_grad_batch: H=%zu tier=%d", H, tier);
  int rc = require_device();
  if (rc) return rc;
  if (tier == 0)
    return lstm_grad<double>(params, obs, acts, advs, rets, oldlps, terms, h0s, c0s, (long)B, (long)T, (long)H,
                             (long)D, (long)A, vfCoef, entCoef, clipEps, false, g, newlp, newval);
  return lstm_grad<float>(params, obs, acts, advs, rets, oldlps, terms, h0s, c0s, (long)B, (long)T, (long)H, (long)D,
                          (long)A, vfCoef, entCoef, clipEps, tier == 2, g, newlp, newval);
}

int pl_lstm_reuse_inputs(int on) {
  pl::g_reuse_inputs = on != 0;
  return PL_OK;
}

int pl_test_lstm_quad(int mode) {
  const int prev = pl::g_lstm_quad ? 1 : 0;
  if (mode >= 0) pl::g_lstm_quad = mode != 0;
  return prev;
}

}  // extern "C"
