// Memory-bound kernels of the MLP PPO+Muon update: column conversion, minibatch gather with the
// advantage statistics, fixed-order reductions (bias gradients, split-K slices, global grad
// norm), the Muon steps around Newton-Schulz (Nesterov, normalise, finalise into the f64 master
// weights and their bf16 shadow), and the fp32 SIMT kernels of the tight (bf16 = 0) tier.
//
// Every reduction has a fixed partition and a fixed fold order, so a run is bit-reproducible.
#include "pl_common.cuh"
#include "pl_gemm.cuh"
#include "pl_mlp.cuh"
#include "pl_runtime.h"

namespace pl {

constexpr int kStreamBlocks = 1184;  // 8 x 148 SMs: fixed partition of the streaming reductions (loads in flight)

__device__ __forceinline__ double block_sum_f64(double v, double* sh) {
  // fixed-shape tree over a 256-thread block
  const int t = threadIdx.x;
  sh[t] = v;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (t < s) sh[t] += sh[t + s];
    __syncthreads();
  }
  double r = sh[0];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------- columns
// obs rows (f64 or f32, D wide) -> bf16 rows Dp wide, zero padded.
template <typename T>
__global__ void __launch_bounds__(256) obs_to_bf16_kernel(const T* __restrict__ src, long NT, int D, int Dp,
                                                          __nv_bfloat16* dst) {
  // one warp per row; four values per lane and step (16- or 32-byte loads, an 8-byte store) when every
  // row starts aligned, else one value per lane
  const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const bool vec = (D % 4) == 0 && (Dp % 4) == 0 && ((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 7) == 0;
  for (long r = (long)blockIdx.x * wpb + (threadIdx.x >> 5); r < NT; r += (long)gridDim.x * wpb) {
    const T* s = src + r * D;
    __nv_bfloat16* d = dst + r * Dp;
    if (vec) {
      for (int c = lane * 4; c < Dp; c += 128) {
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (c < D) {
          if constexpr (sizeof(T) == 4) {
            const float4 q = *reinterpret_cast<const float4*>(s + c);
            v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
          } else {
            const double2 a = *reinterpret_cast<const double2*>(s + c);
            const double2 b = *reinterpret_cast<const double2*>(s + c + 2);
            v[0] = (float)a.x, v[1] = (float)a.y, v[2] = (float)b.x, v[3] = (float)b.y;
          }
        }
        __nv_bfloat162 o[2] = {__floats2bfloat162_rn(v[0], v[1]), __floats2bfloat162_rn(v[2], v[3])};
        *reinterpret_cast<uint2*>(d + c) = *reinterpret_cast<const uint2*>(o);
      }
    } else {
      for (int c = lane; c < Dp; c += 32) d[c] = __float2bfloat16_rn(c < D ? (float)s[c] : 0.f);
    }
  }
}
template <typename T>
__global__ void obs_to_f32_kernel(const T* __restrict__ src, long n, float* dst) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dst[i] = (float)src[i];
}
// scalar columns: act (f64 index) -> int32, perm (f64) -> int32, the rest f64 -> f32 (adv stays f64)
__global__ void columns_kernel(const double* __restrict__ act, const double* __restrict__ ret,
                               const double* __restrict__ olp, const double* __restrict__ ov, long NT, int* act_i,
                               float* ret_f, float* olp_f, float* ov_f) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < NT; i += (long)gridDim.x * blockDim.x) {
    act_i[i] = (int)act[i];
    if (ret) ret_f[i] = (float)ret[i];
    olp_f[i] = (float)olp[i];
    if (ov) ov_f[i] = (float)ov[i];
  }
}
__global__ void perm_kernel(const double* __restrict__ perm, long n, int* out) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    out[i] = (int)perm[i];
}
// pos[perm[k]] = k over the first NT entries (the first epoch's order); entries outside [0, NT) are
// skipped, so pos (zeroed before) stays in range.
__global__ void perm_inverse_kernel(const int* __restrict__ perm, long NT, int* pos) {
  for (long k = (long)blockIdx.x * blockDim.x + threadIdx.x; k < NT; k += (long)gridDim.x * blockDim.x) {
    const int p = perm[k];
    if (p >= 0 && p < NT) pos[p] = (int)k;
  }
}
// out[i] = pos[perm[i]]: row ids of later epochs' orders translated into first-epoch positions.
__global__ void perm_compose_kernel(const int* __restrict__ perm, const int* __restrict__ pos, long NT, long n,
                                    int* out) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int p = perm[i];
    out[i] = (p >= 0 && p < NT) ? pos[p] : 0;
  }
}

// ---------------------------------------------------------------- gather + advantage statistics
// Row k of the minibatch = column row idx[k]; its observation row is oidx[k] when the observations
// are stored in another order (oidx null: idx[k]; obs null: no observation copy). One warp per row for
// the obs copy (16-byte vectors); scalars by lane 0. Each block folds sum(adv), sum(adv^2) of its rows
// into part[blockIdx.x].
template <bool BF16>
__global__ void __launch_bounds__(256) gather_kernel(const int* __restrict__ idx, int Nmb, const void* __restrict__ obs,
                                                     int rowElems, void* X, const int* __restrict__ act_c,
                                                     const double* __restrict__ adv_c, const float* __restrict__ ret_c,
                                                     const float* __restrict__ olp_c, const float* __restrict__ ov_c,
                                                     int* mb_act, float* mb_adv, float* mb_ret, float* mb_olp,
                                                     float* mb_ov, double* part, const int* __restrict__ oidx) {
  __shared__ double sh[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_per_block = (Nmb + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * rows_per_block, r1 = min(Nmb, r0 + rows_per_block);
  double s1 = 0.0, s2 = 0.0;
  for (int k = r0 + warp; k < r1; k += 8) {
    const long src = idx[k];
    const int vec_elems = BF16 ? 8 : 4;  // 16 bytes
    // 16-byte vectors only when every row starts 16-byte aligned (always for the padded bf16 rows)
    const int nvec = (rowElems % vec_elems == 0) ? rowElems / vec_elems : 0;
    if (obs) {
      const long orow = oidx ? (long)oidx[k] : src;
      const uint4* s = reinterpret_cast<const uint4*>((const char*)obs + orow * rowElems * (BF16 ? 2 : 4));
      uint4* d = reinterpret_cast<uint4*>((char*)X + (long)k * rowElems * (BF16 ? 2 : 4));
      int v = lane;
      for (; v + 96 < nvec; v += 128) {  // four vectors per lane in flight: the loads before the stores
        const uint4 a0 = s[v], a1 = s[v + 32], a2 = s[v + 64], a3 = s[v + 96];
        d[v] = a0;
        d[v + 32] = a1;
        d[v + 64] = a2;
        d[v + 96] = a3;
      }
      for (; v < nvec; v += 32) d[v] = s[v];
      if (!BF16) {
        const float* sf = (const float*)obs + orow * rowElems;
        float* df = (float*)X + (long)k * rowElems;
        for (int c = nvec * 4 + lane; c < rowElems; c += 32) df[c] = sf[c];
      }
    }
    if (lane == 0) {
      const double a = adv_c[src];
      mb_act[k] = act_c[src];
      mb_adv[k] = (float)a;
      mb_ret[k] = ret_c[src];
      mb_olp[k] = olp_c[src];
      if (mb_ov) mb_ov[k] = ov_c[src];
      s1 += a;
      s2 += a * a;
    }
  }
  s1 = block_sum_f64(s1, sh);
  s2 = block_sum_f64(s2, sh);
  if (threadIdx.x == 0) {
    part[2 * blockIdx.x] = s1;
    part[2 * blockIdx.x + 1] = s2;
  }
}
// Sum of p[b * stride] over b < n by one warp in a fixed order: lane l folds b = l, l + 32, ... in turn,
// then a butterfly adds the lanes; every lane returns the total.
__device__ __forceinline__ double warp_fold_f64(const double* __restrict__ p, int n, int stride) {
  const int lane = threadIdx.x & 31;
  double s = 0.0;
  for (int b = lane; b < n; b += 32) s += p[(long)b * stride];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}
// ms = [mean, std + 1e-8] (population std), folded over the block partials (one warp).
__global__ void adv_stats_kernel(const double* __restrict__ part, int nb, int n, double* ms) {
  if (blockIdx.x || threadIdx.x >= 32) return;
  const double s1 = warp_fold_f64(part, nb, 2), s2 = warp_fold_f64(part + 1, nb, 2);
  if (threadIdx.x) return;
  const double mean = s1 / (double)n;
  double var = s2 / (double)n - mean * mean;
  if (var < 0.0) var = 0.0;
  ms[0] = mean;
  ms[1] = sqrt(var) + 1e-8;
}

// Data-parallel form: the local (sum, sum of squares, count) folded in order, to be all-reduced.
__global__ void adv_sums_kernel(const double* __restrict__ part, int nb, int n, double* sums) {
  if (blockIdx.x || threadIdx.x >= 32) return;
  const double s1 = warp_fold_f64(part, nb, 2), s2 = warp_fold_f64(part + 1, nb, 2);
  if (threadIdx.x) return;
  sums[0] = s1;
  sums[1] = s2;
  sums[2] = (double)n;
}
__global__ void adv_ms_from_sums_kernel(const double* __restrict__ sums, double* ms) {
  if (threadIdx.x || blockIdx.x) return;
  const double n = sums[2];
  const double mean = sums[0] / n;
  double var = sums[1] / n - mean * mean;
  if (var < 0.0) var = 0.0;
  ms[0] = mean;
  ms[1] = sqrt(var) + 1e-8;
}

// ---------------------------------------------------------------- fixed-order reductions
// out[c] = sum over t of part[t*ld + c] (bias gradients from per-CTA column partials), in two
// fixed-order levels: blockIdx.y sums its run of kColChunk tiles (t ascending) into part2, then
// colsum_final_kernel sums the runs in order. Spreading the tiles over blockIdx.y keeps every SM
// streaming instead of leaving one thread per column to walk thousands of tiles.
constexpr int kColChunk = 32;
__global__ void colsum_reduce_kernel(const float* __restrict__ part, int tiles, long ld, int ncols, float* part2) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= ncols) return;
  const int t0 = blockIdx.y * kColChunk, t1 = min(tiles, t0 + kColChunk);
  float s = 0.f;
  for (int t = t0; t < t1; t++) s += part[(long)t * ld + c];
  part2[(long)blockIdx.y * ncols + c] = s;
}
__global__ void colsum_final_kernel(const float* __restrict__ part2, int runs, long ld, int ncols, float* out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= ncols) return;
  float s = 0.f;
  for (int r = 0; r < runs; r++) s += part2[(long)r * ld + c];
  out[c] = s;
}
// out[i] = sum_s part[s*n + i], s ascending (split-K slices)
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int S, long n, float* out) {
  // four adjacent outputs per thread and step (16-byte loads and store) where the slices allow it;
  // every output still sums its slices in order z = 0, 1, ...
  const long stride = (long)gridDim.x * blockDim.x, t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long n4 = ((n & 3) == 0 && ((uintptr_t)part & 15) == 0 && ((uintptr_t)out & 15) == 0) ? n / 4 : 0;
  for (long i = t; i < n4; i += stride) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int z = 0; z < S; z++) {
      const float4 p = reinterpret_cast<const float4*>(part + (long)z * n)[i];
      s.x += p.x;
      s.y += p.y;
      s.z += p.z;
      s.w += p.w;
    }
    reinterpret_cast<float4*>(out)[i] = s;
  }
  for (long i = n4 * 4 + t; i < n; i += stride) {
    float s = 0.f;
    for (int z = 0; z < S; z++) s += part[(long)z * n + i];
    out[i] = s;
  }
}
// The same sum for many slices over few outputs (S >= 32, n a multiple of 4): one warp per four
// adjacent outputs, lane l sums slices l, l + 32, ... in order, then a fixed butterfly adds the lanes.
__global__ void splitk_reduce_warp_kernel(const float* __restrict__ part, int S, long n4, float* out) {
  const long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= n4) return;  // whole warps leave together
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int z = lane; z < S; z += 32) {
    const float4 p = reinterpret_cast<const float4*>(part + (long)z * n4 * 4)[w];
    s.x += p.x;
    s.y += p.y;
    s.z += p.z;
    s.w += p.w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s.x += __shfl_xor_sync(0xffffffffu, s.x, o);
    s.y += __shfl_xor_sync(0xffffffffu, s.y, o);
    s.z += __shfl_xor_sync(0xffffffffu, s.z, o);
    s.w += __shfl_xor_sync(0xffffffffu, s.w, o);
  }
  if (lane == 0) reinterpret_cast<float4*>(out)[w] = s;
}
// Global gradient norm of g*sc: fixed grid of kStreamBlocks blocks x 256 threads, strided f64 sums.
__global__ void __launch_bounds__(256) gradnorm_part_kernel(const float* __restrict__ g, long P, double sc,
                                                            double* part) {
  __shared__ double sh[256];
  double s = 0.0;
  const long S = (long)gridDim.x * 256;
  long i = (long)blockIdx.x * 256 + threadIdx.x;
  for (; i + 3 * S < P; i += 4 * S) {  // four strides' loads in flight, summed in stride order
    const float a[4] = {g[i], g[i + S], g[i + 2 * S], g[i + 3 * S]};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const double x = (double)a[q] * sc;
      s += x * x;
    }
  }
  for (; i < P; i += S) {
    const double x = (double)g[i] * sc;
    s += x * x;
  }
  s = block_sum_f64(s, sh);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}
// cc = (maxNorm > 0 && gnorm > maxNorm ? maxNorm/gnorm : 1) * sc   (maxNorm <= 0: cc = sc)
__global__ void gradnorm_final_kernel(const double* __restrict__ part, int nb, double maxNorm, double sc, double* cc) {
  if (blockIdx.x || threadIdx.x >= 32) return;
  const double s = warp_fold_f64(part, nb, 1);
  if (threadIdx.x) return;
  const double gnorm = sqrt(s);
  cc[0] = ((maxNorm > 0.0 && gnorm > maxNorm) ? maxNorm / gnorm : 1.0) * sc;
  cc[1] = gnorm;
}

// ---------------------------------------------------------------- Muon around Newton-Schulz
// m <- mu*m + g*cc ; u = g*cc + mu*m (f64); per-block partial sums of u^2 (fixed grid).
__global__ void __launch_bounds__(256) nesterov_kernel(const float* __restrict__ g, const double* __restrict__ cc,
                                                       double* mom, double* u, double mu, long n, double* part) {
  __shared__ double sh[256];
  const double c = cc[0];
  double s = 0.0;
  const long S = (long)gridDim.x * 256;
  long i = (long)blockIdx.x * 256 + threadIdx.x;
  // four grid strides' loads in flight at once; the sum still takes them in stride order
  for (; i + 3 * S < n; i += 4 * S) {
    float gv[4];
    double mv[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      gv[q] = g[i + q * S];
      mv[q] = mom[i + q * S];
    }
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const double gi = (double)gv[q] * c;
      const double m = mu * mv[q] + gi;
      mom[i + q * S] = m;
      const double ui = gi + mu * m;
      u[i + q * S] = ui;
      s += ui * ui;
    }
  }
  for (; i < n; i += S) {
    const double gi = (double)g[i] * c;
    const double m = mu * mom[i] + gi;
    mom[i] = m;
    const double ui = gi + mu * m;
    u[i] = ui;
    s += ui * ui;
  }
  s = block_sum_f64(s, sh);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}
// X = u / (||u||_F + eps) as bf16, stored wide: for rows > cols (TR) the matrix is transposed so
// that X is min(rows,cols) x max(rows,cols) with the long side contiguous (ld = ldx). Blocks walk
// rows (no per-element index division); the transposed form goes through 32 x 32 shared-memory tiles
// so that both the reads of u and the writes of X are coalesced. 256 threads per block.
template <bool TR>
__global__ void __launch_bounds__(256) ns_input_kernel(const double* __restrict__ u, const double* __restrict__ part,
                                                       int nparts, int rows, int cols, double eps, __nv_bfloat16* X,
                                                       long ldx) {
  __shared__ double inv_s;
  __shared__ __nv_bfloat16 tile[32][34];
  if (threadIdx.x < 32) {
    const double s = warp_fold_f64(part, nparts, 1);
    if (threadIdx.x == 0) inv_s = 1.0 / (sqrt(s) + eps);
  }
  __syncthreads();
  const double inv = inv_s;
  if (!TR) {
    const int B = blockDim.x;
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
      const double* ur = u + (long)r * cols;
      __nv_bfloat16* xr = X + (long)r * ldx;
      int c = threadIdx.x;
      for (; c + 3 * B < cols; c += 4 * B) {  // four loads in flight per thread
        const double a[4] = {ur[c], ur[c + B], ur[c + 2 * B], ur[c + 3 * B]};
#pragma unroll
        for (int q = 0; q < 4; q++) xr[c + q * B] = __float2bfloat16_rn((float)(inv * a[q]));
      }
      for (; c < cols; c += B) xr[c] = __float2bfloat16_rn((float)(inv * ur[c]));
    }
    return;
  }
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int tcols = (cols + 31) >> 5, ntiles = ((rows + 31) >> 5) * tcols;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {  // block-uniform trip count
    const int r0 = (t / tcols) * 32, c0 = (t % tcols) * 32;
    for (int j = ty; j < 32; j += 8) {
      const int r = r0 + j, c = c0 + tx;
      if (r < rows && c < cols) tile[j][tx] = __float2bfloat16_rn((float)(inv * u[(long)r * cols + c]));
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
      const int c = c0 + j, r = r0 + tx;
      if (r < rows && c < cols) X[(long)c * ldx + r] = tile[tx][j];
    }
    __syncthreads();
  }
}
// W <- c1*W + c2*X (f64 master, rows x cols row-major) and the bf16 shadow Wb (ldw), from the
// fp32 Newton-Schulz result Xf (wide layout, ldx; transposed back when rows > cols: TR, through
// 32 x 32 shared-memory tiles). 256 threads per block.
template <bool TR>
__global__ void __launch_bounds__(256) ns_finalize_kernel(const float* __restrict__ Xf, long ldx, int rows, int cols,
                                                          double c1, double c2, double* W, __nv_bfloat16* Wb,
                                                          long ldw) {
  if (!TR) {
    for (int r = blockIdx.x; r < rows; r += gridDim.x)
      for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const long i = (long)r * cols + c;
        const double w = c1 * W[i] + c2 * (double)Xf[(long)r * ldx + c];
        W[i] = w;
        if (Wb) Wb[(long)r * ldw + c] = __float2bfloat16_rn((float)w);
      }
    return;
  }
  __shared__ float tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int tcols = (cols + 31) >> 5, ntiles = ((rows + 31) >> 5) * tcols;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {  // block-uniform trip count
    const int r0 = (t / tcols) * 32, c0 = (t % tcols) * 32;
    for (int j = ty; j < 32; j += 8) {
      const int c = c0 + j, r = r0 + tx;
      if (r < rows && c < cols) tile[j][tx] = Xf[(long)c * ldx + r];
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
      const int r = r0 + j, c = c0 + tx;
      if (r < rows && c < cols) {
        const long i = (long)r * cols + c;
        const double w = c1 * W[i] + c2 * (double)tile[tx][j];
        W[i] = w;
        if (Wb) Wb[(long)r * ldw + c] = __float2bfloat16_rn((float)w);
      }
    }
    __syncthreads();
  }
}
// ---------------------------------------------------------------- Muon of a group of equal-shape layers
// The bf16 tier's Muon around Newton-Schulz in three launches per group (blockIdx.y = layer): the
// Nesterov step writes the Newton-Schulz input X = bf16(u) directly, unscaled, with per-block sums of
// u^2; one warp per layer turns them into the first step's factors 1 / (||u|| + eps) and its square
// (applied in that step's G and X' epilogues); the finalisation applies the result and the bias step.
// Per weight element that is 4 + 8 + 8 + 2 bytes for the first phase (gradient, momentum in and out, X)
// where a separate normalisation pass would also write and re-read u in f64.

// The Nesterov arithmetic of one element, in the reference's order (m <- mu m + g cc; u = g cc + mu m).
__device__ __forceinline__ double nesterov_u(float g, double c, double mu, double& m) {
  const double gi = (double)g * c;
  m = mu * m + gi;
  return gi + mu * m;
}

template <bool TR>
__global__ void __launch_bounds__(256) muon_x0_kernel(const MuonGroupArgs a, const double* __restrict__ cc, double mu,
                                                      double* part) {
  __shared__ double sh[256];
  __shared__ float tile[32][33];
  const int q = blockIdx.y;
  const float* __restrict__ g = a.gW[q];
  double* __restrict__ mom = a.mW[q];
  __nv_bfloat16* X = a.X[q];
  const double c = cc[0];
  const int rows = a.rows, cols = a.cols;
  double s = 0.0;
  if (!TR) {
    constexpr int B = 256;
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
      const float* gr = g + (long)r * cols;
      double* mr = mom + (long)r * cols;
      __nv_bfloat16* xr = X ? X + (long)r * a.ldx : nullptr;
      int k = threadIdx.x;
      for (; k + 3 * B < cols; k += 4 * B) {  // four elements' loads in flight per thread
        float gv[4];
        double mv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          gv[j] = gr[k + j * B];
          mv[j] = mr[k + j * B];
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const double ui = nesterov_u(gv[j], c, mu, mv[j]);
          mr[k + j * B] = mv[j];
          s += ui * ui;
          if (xr) xr[k + j * B] = __float2bfloat16_rn((float)ui);
        }
      }
      for (; k < cols; k += B) {
        double m = mr[k];
        const double ui = nesterov_u(gr[k], c, mu, m);
        mr[k] = m;
        s += ui * ui;
        if (xr) xr[k] = __float2bfloat16_rn((float)ui);
      }
    }
  } else {
    // rows > cols: X is cols x ldx; 32 x 32 tiles through shared memory so that the momentum reads
    // and the transposed X writes are both coalesced
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int tcols = (cols + 31) >> 5, ntiles = ((rows + 31) >> 5) * tcols;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {  // block-uniform trip count
      const int r0 = (t / tcols) * 32, c0 = (t % tcols) * 32;
      const int cc0 = c0 + tx;
      float gv[4];
      double mv[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int r = r0 + ty + 8 * j;
        const bool ok = r < rows && cc0 < cols;
        gv[j] = ok ? g[(long)r * cols + cc0] : 0.f;
        mv[j] = ok ? mom[(long)r * cols + cc0] : 0.0;
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int r = r0 + ty + 8 * j;
        float v = 0.f;
        if (r < rows && cc0 < cols) {
          const double ui = nesterov_u(gv[j], c, mu, mv[j]);
          mom[(long)r * cols + cc0] = mv[j];
          s += ui * ui;
          v = (float)ui;
        }
        tile[ty + 8 * j][tx] = v;
      }
      __syncthreads();
      if (X)
        for (int j = ty; j < 32; j += 8) {
          const int cx = c0 + j, r = r0 + tx;
          if (r < rows && cx < cols) X[(long)cx * a.ldx + r] = __float2bfloat16_rn(tile[tx][j]);
        }
      __syncthreads();
    }
  }
  if (part) {
    s = block_sum_f64(s, sh);
    if (threadIdx.x == 0) part[(long)q * gridDim.x + blockIdx.x] = s;
  }
}

// One warp per layer: the layer's partials folded in block order.
__global__ void muon_scale_kernel(const double* __restrict__ part, int blocks, int nb, double eps, float* scale) {
  const int q = blockIdx.x;
  const double s = warp_fold_f64(part + (long)q * blocks, blocks, 1);
  if (threadIdx.x == 0) {
    const double inv = 1.0 / (sqrt(s) + eps);
    scale[q] = (float)inv;
    scale[nb + q] = (float)(inv * inv);
  }
}

template <bool TR>
__global__ void __launch_bounds__(256) muon_finalize_kernel(const MuonGroupArgs a, double c1, double c2,
                                                            const double* __restrict__ cc, double lr, double wd,
                                                            double mu) {
  __shared__ float tile[32][33];
  const int q = blockIdx.y;
  const float* __restrict__ Xf = a.Xf[q];
  double* __restrict__ W = a.W[q];
  __nv_bfloat16* Wb = a.Wb[q];
  const int rows = a.rows, cols = a.cols;
  if (blockIdx.x == 0 && a.b[q]) {  // the bias: stepVec on g cc, as the f64 reference orders it
    const double c = cc[0];
    for (int i = threadIdx.x; i < rows; i += blockDim.x) {
      double m = a.mb[q][i];
      const double upd = nesterov_u(a.gb[q][i], c, mu, m);
      const double nbv = a.b[q][i] * (1.0 - lr * wd) + lr * upd;
      a.b[q][i] = nbv;
      a.mb[q][i] = m;
      if (a.bf[q]) a.bf[q][i] = (float)nbv;
    }
  }
  if (!TR) {
    constexpr int B = 256;
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
      const float* xr = Xf + (long)r * a.ldx;
      double* wr = W + (long)r * cols;
      __nv_bfloat16* br = Wb ? Wb + (long)r * a.ldw : nullptr;
      int k = threadIdx.x;
      for (; k + 3 * B < cols; k += 4 * B) {
        float xv[4];
        double wv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          xv[j] = xr[k + j * B];
          wv[j] = wr[k + j * B];
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const double w = c1 * wv[j] + c2 * (double)xv[j];
          wr[k + j * B] = w;
          if (br) br[k + j * B] = __float2bfloat16_rn((float)w);
        }
      }
      for (; k < cols; k += B) {
        const double w = c1 * wr[k] + c2 * (double)xr[k];
        wr[k] = w;
        if (br) br[k] = __float2bfloat16_rn((float)w);
      }
    }
    return;
  }
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int tcols = (cols + 31) >> 5, ntiles = ((rows + 31) >> 5) * tcols;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {  // block-uniform trip count
    const int r0 = (t / tcols) * 32, c0 = (t % tcols) * 32;
    for (int j = ty; j < 32; j += 8) {
      const int cx = c0 + j, r = r0 + tx;
      if (r < rows && cx < cols) tile[j][tx] = Xf[(long)cx * a.ldx + r];
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
      const int r = r0 + j, cx = c0 + tx;
      if (r < rows && cx < cols) {
        const long i = (long)r * cols + cx;
        const double w = c1 * W[i] + c2 * (double)tile[tx][j];
        W[i] = w;
        if (Wb) Wb[(long)r * a.ldw + cx] = __float2bfloat16_rn((float)w);
      }
    }
    __syncthreads();
  }
}
// f64 master weights -> bf16 shadow (padded, ld) / fp32 copies
__global__ void w_to_bf16_kernel(const double* __restrict__ W, int rows, int cols, __nv_bfloat16* Wb, long ldw) {
  for (int r = blockIdx.x; r < rows; r += gridDim.x)
    for (int c = threadIdx.x; c < cols; c += blockDim.x)
      Wb[(long)r * ldw + c] = __float2bfloat16_rn((float)W[(long)r * cols + c]);
}
__global__ void f64_to_f32_kernel(const double* __restrict__ s, long n, float* d) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) d[i] = (float)s[i];
}
__global__ void f32_to_f64_kernel(const float* __restrict__ s, long n, double* d) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) d[i] = (double)s[i];
}

// ---------------------------------------------------------------- tight tier (fp32 SIMT)
// C[m,n] = alpha * sum_k A(m,k) B(n,k), A(m,k) = A[m*ars + k*acs], B(n,k) = B[n*brs + k*bcs]. Split K:
// blockIdx.z sums k in [z*kc, (z+1)*kc) into C + z*cz (kc = K and cz = 0 without a split).
// Epilogues (SE): SGEMM_PLAIN stores alpha * acc; SGEMM_BIAS_ACT stores Z = acc + bias[n] into C and
// act(Z) into X (bias_act_f32_kernel's arithmetic); SGEMM_ACT_GRAD stores acc * act'(X[m, n]) with X
// the pre-activation (act_grad_f32_kernel's). ones_col >= 0 makes column ones_col of B all ones
// (the weight-gradient split then also sums the bias gradient, as one more output column).
enum { SGEMM_PLAIN = 0, SGEMM_BIAS_ACT = 1, SGEMM_ACT_GRAD = 2 };
template <int SE>
__global__ void __launch_bounds__(256) sgemm_kernel(int M, int N, int K, const float* __restrict__ A, long ars, long acs,
                                                    const float* __restrict__ B, long brs, long bcs, float* C, long ldc,
                                                    float alpha, int kc, long cz, int ones_col,
                                                    const float* __restrict__ bias, float* X, int act) {
  __shared__ float As[16][65], Bs[16][65];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int kb = blockIdx.z * kc, ke = min(K, kb + kc);
  C += blockIdx.z * cz;
  float acc[4][4] = {};
  for (int k0 = kb; k0 < ke; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i / 64, mm = i % 64;
      const int m = m0 + mm, n = n0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < ke) ? A[(long)m * ars + (long)k * acs] : 0.f;
      Bs[kk][mm] = (n < N && k < ke) ? (n == ones_col ? 1.f : B[(long)n * brs + (long)k * bcs]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; kk++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        a[i] = As[kk][ty * 4 + i];
        b[i] = Bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] += a[i] * b[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < M && n < N) {
        const long o = (long)m * ldc + n;
        if constexpr (SE == SGEMM_BIAS_ACT) {
          const float z = acc[i][j] + bias[n];
          C[o] = z;
          X[o] = act_fwd(z, act);
        } else if constexpr (SE == SGEMM_ACT_GRAD) {
          const float d = alpha * acc[i][j], z = X[o];
          C[o] = (act == 0) ? (z > 0.f ? d : 0.f) : (act == 2 ? d : d * act_grad(z, act));
        } else {
          C[o] = alpha * acc[i][j];
        }
      }
    }
}
// Out[r, o] = sum_k H[r, k] W[o, k] + b[o] for a few outputs (O <= kSkinnyO) over K a multiple of 4:
// one warp per row, each lane a strided run of 16-byte pieces of the row, then a fixed butterfly per
// output. W and b sit in shared memory.
constexpr int kSkinnyO = 8, kSkinnyK = 1024;  // W in shared memory: 32 KB
__global__ void __launch_bounds__(256) skinny_rows_kernel(const float* __restrict__ H, int rows, int K,
                                                          const float* __restrict__ W, const float* __restrict__ b,
                                                          int O, float* Out) {
  __shared__ float4 sW[kSkinnyO * kSkinnyK / 4];
  __shared__ float sb[kSkinnyO];
  const int K4 = K / 4;
  for (int i = threadIdx.x; i < O * K4; i += blockDim.x) sW[i] = reinterpret_cast<const float4*>(W)[i];
  if (threadIdx.x < O) sb[threadIdx.x] = b[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long wpb = blockDim.x >> 5;
  for (long r = (long)blockIdx.x * wpb + (threadIdx.x >> 5); r < rows; r += (long)gridDim.x * wpb) {
    const float4* h = reinterpret_cast<const float4*>(H + r * K);
    float acc[kSkinnyO];
#pragma unroll
    for (int o = 0; o < kSkinnyO; o++) acc[o] = 0.f;
    for (int q = lane; q < K4; q += 32) {
      const float4 x = h[q];
#pragma unroll
      for (int o = 0; o < kSkinnyO; o++) {
        if (o < O) {
          const float4 w = sW[o * K4 + q];
          acc[o] += x.x * w.x + x.y * w.y + x.z * w.z + x.w * w.w;
        }
      }
    }
#pragma unroll
    for (int o = 0; o < kSkinnyO; o++) {
#pragma unroll
      for (int off = 16; off; off >>= 1) acc[o] += __shfl_xor_sync(0xffffffffu, acc[o], off);
    }
    if (lane < O) {
      float v = acc[0];
#pragma unroll
      for (int o = 1; o < kSkinnyO; o++)
        if (lane == o) v = acc[o];
      Out[r * O + lane] = v + sb[lane];
    }
  }
}
// Weight and bias gradient partials of a small layer (out + in <= 192): block z copies rows
// [64 z, 64 z + 64) of dZ (ldz) and Hin (ldh) into shared memory with coalesced loads, then each thread
// sums its outputs (o, c) over those rows in row order, c = in being the bias (a column of ones), into
// part[z][o][c]; splitk_reduce_wb_kernel sums the slices.
constexpr int kWgRows = 64, kWgMaxCols = 192;
__global__ void __launch_bounds__(256) wgrad_small_kernel(int out, int in, int K, const float* __restrict__ dZ,
                                                          long ldz, const float* __restrict__ Hin, long ldh,
                                                          float* part) {
  __shared__ __align__(16) float sm[kWgRows * kWgMaxCols];
  float* sZ = sm;                   // [rows][out]
  float* sH = sm + kWgRows * out;   // [rows][in] (16-byte aligned when out is a multiple of 4)
  const int r0 = blockIdx.x * kWgRows, nr = min(kWgRows, K - r0);
  // dense rows (ld = width) make the slice one contiguous block: 16-byte loads, several in flight
  auto stage = [&](const float* __restrict__ src, long ld, int w, float* dst) {
    const float* base = src + (long)r0 * ld;
    const int n = nr * w;
    if (ld == w && (n & 3) == 0 && ((uintptr_t)base & 15) == 0 && ((uintptr_t)dst & 15) == 0) {
      const float4* s4 = reinterpret_cast<const float4*>(base);
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll 4
      for (int i = threadIdx.x; i < n / 4; i += blockDim.x) d4[i] = s4[i];
    } else {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int r = i / w, c = i - r * w;
        dst[i] = base[(long)r * ld + c];
      }
    }
  };
  stage(dZ, ldz, out, sZ);
  stage(Hin, ldh, in, sH);
  __syncthreads();
  const int n = in + 1, total = out * n;
  float* dst = part + (long)blockIdx.x * total;
  for (int q = threadIdx.x; q < total; q += blockDim.x) {
    const int o = q / n, c = q - o * n;
    float acc = 0.f;
    if (c < in) {
      for (int r = 0; r < nr; r++) acc += sZ[r * out + o] * sH[r * in + c];
    } else {
      for (int r = 0; r < nr; r++) acc += sZ[r * out + o];
    }
    dst[q] = acc;
  }
}
// Split-K slices of a weight gradient with its bias column: part[s][m][in + 1]; out dW[m][in] and
// db[m], each the sum over s in a fixed order (lane-strided runs, then a butterfly), one warp per output.
__global__ void splitk_reduce_wb_kernel(const float* __restrict__ part, int S, int M, int in, float* dW, float* db) {
  const long n = (long)M * (in + 1);
  const long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= n) return;  // whole warps leave together
  float s = 0.f;
  for (int z = lane; z < S; z += 32) s += part[(long)z * n + w];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    const int m = (int)(w / (in + 1)), c = (int)(w % (in + 1));
    if (c < in)
      dW[(long)m * in + c] = s;
    else
      db[m] = s;
  }
}
// Z <- Z + b (row-major M x N), H = act(Z)
__global__ void bias_act_f32_kernel(float* Z, float* H, const float* __restrict__ b, long M, int N, int act) {
  const long n = M * N;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float z = Z[i] + b[i % N];
    Z[i] = z;
    if (H) H[i] = act_fwd(z, act);
  }
}
// dZ = dH * act'(Z)
__global__ void act_grad_f32_kernel(float* dH, const float* __restrict__ Z, long n, int act) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dH[i] = (act == 0) ? (Z[i] > 0.f ? dH[i] : 0.f) : (act == 2 ? dH[i] : dH[i] * act_grad(Z[i], act));
}
// Per-row PPO objective gradient on fp32 logits Out[M x O] (the reference's k_ppo_dout math,
// ffi/puffercuda.cu:171-185, with the value clip of :133-141): dOut[M x O].
__global__ void ppo_rows_f32_kernel(const float* __restrict__ Out, int M, int A, const int* __restrict__ act,
                                    const float* __restrict__ adv, const double* __restrict__ ms,
                                    const float* __restrict__ ret, const float* __restrict__ olp,
                                    const float* __restrict__ ov, float vf, float ent, float clip, float vfclip,
                                    float* dOut, float* newlp, float* newval) {
  int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= M) return;
  const int O = A + 1;
  const float* out = Out + (long)n * O;
  float* d = dOut + (long)n * O;
  const int a = act[n];
  float ad = adv[n];
  if (ms) ad = (float)(((double)ad - ms[0]) / ms[1]);
  const float rt = ret[n], ol = olp[n];
  float se = 0.f;
  for (int k = 0; k < A; k++) se += expf(out[k]);
  const float lse = logf(se);
  float pout = 0.f;
  for (int k = 0; k < A; k++) pout += expf(out[k] - lse) * out[k];
  const float logpA = out[a] - lse, ratio = expf(logpA - ol);
  const float lo = 1.f - clip, hi = 1.f + clip;
  const float rc = ratio < lo ? lo : (ratio > hi ? hi : ratio);
  const float s1 = ad * ratio, s2 = ad * rc;
  const float dPol = (s1 <= s2) ? ad * ratio : ad * ((lo < ratio && ratio < hi) ? 1.f : 0.f) * ratio;
  for (int k = 0; k < A; k++) {
    const float p = expf(out[k] - lse);
    d[k] = dPol * ((k == a ? 1.f : 0.f) - p) + ent * p * (pout - out[k]);
  }
  const float vnew = out[A];
  float dv = vnew - rt;
  if (ov && vfclip > 0.f) {
    const float vold = ov[n], dd = vnew - vold;
    const float vcl = vold + (dd < -vfclip ? -vfclip : (dd > vfclip ? vfclip : dd));
    if (!((vnew - rt) * (vnew - rt) >= (vcl - rt) * (vcl - rt)) && !(dd > -vfclip && dd < vfclip)) dv = 0.f;
  }
  d[A] = -vf * dv;
  if (newlp) newlp[n] = logpA;
  if (newval) newval[n] = vnew;
}
// ---------------------------------------------------------------- wide action heads
// Per-row PPO objective gradient of the multi-discrete (mode 1) and Gaussian (mode 2) heads, the
// resident wide update's k_ppo_dout_md / k_ppo_dout_cont (ffi/puffercuda.cu:706-727, 1767-1790):
//  mode 1: W categorical heads of sizes hs[0..W) over the first sum(hs) logits; the joint log-prob is
//          the sum of the heads' (log-softmax without max subtraction, as the reference); one clip on
//          the joint ratio; each head's logits get dPol (onehot - p) + ent p (sum p l - l);
//  mode 2: W dims, out = [means (W) | raw log-stds (W) | value]; log-std clamped to [lslo, lshi];
//          d/dmean = dPol z / std, d/draw-logstd = (dPol (z^2 - 1) + ent) inside the clamp, 0 outside;
// value (column O-1) with the PufferLib value clip when ov != NULL and vfclip > 0. Out has ld `ldo`
// and gets `bias` added when it is not NULL (the fast tier's GEMM writes no bias); the advantage is
// normalised with ms = [mean, std + 1e-8] when ms != NULL. dOut [M x ldd] (zero past O). Each
// 128-row block also writes its column sums of dOut (colpart[blockIdx.x][c], c < ldd) and its six
// loss sums (loss_part[blockIdx.x][0..5]: pg, value, entropy, kl, old kl, clipped).
template <typename S>
__device__ __forceinline__ void st_elem(S* p, long i, float v);
template <>
__device__ __forceinline__ void st_elem<float>(float* p, long i, float v) {
  p[i] = v;
}
template <>
__device__ __forceinline__ void st_elem<__nv_bfloat16>(__nv_bfloat16* p, long i, float v) {
  p[i] = __float2bfloat16_rn(v);
}
// The action of one multi-discrete head as a logit index, held inside the head so that a malformed
// action column cannot read past the row (valid actions are unchanged).
__device__ __forceinline__ int head_action(float a, int sz) {
  const int i = (int)a;
  return i < 0 ? 0 : (i >= sz ? sz - 1 : i);
}
template <typename S>
__global__ void __launch_bounds__(128) ppo_rows_wide_kernel(
    const float* __restrict__ Out, int ldo, const float* __restrict__ bias, int M, int O, int ldd, int mode, int W,
    const int* __restrict__ hs, const float* __restrict__ actw, const float* __restrict__ adv,
    const double* __restrict__ ms, const float* __restrict__ ret, const float* __restrict__ olp,
    const float* __restrict__ ov, float vf, float ent, float clip, float vfclip, float lslo, float lshi, S* dOut,
    float* colpart, float* loss_part) {
  __shared__ float red[4][128];
  __shared__ float lred[4][8];
  const int n = blockIdx.x * 128 + threadIdx.x;
  const bool ok = n < M;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* out = Out + (long)(ok ? n : 0) * ldo;
  auto lg = [&](int k) { return out[k] + (bias ? bias[k] : 0.f); };
  float ad = ok ? adv[n] : 0.f;
  if (ms && ok) ad = (float)(((double)ad - ms[0]) / ms[1]);
  const float* a = actw + (long)(ok ? n : 0) * W;
  // joint log-prob and the entropy of the row
  float logp = 0.f, entr = 0.f;
  if (mode == 1) {
    int off = 0;
    for (int h = 0; h < W; h++) {
      const int sz = hs[h];
      float se = 0.f;
      for (int k = 0; k < sz; k++) se += expf(lg(off + k));
      const float lse = logf(se);
      logp += lg(off + head_action(a[h], sz)) - lse;
      float pout = 0.f;
      for (int k = 0; k < sz; k++) pout += expf(lg(off + k) - lse) * lg(off + k);
      entr += lse - pout;
      off += sz;
    }
  } else {
    for (int i = 0; i < W; i++) {
      const float lsr = lg(W + i);
      const float ls = lsr < lslo ? lslo : (lsr > lshi ? lshi : lsr);
      const float z = (a[i] - lg(i)) * expf(-ls);
      logp += -0.5f * z * z - ls - 0.9189385332046727f;
      entr += ls + 1.4189385332046727f;
    }
  }
  const float lgr = logp - (ok ? olp[n] : 0.f);
  const float ratio = expf(lgr);
  const float lo = 1.f - clip, hi = 1.f + clip;
  const float rc = ratio < lo ? lo : (ratio > hi ? hi : ratio);
  const float s1 = ad * ratio, s2 = ad * rc;
  const float dPol = s1 <= s2 ? ad * ratio : ad * ((lo < ratio && ratio < hi) ? 1.f : 0.f) * ratio;
  const float vnew = lg(O - 1), rt = ok ? ret[n] : 0.f;
  float dv = vnew - rt, vl = 0.5f * (vnew - rt) * (vnew - rt);
  if (ov && vfclip > 0.f && ok) {
    const float vold = ov[n], dd = vnew - vold;
    const float vcl = vold + (dd < -vfclip ? -vfclip : (dd > vfclip ? vfclip : dd));
    const float du = (vnew - rt) * (vnew - rt), cc = (vcl - rt) * (vcl - rt);
    if (!(du >= cc) && !(dd > -vfclip && dd < vfclip)) dv = 0.f;
    vl = 0.5f * (cc > du ? cc : du);
  }
  // per column: write dOut and fold the block's column sums
  S* drow = dOut + (long)(ok ? n : 0) * ldd;
  auto emit = [&](int k, float v) {
    if (!ok) v = 0.f;
    if (ok) st_elem(drow, k, v);
    float w = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (lane == 0) red[warp][k & 127] = w;
  };
  int k0 = 0;  // columns are folded in chunks of 128 (ldd <= 128 keeps it to one)
  for (int base = 0; base < ldd; base += 128) {
    const int top = min(ldd, base + 128);
    for (int k = base; k < top; k++) {
      float v = 0.f;
      if (k < O - 1) {
        if (mode == 1) {
          // head of column k
          int off = 0, h = 0;
          while (h < W && k >= off + hs[h]) off += hs[h++];
          const int sz = hs[h];
          float se = 0.f;
          for (int j = 0; j < sz; j++) se += expf(lg(off + j));
          const float lse = logf(se);
          float pout = 0.f;
          for (int j = 0; j < sz; j++) pout += expf(lg(off + j) - lse) * lg(off + j);
          const float p = expf(lg(k) - lse);
          v = dPol * ((k - off == head_action(a[h], sz) ? 1.f : 0.f) - p) + ent * p * (pout - lg(k));
        } else if (k < W) {
          const float lsr = lg(W + k);
          const float ls = lsr < lslo ? lslo : (lsr > lshi ? lshi : lsr);
          const float is = expf(-ls);
          const float z = (a[k] - lg(k)) * is;
          v = dPol * z * is;
        } else {
          const int i = k - W;
          const float lsr = lg(k);
          const float ls = lsr < lslo ? lslo : (lsr > lshi ? lshi : lsr);
          const float z = (a[i] - lg(i)) * expf(-ls);
          v = (lslo < lsr && lsr < lshi) ? dPol * (z * z - 1.f) + ent : 0.f;
        }
      } else if (k == O - 1) {
        v = -vf * dv;
      }
      emit(k, v);
    }
    __syncthreads();
    for (int k = base + threadIdx.x; k < top; k += 128)
      colpart[(long)blockIdx.x * ldd + k] =
          ((red[0][k & 127] + red[1][k & 127]) + red[2][k & 127]) + red[3][k & 127];
    __syncthreads();
    k0 = top;
  }
  (void)k0;
  if (loss_part) {
    float lt[6] = {ok ? fmaxf(-ad * ratio, -ad * rc) : 0.f, ok ? vl : 0.f, ok ? entr : 0.f,
                   ok ? (ratio - 1.f) - lgr : 0.f, ok ? -lgr : 0.f,
                   ok ? ((ratio < lo || ratio > hi) ? 1.f : 0.f) : 0.f};
#pragma unroll
    for (int q = 0; q < 6; q++) {
      float w = lt[q];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
      if (lane == 0) lred[warp][q] = w;
    }
    __syncthreads();
    if (threadIdx.x < 6)
      loss_part[(long)blockIdx.x * 8 + threadIdx.x] =
          ((lred[0][threadIdx.x] + lred[1][threadIdx.x]) + lred[2][threadIdx.x]) + lred[3][threadIdx.x];
  }
}
// dst[k][0..W) = src[idx[k]][0..W)
__global__ void gather_rows_f32_kernel(const int* __restrict__ idx, int Nmb, const float* __restrict__ src, int W,
                                       float* dst) {
  const long n = (long)Nmb * W;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long k = i / W;
    dst[i] = src[(long)idx[k] * W + (i - k * W)];
  }
}
__global__ void f64_to_f32_rows_kernel(const double* __restrict__ s, long n, float* d) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) d[i] = (float)s[i];
}

// gb[c] = sum_n M[n*N + c] (sequential per column, deterministic)
// Column sums of a row-major rows x N matrix in a fixed order, two levels: block (x, y) takes 32
// columns of the row chunk [y*chunk, (y+1)*chunk); its 8 row lanes each sum every 8th row of the chunk
// in order and are combined in lane order, giving part[y*N + c]; colsum_parts_kernel then sums the
// chunks in order. (One thread per column walking all rows left the GPU idle on long minibatches.)
__global__ void __launch_bounds__(256) colsum_chunk_f32_kernel(const float* __restrict__ Mx, long rows, int N,
                                                               long chunk, float* part) {
  __shared__ float sh[8][33];
  const int cl = threadIdx.x & 31, rl = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cl;
  const long r0 = (long)blockIdx.y * chunk, r1 = min(rows, r0 + chunk);
  float s = 0.f;
  if (c < N)
    for (long r = r0 + rl; r < r1; r += 8) s += Mx[r * N + c];
  sh[rl][cl] = s;
  __syncthreads();
  if (rl == 0 && c < N) {
    float t = sh[0][cl];
#pragma unroll
    for (int q = 1; q < 8; q++) t += sh[q][cl];
    part[(long)blockIdx.y * N + c] = t;
  }
}
__global__ void colsum_parts_kernel(const float* __restrict__ part, int chunks, int N, float* out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= N) return;
  float s = 0.f;
  for (int y = 0; y < chunks; y++) s += part[(long)y * N + c];
  out[c] = s;
}

// ---------------------------------------------------------------- host launchers
// One block per row (or tile) up to 148 x 16 blocks, at least one.
static inline unsigned rowwise_grid(long units) { return (unsigned)std::max(1L, std::min(units, 148L * 16)); }
static inline unsigned grid_for(long n, int block = 256, long cap = 148 * 16) {
  long g = (n + block - 1) / block;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (unsigned)g;
}

int launch_obs_to_bf16_f64(const double* src, long NT, int D, int Dp, __nv_bfloat16* dst, cudaStream_t st) {
  obs_to_bf16_kernel<double><<<rowwise_grid(ceil_div(NT, 8)), 256, 0, st>>>(src, NT, D, Dp, dst);
  count_launch();
  PL_LAUNCH("obs_to_bf16_kernel");
  return PL_OK;
}
int launch_obs_to_bf16_f32(const float* src, long NT, int D, int Dp, __nv_bfloat16* dst, cudaStream_t st) {
  obs_to_bf16_kernel<float><<<rowwise_grid(ceil_div(NT, 8)), 256, 0, st>>>(src, NT, D, Dp, dst);
  count_launch();
  PL_LAUNCH("obs_to_bf16_kernel");
  return PL_OK;
}
int launch_obs_to_f32_f64(const double* src, long n, float* dst, cudaStream_t st) {
  obs_to_f32_kernel<double><<<grid_for(n), 256, 0, st>>>(src, n, dst);
  count_launch();
  PL_LAUNCH("obs_to_f32_kernel");
  return PL_OK;
}
int launch_columns(const double* act, const double* ret, const double* olp, const double* ov, long NT, int* act_i,
                   float* ret_f, float* olp_f, float* ov_f, cudaStream_t st) {
  columns_kernel<<<grid_for(NT), 256, 0, st>>>(act, ret, olp, ov, NT, act_i, ret_f, olp_f, ov_f);
  count_launch();
  PL_LAUNCH("columns_kernel");
  return PL_OK;
}
int launch_perm_positions(const int* perm, long NT, long n, int* pos, int* out, cudaStream_t st) {
  PL_CUDA(cudaMemsetAsync(pos, 0, sizeof(int) * NT, st));
  perm_inverse_kernel<<<grid_for(NT), 256, 0, st>>>(perm, NT, pos);
  perm_compose_kernel<<<grid_for(n), 256, 0, st>>>(perm, pos, NT, n, out);
  count_launch(2);
  PL_LAUNCH("perm_compose_kernel");
  return PL_OK;
}
int launch_perm(const double* perm, long n, int* out, cudaStream_t st) {
  perm_kernel<<<grid_for(n), 256, 0, st>>>(perm, n, out);
  count_launch();
  PL_LAUNCH("perm_kernel");
  return PL_OK;
}
int launch_adv_ms_from_sums(const double* sums, double* ms, cudaStream_t st) {
  adv_ms_from_sums_kernel<<<1, 32, 0, st>>>(sums, ms);
  count_launch();
  PL_LAUNCH("adv_ms_from_sums_kernel");
  return PL_OK;
}
int launch_gather(bool bf16, const int* idx, int Nmb, const void* obs, int rowElems, void* X, const int* act_c,
                  const double* adv_c, const float* ret_c, const float* olp_c, const float* ov_c, int* mb_act,
                  float* mb_adv, float* mb_ret, float* mb_olp, float* mb_ov, double* part, double* ms,
                  cudaStream_t st, double* sums, const int* oidx) {
  const int nb = (int)(Nmb < kStreamBlocks * 8 ? (Nmb + 7) / 8 : kStreamBlocks);
  if (bf16)
    gather_kernel<true><<<nb, 256, 0, st>>>(idx, Nmb, obs, rowElems, X, act_c, adv_c, ret_c, olp_c, ov_c, mb_act,
                                            mb_adv, mb_ret, mb_olp, mb_ov, part, oidx);
  else
    gather_kernel<false><<<nb, 256, 0, st>>>(idx, Nmb, obs, rowElems, X, act_c, adv_c, ret_c, olp_c, ov_c, mb_act,
                                             mb_adv, mb_ret, mb_olp, mb_ov, part, oidx);
  if (sums)
    adv_sums_kernel<<<1, 32, 0, st>>>(part, nb, Nmb, sums);
  else
    adv_stats_kernel<<<1, 32, 0, st>>>(part, nb, Nmb, ms);
  count_launch(2);
  PL_LAUNCH("gather_kernel");
  return PL_OK;
}
// part holds `tiles` rows of ld floats followed by room for ceil(tiles / kColChunk) rows of ncols
// (the second level of the reduction).
long colsum_scratch_elems(int tiles, long ld) { return (long)tiles * ld + ceil_div(tiles, kColChunk) * ld; }
int launch_colsum_reduce(const float* part, int tiles, long ld, int ncols, float* out, cudaStream_t st) {
  const int runs = (int)ceil_div(tiles, kColChunk);
  if (runs <= 1) {
    colsum_final_kernel<<<(unsigned)ceil_div(ncols, 128), 128, 0, st>>>(part, tiles, ld, ncols, out);
    count_launch();
  } else {
    float* part2 = const_cast<float*>(part) + (long)tiles * ld;
    dim3 g1((unsigned)ceil_div(ncols, 128), (unsigned)runs);
    colsum_reduce_kernel<<<g1, 128, 0, st>>>(part, tiles, ld, ncols, part2);
    colsum_final_kernel<<<(unsigned)ceil_div(ncols, 128), 128, 0, st>>>(part2, runs, ncols, ncols, out);
    count_launch(2);
  }
  PL_LAUNCH("colsum_reduce_kernel");
  return PL_OK;
}
int launch_splitk_reduce(const float* part, int S, long n, float* out, cudaStream_t st) {
  if (S >= 32 && (n & 3) == 0 && ((uintptr_t)part & 15) == 0 && ((uintptr_t)out & 15) == 0) {
    splitk_reduce_warp_kernel<<<(unsigned)ceil_div(n / 4 * 32, 256), 256, 0, st>>>(part, S, n / 4, out);
    count_launch();
    PL_LAUNCH("splitk_reduce_warp_kernel");
    return PL_OK;
  }
  splitk_reduce_kernel<<<grid_for(n), 256, 0, st>>>(part, S, n, out);
  count_launch();
  PL_LAUNCH("splitk_reduce_kernel");
  return PL_OK;
}
int launch_gradnorm(const float* g, long P, double sc, double maxNorm, double* part, double* cc, cudaStream_t st) {
  gradnorm_part_kernel<<<kStreamBlocks, 256, 0, st>>>(g, P, sc, part);
  gradnorm_final_kernel<<<1, 32, 0, st>>>(part, kStreamBlocks, maxNorm, sc, cc);
  count_launch(2);
  PL_LAUNCH("gradnorm_kernel");
  return PL_OK;
}
int launch_nesterov(const float* g, const double* cc, double* mom, double* u, double mu, long n, double* part,
                    int* nparts, cudaStream_t st) {
  const int nb = (int)(n < (long)kStreamBlocks * 256 ? ceil_div(n, 256) : kStreamBlocks);
  nesterov_kernel<<<nb, 256, 0, st>>>(g, cc, mom, u, mu, n, part);
  *nparts = nb;
  count_launch();
  PL_LAUNCH("nesterov_kernel");
  return PL_OK;
}
int launch_ns_input(const double* u, const double* part, int nparts, int rows, int cols, double eps,
                    __nv_bfloat16* X, long ldx, cudaStream_t st) {
  if (rows > cols)
    ns_input_kernel<true><<<rowwise_grid(ceil_div(rows, 32) * ceil_div(cols, 32)), 256, 0, st>>>(u, part, nparts, rows,
                                                                                               cols, eps, X, ldx);
  else
    ns_input_kernel<false><<<rowwise_grid(rows), 256, 0, st>>>(u, part, nparts, rows, cols, eps, X, ldx);
  count_launch();
  PL_LAUNCH("ns_input_kernel");
  return PL_OK;
}
int launch_ns_finalize(const float* Xf, long ldx, int rows, int cols, double c1, double c2, double* W,
                       __nv_bfloat16* Wb, long ldw, cudaStream_t st) {
  if (rows > cols)
    ns_finalize_kernel<true><<<rowwise_grid(ceil_div(rows, 32) * ceil_div(cols, 32)), 256, 0, st>>>(Xf, ldx, rows,
                                                                                                   cols, c1, c2, W, Wb,
                                                                                                   ldw);
  else
    ns_finalize_kernel<false><<<rowwise_grid(rows), 256, 0, st>>>(Xf, ldx, rows, cols, c1, c2, W, Wb, ldw);
  count_launch();
  PL_LAUNCH("ns_finalize_kernel");
  return PL_OK;
}
int muon_group_blocks(int rows, int cols, int nb_total) {
  const long units = rows > cols ? (long)ceil_div(rows, 32) * ceil_div(cols, 32) : (long)rows;
  const long per = std::max(1L, (long)kMuonBlocksMax / std::max(1, nb_total));
  return (int)std::max(1L, std::min(units, per));
}
int launch_muon_x0(const MuonGroupArgs& a, int blocks, const double* cc, double mu, double* part, cudaStream_t st) {
  PL_REQUIRE(a.nb >= 1 && a.nb <= kMuonGroupMax && blocks >= 1, PL_ERR_INVALID, "launch_muon_x0: group of %d", a.nb);
  const dim3 grid((unsigned)blocks, (unsigned)a.nb);
  if (a.rows > a.cols)
    muon_x0_kernel<true><<<grid, 256, 0, st>>>(a, cc, mu, part);
  else
    muon_x0_kernel<false><<<grid, 256, 0, st>>>(a, cc, mu, part);
  count_launch();
  PL_LAUNCH("muon_x0_kernel");
  return PL_OK;
}
int launch_muon_scale(const double* part, int blocks, int nb, double eps, float* scale, cudaStream_t st) {
  muon_scale_kernel<<<(unsigned)nb, 32, 0, st>>>(part, blocks, nb, eps, scale);
  count_launch();
  PL_LAUNCH("muon_scale_kernel");
  return PL_OK;
}
int launch_muon_finalize(const MuonGroupArgs& a, int blocks, double lr, double wd, double mu, double s,
                         const double* cc, cudaStream_t st) {
  PL_REQUIRE(a.nb >= 1 && a.nb <= kMuonGroupMax && blocks >= 1, PL_ERR_INVALID, "launch_muon_finalize: group of %d",
             a.nb);
  const dim3 grid((unsigned)blocks, (unsigned)a.nb);
  if (a.rows > a.cols)
    muon_finalize_kernel<true><<<grid, 256, 0, st>>>(a, 1.0 - lr * wd, lr * s, cc, lr, wd, mu);
  else
    muon_finalize_kernel<false><<<grid, 256, 0, st>>>(a, 1.0 - lr * wd, lr * s, cc, lr, wd, mu);
  count_launch();
  PL_LAUNCH("muon_finalize_kernel");
  return PL_OK;
}
int launch_w_to_bf16(const double* W, int rows, int cols, __nv_bfloat16* Wb, long ldw, cudaStream_t st) {
  w_to_bf16_kernel<<<rowwise_grid(rows), 256, 0, st>>>(W, rows, cols, Wb, ldw);
  count_launch();
  PL_LAUNCH("w_to_bf16_kernel");
  return PL_OK;
}
int launch_f64_to_f32(const double* s, long n, float* d, cudaStream_t st) {
  f64_to_f32_kernel<<<grid_for(n), 256, 0, st>>>(s, n, d);
  count_launch();
  PL_LAUNCH("f64_to_f32_kernel");
  return PL_OK;
}
int launch_f32_to_f64(const float* s, long n, double* d, cudaStream_t st) {
  f32_to_f64_kernel<<<grid_for(n), 256, 0, st>>>(s, n, d);
  count_launch();
  PL_LAUNCH("f32_to_f64_kernel");
  return PL_OK;
}
int launch_sgemm(int M, int N, int K, const float* A, long ars, long acs, const float* B, long brs, long bcs, float* C,
                 long ldc, float alpha, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div(N, 64), (unsigned)ceil_div(M, 64));
  sgemm_kernel<SGEMM_PLAIN><<<grid, 256, 0, st>>>(M, N, K, A, ars, acs, B, brs, bcs, C, ldc, alpha, K, 0, -1, nullptr,
                                                  nullptr, 0);
  count_launch();
  PL_LAUNCH("sgemm_kernel");
  return PL_OK;
}
int launch_sgemm_bias_act(int M, int N, int K, const float* A, long lda, const float* W, const float* b, float* Z,
                          float* H, int act, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div(N, 64), (unsigned)ceil_div(M, 64));
  sgemm_kernel<SGEMM_BIAS_ACT><<<grid, 256, 0, st>>>(M, N, K, A, lda, 1, W, K, 1, Z, N, 1.f, K, 0, -1, b, H, act);
  count_launch();
  PL_LAUNCH("sgemm_kernel");
  return PL_OK;
}
int launch_sgemm_act_grad(int M, int N, int K, const float* A, long lda, const float* W, const float* Z, float* dH,
                          int act, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div(N, 64), (unsigned)ceil_div(M, 64));
  sgemm_kernel<SGEMM_ACT_GRAD><<<grid, 256, 0, st>>>(M, N, K, A, lda, 1, W, 1, N, dH, N, 1.f, K, 0, -1, nullptr,
                                                     const_cast<float*>(Z), act);
  count_launch();
  PL_LAUNCH("sgemm_kernel");
  return PL_OK;
}
bool skinny_rows_ok(int K, int O) { return O >= 1 && O <= kSkinnyO && K % 4 == 0 && K <= kSkinnyK; }
int launch_skinny_rows(const float* H, int rows, int K, const float* W, const float* b, int O, float* Out,
                       cudaStream_t st) {
  PL_REQUIRE(skinny_rows_ok(K, O), PL_ERR_INVALID, "skinny row product: K %d, O %d out of range", K, O);
  PL_REQUIRE(((uintptr_t)H & 15) == 0 && ((uintptr_t)W & 15) == 0, PL_ERR_INVALID, "skinny row product: unaligned");
  const unsigned nb = (unsigned)std::min<long>(ceil_div(rows, 8), 148L * 8);
  if (nb == 0) return PL_OK;
  skinny_rows_kernel<<<nb, 256, 0, st>>>(H, rows, K, W, b, O, Out);
  count_launch();
  PL_LAUNCH("skinny_rows_kernel");
  return PL_OK;
}
long splitk_wb_elems(int K, int out, int in) {
  if (out + in <= kWgMaxCols) return ceil_div(K, kWgRows) * out * (long)(in + 1);  // wgrad_small_kernel
  return std::min<long>(ceil_div(K, 64), ceil_div(8 * 148, ceil_div(in + 1, 64) * ceil_div(out, 64))) * out *
         (long)(in + 1);
}
int launch_wgrad_bias_f32(int out, int in, int K, const float* dZ, long ldz, const float* Hin, long ldh, float* dW,
                          float* db, float* ws, long ws_elems, cudaStream_t st) {
  const int N = in + 1;
  const long slices = ceil_div(K, kWgRows);
  if (out + in <= kWgMaxCols && slices * out * (long)N <= ws_elems && slices <= 65535) {
    // small layer: one 64-row slice per block staged through shared memory (all of a slice's outputs
    // from one copy of its rows), instead of 64 x 64 tiles that such a layer mostly leaves empty
    wgrad_small_kernel<<<(unsigned)slices, 256, 0, st>>>(out, in, K, dZ, ldz, Hin, ldh, ws);
    splitk_reduce_wb_kernel<<<(unsigned)ceil_div((long)out * N * 32, 256), 256, 0, st>>>(ws, (int)slices, out, in, dW,
                                                                                       db);
    count_launch(2);
    PL_LAUNCH("wgrad_small_kernel");
    return PL_OK;
  }
  const long tiles = ceil_div(N, 64) * ceil_div(out, 64), mn = (long)out * N;
  long S = std::min<long>(ceil_div(K, 64), ceil_div(8 * 148, tiles));
  S = std::min<long>(S, ws_elems / mn);
  PL_REQUIRE(S >= 1, PL_ERR_INVALID, "weight-gradient workspace too small");
  const int kc = (int)round_up(ceil_div(K, S), 16);
  S = ceil_div(K, kc);
  dim3 grid((unsigned)ceil_div(N, 64), (unsigned)ceil_div(out, 64), (unsigned)S);
  sgemm_kernel<SGEMM_PLAIN><<<grid, 256, 0, st>>>(out, N, K, dZ, 1, ldz, Hin, 1, ldh, ws, N, 1.f, kc, mn, in, nullptr,
                                                  nullptr, 0);
  splitk_reduce_wb_kernel<<<(unsigned)ceil_div(mn * 32, 256), 256, 0, st>>>(ws, (int)S, out, in, dW, db);
  count_launch(2);
  PL_LAUNCH("splitk_reduce_wb_kernel");
  return PL_OK;
}
// A long-K product with few output tiles (the weight gradients, K = the minibatch rows) would leave
// all but a few SMs idle walking K: split K over blockIdx.z into slices of the workspace (S * M * N
// floats, C dense: ldc = N), then sum the slices in a fixed order (deterministic). Each slice is a
// chain of dependent global loads, 16 rows per step, so slices are kept short (64 rows) as long as
// the grid stays within eight CTAs per SM.
int launch_sgemm_splitk(int M, int N, int K, const float* A, long ars, long acs, const float* B, long brs, long bcs,
                        float* C, long ldc, float* ws, long ws_elems, cudaStream_t st) {
  const long tiles = ceil_div(N, 64) * ceil_div(M, 64), mn = (long)M * N;
  long S = std::min<long>(ceil_div(K, 64), ceil_div(8 * 148, tiles));
  if (ws && mn > 0) S = std::min<long>(S, ws_elems / mn);
  if (S < 2 || !ws || ldc != N) return launch_sgemm(M, N, K, A, ars, acs, B, brs, bcs, C, ldc, 1.f, st);
  const int kc = (int)round_up(ceil_div(K, S), 16);
  S = ceil_div(K, kc);
  dim3 grid((unsigned)ceil_div(N, 64), (unsigned)ceil_div(M, 64), (unsigned)S);
  sgemm_kernel<SGEMM_PLAIN><<<grid, 256, 0, st>>>(M, N, K, A, ars, acs, B, brs, bcs, ws, N, 1.f, kc, mn, -1, nullptr,
                                                  nullptr, 0);
  count_launch();
  PL_LAUNCH("sgemm_kernel");
  return launch_splitk_reduce(ws, (int)S, mn, C, st);
}
int launch_bias_act_f32(float* Z, float* H, const float* b, long M, int N, int act, cudaStream_t st) {
  bias_act_f32_kernel<<<grid_for(M * N), 256, 0, st>>>(Z, H, b, M, N, act);
  count_launch();
  PL_LAUNCH("bias_act_f32_kernel");
  return PL_OK;
}
int launch_act_grad_f32(float* dH, const float* Z, long n, int act, cudaStream_t st) {
  act_grad_f32_kernel<<<grid_for(n), 256, 0, st>>>(dH, Z, n, act);
  count_launch();
  PL_LAUNCH("act_grad_f32_kernel");
  return PL_OK;
}
int launch_ppo_rows_wide(bool bf16_out, const float* Out, int ldo, const float* bias, int M, int O, int ldd, int mode,
                        int W, const int* hs, const float* actw, const float* adv, const double* ms, const float* ret,
                        const float* olp, const float* ov, float vf, float ent, float clip, float vfclip, float lslo,
                        float lshi, void* dOut, float* colpart, float* loss_part, cudaStream_t st) {
  const unsigned nb = (unsigned)ceil_div(M, 128);
  if (bf16_out)
    ppo_rows_wide_kernel<__nv_bfloat16><<<nb, 128, 0, st>>>(Out, ldo, bias, M, O, ldd, mode, W, hs, actw, adv, ms, ret,
                                                            olp, ov, vf, ent, clip, vfclip, lslo, lshi,
                                                            (__nv_bfloat16*)dOut, colpart, loss_part);
  else
    ppo_rows_wide_kernel<float><<<nb, 128, 0, st>>>(Out, ldo, bias, M, O, ldd, mode, W, hs, actw, adv, ms, ret, olp, ov,
                                                    vf, ent, clip, vfclip, lslo, lshi, (float*)dOut, colpart,
                                                    loss_part);
  count_launch();
  PL_LAUNCH("ppo_rows_wide_kernel");
  return PL_OK;
}
int launch_gather_rows_f32(const int* idx, int Nmb, const float* src, int W, float* dst, cudaStream_t st) {
  gather_rows_f32_kernel<<<grid_for((long)Nmb * W), 256, 0, st>>>(idx, Nmb, src, W, dst);
  count_launch();
  PL_LAUNCH("gather_rows_f32_kernel");
  return PL_OK;
}
int launch_f64_to_f32_rows(const double* s, long n, float* d, cudaStream_t st) {
  f64_to_f32_rows_kernel<<<grid_for(n), 256, 0, st>>>(s, n, d);
  count_launch();
  PL_LAUNCH("f64_to_f32_rows_kernel");
  return PL_OK;
}
int launch_ppo_rows_f32(const float* Out, int M, int A, const int* act, const float* adv, const double* ms,
                        const float* ret, const float* olp, const float* ov, float vf, float ent, float clip,
                        float vfclip, float* dOut, float* newlp, float* newval, cudaStream_t st) {
  ppo_rows_f32_kernel<<<(unsigned)ceil_div(M, 128), 128, 0, st>>>(Out, M, A, act, adv, ms, ret, olp, ov, vf, ent, clip,
                                                                  vfclip, dOut, newlp, newval);
  count_launch();
  PL_LAUNCH("ppo_rows_f32_kernel");
  return PL_OK;
}
int launch_colsum_f32(const float* Mx, long rows, int N, float* out, float* ws, long ws_elems, cudaStream_t st) {
  PL_REQUIRE(N > 0 && ws && ws_elems >= N, PL_ERR_INVALID, "colsum: workspace of %ld floats for %d columns", ws_elems,
             N);
  long chunks = std::min<long>(std::max<long>(1, ceil_div(rows, 128)), ws_elems / N);
  chunks = std::min<long>(chunks, 65535);
  const long chunk = std::max<long>(1, ceil_div(rows, chunks));
  chunks = std::max<long>(1, ceil_div(rows, chunk));
  colsum_chunk_f32_kernel<<<dim3((unsigned)ceil_div(N, 32), (unsigned)chunks), 256, 0, st>>>(Mx, rows, N, chunk, ws);
  colsum_parts_kernel<<<(unsigned)ceil_div(N, 128), 128, 0, st>>>(ws, (int)chunks, N, out);
  count_launch(2);
  PL_LAUNCH("colsum_chunk_f32_kernel");
  return PL_OK;
}

}  // namespace pl
