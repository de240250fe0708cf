// MinGRU PPO+Muon update path: the recurrent policy of Puffer/Net/MinGRU.lean:9-17 trained by the
// minibatch chain of Puffer/RL/MinGRUTrain.lean:800-850 (V-trace with live importance ratios and
// values, prioritised segment sampling, BPTT PPO gradient, value/ratio iterate, clip, Muon).
//
// Layout of one minibatch (Bmb sampled segments x T steps): rows are time-major, r = t*Bmb + b, so
// every GEMM of the network covers all T steps at once ([R x .] with R = T*Bmb), and the only
// sequential work, the scan over t, is elementwise over (b, j):
//
//   forward   h0 = enc(X W_enc^T + b_enc)              GEMM (bias/activation in the epilogue)
//             Y_l = h_l W_l^T                          GEMM, [R x K*H] = [hid | gate | (proj)]
//             o_t = (1 - z_t) o_{t-1} + z_t g(hid_t)    scan over t, z = sigmoid(gate), state reset
//             h_{l+1} = hg o + (1 - hg) h_l  (K = 3)    after a terminal; hg = sigmoid(proj)
//             Out = h_L [W_dec; w_val]^T + b            GEMM, fp32 logits and value
//   backward  dOut from the PPO objective per row; dh_L = dOut W_out; per layer the reverse scan
//             gives dY (and the highway part of dh_l), dW_l = dY^T h_l, dh_l += dY W_l; the encoder
//             takes dE = dh_0 * enc'(Z); dW_enc = dE^T X; bias gradients are column sums.
//
// Two tiers: tight (fp32 SIMT GEMMs, fp32 activations; the parity tier) and fast (bf16 tcgen05
// GEMMs with fp32 accumulation, bf16 activations; the recurrent state itself is carried in fp32
// registers through every scan).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <vector>

#include "../../include/pufferlean_b200.h"
#include "pl_comm.h"
#include "pl_common.cuh"
#include "pl_gemm.cuh"
#include "pl_mlp.cuh"
#include "pl_muon.cuh"
#include "pl_runtime.h"

namespace pl {
namespace {

typedef __nv_bfloat16 bf16;

template <typename S>
__device__ __forceinline__ float ldv(const S* p, long i);
template <>
__device__ __forceinline__ float ldv<float>(const float* p, long i) {
  return p[i];
}
template <>
__device__ __forceinline__ float ldv<bf16>(const bf16* p, long i) {
  return __bfloat162float(p[i]);
}
template <typename S>
__device__ __forceinline__ void stv(S* p, long i, float v);
template <>
__device__ __forceinline__ void stv<float>(float* p, long i, float v) {
  p[i] = v;
}
template <>
__device__ __forceinline__ void stv<bf16>(bf16* p, long i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

inline unsigned blocks_for(long n, int block = 256, long cap = 148 * 32) {
  long g = (n + block - 1) / block;
  return (unsigned)std::max<long>(1, std::min(g, cap));
}
inline long rup(long x, long m) { return (x + m - 1) / m * m; }

// ---------------------------------------------------------------- minibatch gather
// X[r][c] = traj[(seg[b]*T + t)*D + c] for c < D, 0 in the padding (r = t*Bmb + b)
template <typename S>
__global__ void mg_gather_obs_kernel(const float* __restrict__ traj, const double* __restrict__ seg, int Bmb, int T,
                                     int D, int Dp, S* X) {
  const long n = (long)T * Bmb * Dp;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / Dp;
    const int c = (int)(i - r * Dp);
    const int t = (int)(r / Bmb), b = (int)(r - (long)t * Bmb);
    float v = 0.f;
    if (c < D) v = traj[((long)seg[b] * T + t) * D + c];
    stv(X, i, v);
  }
}
// host-mode obs: src f64 [R x D] (already time-major) -> X [R x Dp]
template <typename S>
__global__ void mg_obs_rows_kernel(const double* __restrict__ src, long R, int D, int Dp, S* X) {
  const long n = R * Dp;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / Dp;
    const int c = (int)(i - r * Dp);
    stv(X, i, c < D ? (float)src[r * D + c] : 0.f);
  }
}

// Advantage mean and population std over the Bmb*T sampled entries (index q = b*T + t), in two
// passes (sum, then squared deviations) over a fixed grid of kAdvBlocks blocks: each block writes
// its partial, the last block to finish folds the partials in block order (the counter makes the
// finish order irrelevant) and resets the counter. ms = [mean, std + 1e-8].
constexpr int kAdvBlocks = 64;
// With raw != 0 (data parallel), the last block stores the plain total in ms[2 + sq] for an
// all-reduce over ranks, and mg_adv_final_kernel divides by the all-rank count.
__global__ void __launch_bounds__(256) mg_adv_ms_kernel(const double* __restrict__ adv,
                                                        const double* __restrict__ seg, int Bmb, int T, int sq,
                                                        double* ms, double* part, unsigned* counter, int raw) {
  __shared__ double sh[256];
  __shared__ bool last;
  const long n = (long)Bmb * T;
  const int tid = threadIdx.x;
  const double mean = sq ? ms[0] : 0.0;
  double s = 0.0;
  for (long q = (long)blockIdx.x * 256 + tid; q < n; q += (long)gridDim.x * 256) {
    const int b = (int)(q / T), t = (int)(q - (long)b * T);
    const double a = adv[(long)seg[b] * T + t];
    s += sq ? (a - mean) * (a - mean) : a;
  }
  sh[tid] = s;
  __syncthreads();
  for (int k = 128; k > 0; k >>= 1) {
    if (tid < k) sh[tid] += sh[tid + k];
    __syncthreads();
  }
  if (tid == 0) {
    part[blockIdx.x] = sh[0];
    __threadfence();
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && tid == 0) {
    __threadfence();
    double tot = 0.0;
    for (int i = 0; i < (int)gridDim.x; i++) tot += ((volatile double*)part)[i];
    const double d = (double)(n > 0 ? n : 1);
    if (raw)
      ms[2 + sq] = tot;
    else if (sq)
      ms[1] = sqrt(tot / d) + 1e-8;
    else
      ms[0] = tot / d;
    *counter = 0;
  }
}
__global__ void mg_adv_final_kernel(double* ms, double n, int sq) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    if (sq)
      ms[1] = sqrt(ms[3] / n) + 1e-8;
    else
      ms[0] = ms[2] / n;
  }
}
// Per-row minibatch scalars from the resident columns (the layout of the host gather,
// ffi/pufferffi.c:1137-1176): os = t*Bmb + b, si = seg[b]*T + t.
__global__ void mg_gather_scal_kernel(const double* __restrict__ act, const double* __restrict__ logp,
                                      const double* __restrict__ term, const double* __restrict__ adv,
                                      const double* __restrict__ value, const double* __restrict__ seg,
                                      const double* __restrict__ mbp, const double* __restrict__ ms, int Bmb, int T,
                                      int W, int* act_i, float* adv_f, float* ret_f, float* olp_f, float* ov_f,
                                      float* term_f) {
  const long n = (long)T * Bmb;
  for (long os = (long)blockIdx.x * blockDim.x + threadIdx.x; os < n; os += (long)gridDim.x * blockDim.x) {
    const int t = (int)(os / Bmb), b = (int)(os - (long)t * Bmb);
    const long si = (long)seg[b] * T + t;
    const double a = adv[si], v = value[si];
    for (int h = 0; h < W; h++) act_i[os * W + h] = (int)(unsigned long long)act[si * W + h];
    adv_f[os] = (float)(mbp[b] * (a - ms[0]) / ms[1]);
    ret_f[os] = (float)(a + v);
    olp_f[os] = (float)logp[si];
    ov_f[os] = (float)v;
    term_f[os] = term[si] > 0.5 ? 1.f : 0.f;
  }
}
// Host-mode scalars: scal = [act | adv | ret | old | term | ov], R time-major entries each, the act
// block W per row ([r*W + h]) with multi-discrete heads (ffi/puffercuda.cu:5216-5221).
__global__ void mg_scal_rows_kernel(const double* __restrict__ scal, long R, int W, int* act_i, float* adv_f,
                                    float* ret_f, float* olp_f, float* ov_f, float* term_f) {
  const double* s1 = scal + (long)W * R;
  for (long r = (long)blockIdx.x * blockDim.x + threadIdx.x; r < R; r += (long)gridDim.x * blockDim.x) {
    for (int h = 0; h < W; h++) act_i[r * W + h] = (int)(unsigned long long)scal[r * W + h];
    adv_f[r] = (float)s1[r];
    ret_f[r] = (float)s1[R + r];
    olp_f[r] = (float)s1[2 * R + r];
    term_f[r] = s1[3 * R + r] != 0.0 ? 1.f : 0.f;
    ov_f[r] = (float)s1[4 * R + r];
  }
}

// ---------------------------------------------------------------- scans
// Two adjacent columns per thread (VEC = 2) as one 4-byte (bf16) or 8-byte (fp32) access.
template <int VEC>
__device__ __forceinline__ void ldp(const float* p, float (&v)[VEC]) {
  if constexpr (VEC == 2) {
    const float2 q = *reinterpret_cast<const float2*>(p);
    v[0] = q.x;
    v[1] = q.y;
  } else {
    v[0] = p[0];
  }
}
template <int VEC>
__device__ __forceinline__ void ldp(const bf16* p, float (&v)[VEC]) {
  if constexpr (VEC == 2) {
    const float2 q = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    v[0] = q.x;
    v[1] = q.y;
  } else {
    v[0] = __bfloat162float(p[0]);
  }
}
template <int VEC>
__device__ __forceinline__ void stp(float* p, const float (&v)[VEC]) {
  if constexpr (VEC == 2)
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  else
    p[0] = v[0];
}
template <int VEC>
__device__ __forceinline__ void stp(bf16* p, const float (&v)[VEC]) {
  if constexpr (VEC == 2)
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
  else
    p[0] = __float2bfloat16_rn(v[0]);
}
// Logistic function: the fast tier uses the hardware exponential and division approximations,
// the tight tier the accurate library calls.
template <bool FAST>
__device__ __forceinline__ float sigm(float x) {
  if constexpr (FAST)
    return __fdividef(1.f, 1.f + __expf(-x));
  else
    return 1.f / (1.f + expf(-x));
}

// Forward scan of one layer: thread (b, columns j..j+VEC-1) walks t = 0..T-1 with the states in
// registers. Y [R x K*H], hin/hout/Os [R x H], term [R] (1 = terminal at that step). The inputs of a
// step do not depend on the state, so they are loaded kScanU steps at a time ahead of the
// recurrence: the loads of a group are all in flight together and only the arithmetic is serial.
constexpr int kScanU = 4;
// The reverse scan holds more live values per step; two steps ahead keep it at 4 blocks of 256 per
// SM (<= 64 registers), so its 512-block grids (512 segments x 512 columns) finish in one wave.
constexpr int kScanUB = 2;
template <typename S, int K, int VEC, bool FAST>
__global__ void __launch_bounds__(256) mg_scan_fwd_kernel(const S* __restrict__ Y, const S* __restrict__ hin,
                                                          S* __restrict__ hout, S* __restrict__ Os,
                                                          const float* __restrict__ term, int B, int H, int T) {
  const int HV = H / VEC;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)B * HV) return;
  const int b = (int)(idx / HV), j = (int)(idx - (long)b * HV) * VEC;
  const long KH = (long)K * H, sY = (long)B * KH, sH = (long)B * H;
  const S* py = Y + (long)b * KH + j;
  const S* ph = hin + (long)b * H + j;
  S* po = Os + (long)b * H + j;
  S* pout = hout + (long)b * H + j;
  const float* pt = term + b;
  float state[VEC];
#pragma unroll
  for (int v = 0; v < VEC; v++) state[v] = 0.f;
  for (int t0 = 0; t0 < T; t0 += kScanU) {
    float hid[kScanU][VEC], gate[kScanU][VEC], proj[kScanU][VEC], hi[kScanU][VEC], tm[kScanU];
#pragma unroll
    for (int u = 0; u < kScanU; u++) {
      if (t0 + u < T) {
        ldp<VEC>(py + u * sY, hid[u]);
        ldp<VEC>(py + u * sY + H, gate[u]);
        if (K == 3) {
          ldp<VEC>(py + u * sY + 2 * H, proj[u]);
          ldp<VEC>(ph + u * sH, hi[u]);
        }
        tm[u] = pt[(long)u * B];
      }
    }
#pragma unroll
    for (int u = 0; u < kScanU; u++) {
      if (t0 + u < T) {
        float o[VEC], hn[VEC];
#pragma unroll
        for (int v = 0; v < VEC; v++) {
          const float z = sigm<FAST>(gate[u][v]);
          const float g = hid[u][v] >= 0.f ? hid[u][v] + 0.5f : sigm<FAST>(hid[u][v]);
          o[v] = (1.f - z) * state[v] + z * g;
          if (K == 3) {
            const float hg = sigm<FAST>(proj[u][v]);
            hn[v] = hg * o[v] + (1.f - hg) * hi[u][v];
          } else {
            hn[v] = o[v];
          }
          state[v] = tm[u] != 0.f ? 0.f : o[v];
        }
        stp<VEC>(po + u * sH, o);
        stp<VEC>(pout + u * sH, hn);
      }
    }
    py += kScanU * sY;
    ph += kScanU * sH;
    po += kScanU * sH;
    pout += kScanU * sH;
    pt += (long)kScanU * B;
  }
}
// Reverse scan of one layer (the per-element backward of ffi/pufferffi.c:840-868): dY [R x K*H],
// dhn [R x H] = the highway part of the gradient reaching the layer input (K = 3). Loads run kScanU
// steps ahead of the reverse recurrence, as in the forward scan.
template <typename S, int K, int VEC, bool FAST>
__global__ void __launch_bounds__(256, 4) mg_scan_bwd_kernel(const S* __restrict__ Y, const S* __restrict__ Os,
                                                          const S* __restrict__ hin, const S* __restrict__ dh,
                                                          S* __restrict__ dY, S* __restrict__ dhn,
                                                          const float* __restrict__ term, int B, int H, int T) {
  const int HV = H / VEC;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)B * HV) return;
  const int b = (int)(idx / HV), j = (int)(idx - (long)b * HV) * VEC;
  const long KH = (long)K * H, sY = (long)B * KH, sH = (long)B * H;
  const long last = (long)(T - 1);
  const S* py = Y + last * sY + (long)b * KH + j;
  S* pdy = dY + last * sY + (long)b * KH + j;
  const long oH = last * sH + (long)b * H + j;
  const S* po = Os + oH;
  const S* ph = hin + oH;
  const S* pd = dh + oH;
  S* pdn = dhn ? dhn + oH : nullptr;
  const float* pt = term + last * B + b;
  float dOnext[VEC];
#pragma unroll
  for (int v = 0; v < VEC; v++) dOnext[v] = 0.f;
  for (int t1 = T - 1; t1 >= 0; t1 -= kScanUB) {
    float hid[kScanUB][VEC], gate[kScanUB][VEC], proj[kScanUB][VEC], hi[kScanUB][VEC], o[kScanUB][VEC],
        prev[kScanUB][VEC], dhv[kScanUB][VEC];
    bool flow[kScanUB];
#pragma unroll
    for (int u = 0; u < kScanUB; u++) {
      const int t = t1 - u;
      if (t >= 0) {
        flow[u] = t > 0 && pt[-(long)(u + 1) * B] == 0.f;  // no state (and no gradient) across a terminal
        ldp<VEC>(py - u * sY, hid[u]);
        ldp<VEC>(py - u * sY + H, gate[u]);
        if (K == 3) {
          ldp<VEC>(py - u * sY + 2 * H, proj[u]);
          ldp<VEC>(ph - u * sH, hi[u]);
        }
        ldp<VEC>(po - u * sH, o[u]);
        if (t > 0)
          ldp<VEC>(po - (u + 1) * sH, prev[u]);
        else
#pragma unroll
          for (int v = 0; v < VEC; v++) prev[u][v] = 0.f;
        ldp<VEC>(pd - u * sH, dhv[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kScanUB; u++) {
      const int t = t1 - u;
      if (t >= 0) {
        float dyh[VEC], dyg[VEC], dyp[VEC], dhw[VEC];
#pragma unroll
        for (int v = 0; v < VEC; v++) {
          const float pv = flow[u] ? prev[u][v] : 0.f;
          const float z = sigm<FAST>(gate[u][v]);
          const float sh = sigm<FAST>(hid[u][v]);
          const float g = hid[u][v] >= 0.f ? hid[u][v] + 0.5f : sh;
          const float dhj = dhv[u][v];
          float dout;
          if (K == 3) {
            const float hg = sigm<FAST>(proj[u][v]);
            const float dhg = dhj * (o[u][v] - hi[u][v]);
            dout = dhj * hg + dOnext[v];
            dhw[v] = dhj * (1.f - hg);
            dyp[v] = dhg * hg * (1.f - hg);
          } else {
            dout = dhj + dOnext[v];
          }
          const float dz = dout * (g - pv);
          const float dprev = dout * (1.f - z);
          const float dg = dout * z;
          const float sg = hid[u][v] >= 0.f ? 1.f : sh * (1.f - sh);
          dyh[v] = dg * sg;
          dyg[v] = dz * z * (1.f - z);
          dOnext[v] = flow[u] ? dprev : 0.f;
        }
        stp<VEC>(pdy - u * sY, dyh);
        stp<VEC>(pdy - u * sY + H, dyg);
        if (K == 3) {
          stp<VEC>(pdy - u * sY + 2 * H, dyp);
          stp<VEC>(pdn - u * sH, dhw);
        }
      }
    }
    py -= kScanUB * sY;
    pdy -= kScanUB * sY;
    po -= kScanUB * sH;
    ph -= kScanUB * sH;
    pd -= kScanUB * sH;
    if (pdn) pdn -= kScanUB * sH;
    pt -= (long)kScanUB * B;
  }
}

// ---------------------------------------------------------------- PPO head (per row)
// The recurrent path's head math (ffi/puffercuda.cu:4910-4930): log-softmax with the max
// subtracted, clipped surrogate, entropy bonus, clipped value loss. Out [R x ldo] fp32 without the
// bias; bout [A+1]. dOut [R x Op] (zero past A+1). lossrow (optional) [R x 8]: pg, vloss, entropy,
// old_kl, kl, clipped.
template <typename S>
__global__ void mg_ppo_rows_kernel(const float* __restrict__ Out, int ldo, const float* __restrict__ bout, long R,
                                   int A, int Op, const int* __restrict__ act, const float* __restrict__ adv,
                                   const float* __restrict__ ret, const float* __restrict__ olp,
                                   const float* __restrict__ ov, float vf, float ent, float clip, float vfclip, S* dOut,
                                   float* newlp, float* newval, float* lossrow) {
  for (long r = (long)blockIdx.x * blockDim.x + threadIdx.x; r < R; r += (long)gridDim.x * blockDim.x) {
    const float* o = Out + r * ldo;
    float mx = o[0] + bout[0];
    for (int k = 1; k < A; k++) mx = fmaxf(mx, o[k] + bout[k]);
    float se = 0.f;
    for (int k = 0; k < A; k++) se += expf(o[k] + bout[k] - mx);
    const float lse = mx + logf(se);
    float pout = 0.f;
    for (int k = 0; k < A; k++) {
      const float l = o[k] + bout[k];
      pout += expf(l - lse) * l;
    }
    const int a = act[r];
    const float logpA = o[a] + bout[a] - lse;
    const float ratio = expf(logpA - olp[r]);
    const float lo = 1.f - clip, hi = 1.f + clip;
    const float rc = ratio < lo ? lo : (ratio > hi ? hi : ratio);
    const float ad = adv[r];
    const float s1 = ad * ratio, s2 = ad * rc;
    const float dPol = s1 <= s2 ? ad * ratio : ad * ((lo < ratio && ratio < hi) ? 1.f : 0.f) * ratio;
    const float vnew = o[A] + bout[A], rt = ret[r], vold = ov[r];
    float dvl = vnew - rt;
    float vcl = vnew;
    if (vfclip > 0.f) {
      const float dd = vnew - vold;
      vcl = vold + (dd < -vfclip ? -vfclip : (dd > vfclip ? vfclip : dd));
      const float du = (vnew - rt) * (vnew - rt), cc = (vcl - rt) * (vcl - rt);
      if (!(du >= cc) && !(dd > -vfclip && dd < vfclip)) dvl = 0.f;
    }
    S* d = dOut + r * Op;
    for (int k = 0; k < A; k++) {
      const float l = o[k] + bout[k];
      const float p = expf(l - lse);
      stv(d, k, dPol * ((k == a ? 1.f : 0.f) - p) + ent * p * (pout - l));
    }
    stv(d, A, -vf * dvl);
    for (int k = A + 1; k < Op; k++) stv(d, k, 0.f);
    newlp[r] = logpA;
    newval[r] = vnew;
    if (lossrow) {
      const float lgr = logpA - olp[r];
      float* lr = lossrow + r * 8;
      lr[0] = fmaxf(-ad * ratio, -ad * rc);
      const float du = (vnew - rt) * (vnew - rt), cc = (vcl - rt) * (vcl - rt);
      lr[1] = 0.5f * ((vfclip > 0.f && cc > du) ? cc : du);
      lr[2] = lse - pout;  // entropy: -sum p (l - lse)
      lr[3] = -lgr;
      lr[4] = (ratio - 1.f) - lgr;
      lr[5] = (ratio < lo || ratio > hi) ? 1.f : 0.f;
    }
  }
}

// Multi-discrete heads (ffi/puffercuda.cu:4940-4980, k_mg_ppo_b_md): W heads of sizes hs over the A
// logits; per head the max-subtracted softmax; the joint log-prob accumulated in double as
// sum_h log(exp(x_a - m) / se), the form of the sampler that produced the old log-prob; one clipped
// ratio for the row. An action index outside its head is held inside it (valid columns never are).
template <typename S>
__global__ void mg_ppo_rows_md_kernel(const float* __restrict__ Out, int ldo, const float* __restrict__ bout, long R,
                                      int A, int Op, int W, const int* __restrict__ hs, const int* __restrict__ act,
                                      const float* __restrict__ adv, const float* __restrict__ ret,
                                      const float* __restrict__ olp, const float* __restrict__ ov, float vf, float ent,
                                      float clip, float vfclip, S* dOut, float* newlp, float* newval, float* lossrow) {
  for (long r = (long)blockIdx.x * blockDim.x + threadIdx.x; r < R; r += (long)gridDim.x * blockDim.x) {
    const float* o = Out + r * ldo;
    const int* ar = act + r * W;
    auto lg = [&](int k) { return o[k] + bout[k]; };
    double joint = 0.0;
    float entr = 0.f;
    int off = 0;
    for (int h = 0; h < W; h++) {
      const int sz = hs[h];
      int a = ar[h];
      a = a < 0 ? 0 : (a >= sz ? sz - 1 : a);
      float mx = lg(off);
      for (int k = 1; k < sz; k++) mx = fmaxf(mx, lg(off + k));
      float se = 0.f;
      for (int k = 0; k < sz; k++) se += expf(lg(off + k) - mx);
      joint += log(exp((double)lg(off + a) - (double)mx) / (double)se);
      if (lossrow) {
        const float lse = mx + logf(se);
        float pout = 0.f;
        for (int k = 0; k < sz; k++) pout += expf(lg(off + k) - lse) * lg(off + k);
        entr += lse - pout;
      }
      off += sz;
    }
    const float ratio = (float)exp(joint - (double)olp[r]);
    const float lo = 1.f - clip, hi = 1.f + clip;
    const float rc = ratio < lo ? lo : (ratio > hi ? hi : ratio);
    const float ad = adv[r];
    const float s1 = ad * ratio, s2 = ad * rc;
    const float dPol = s1 <= s2 ? ad * ratio : ad * ((lo < ratio && ratio < hi) ? 1.f : 0.f) * ratio;
    const float vnew = lg(A), rt = ret[r], vold = ov[r];
    float dvl = vnew - rt;
    float vcl = vnew;
    if (vfclip > 0.f) {
      const float dd = vnew - vold;
      vcl = vold + (dd < -vfclip ? -vfclip : (dd > vfclip ? vfclip : dd));
      const float du = (vnew - rt) * (vnew - rt), cc = (vcl - rt) * (vcl - rt);
      if (!(du >= cc) && !(dd > -vfclip && dd < vfclip)) dvl = 0.f;
    }
    S* d = dOut + r * Op;
    off = 0;
    for (int h = 0; h < W; h++) {
      const int sz = hs[h];
      int a = ar[h];
      a = a < 0 ? 0 : (a >= sz ? sz - 1 : a);
      float mx = lg(off);
      for (int k = 1; k < sz; k++) mx = fmaxf(mx, lg(off + k));
      float se = 0.f;
      for (int k = 0; k < sz; k++) se += expf(lg(off + k) - mx);
      const float lse = mx + logf(se);
      float pout = 0.f;
      for (int k = 0; k < sz; k++) pout += expf(lg(off + k) - lse) * lg(off + k);
      for (int k = 0; k < sz; k++) {
        const float l = lg(off + k), p = expf(l - lse);
        stv(d, off + k, dPol * ((k == a ? 1.f : 0.f) - p) + ent * p * (pout - l));
      }
      off += sz;
    }
    stv(d, A, -vf * dvl);
    for (int k = A + 1; k < Op; k++) stv(d, k, 0.f);
    newlp[r] = (float)joint;
    newval[r] = vnew;
    if (lossrow) {
      const float lgr = (float)joint - olp[r];
      float* lr = lossrow + r * 8;
      lr[0] = fmaxf(-ad * ratio, -ad * rc);
      const float du = (vnew - rt) * (vnew - rt), cc = (vcl - rt) * (vcl - rt);
      lr[1] = 0.5f * ((vfclip > 0.f && cc > du) ? cc : du);
      lr[2] = entr;
      lr[3] = -lgr;
      lr[4] = (ratio - 1.f) - lgr;
      lr[5] = (ratio < lo || ratio > hi) ? 1.f : 0.f;
    }
  }
}

// ---------------------------------------------------------------- reductions, elementwise
// part[chunk][c] = sum of rows [chunk*rows_per, ...) of column c.
// Column sums of one chunk of rows: a 32 x 8 block, thread (x, y) sums column 32 blockIdx.x + x over
// the chunk's rows y, y + 8, ..., and row 0 adds the 8 partials in order (deterministic). Eight threads
// per column keep narrow sums (the head's A + 1 columns) from running one thread per column.
template <typename S>
__global__ void __launch_bounds__(256) mg_colsum_part_kernel(const S* __restrict__ M, long R, long ld, int N,
                                                             int rows_per, float* part) {
  __shared__ float sh[8][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  const long r0 = (long)blockIdx.y * rows_per, r1 = min(R, r0 + (long)rows_per);
  float s = 0.f;
  if (c < N)
    for (long r = r0 + threadIdx.y; r < r1; r += 8) s += ldv(M, r * ld + c);
  sh[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < N) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++) t += sh[k][threadIdx.x];
    part[(long)blockIdx.y * N + c] = t;
  }
}
// out[c] = sum over chunks of part[chunk][c]: one warp per column, lane l takes chunks l, l + 32, ...,
// then a fixed shuffle tree (deterministic).
__global__ void __launch_bounds__(256) mg_colsum_final_kernel(const float* __restrict__ part, int chunks, int N,
                                                              float* out) {
  const int c = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (c >= N) return;  // warp-uniform
  float s = 0.f;
  for (int k = lane; k < chunks; k += 32) s += part[(long)k * N + c];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) out[c] = s;
}
// dE = dh * enc'(Z) in place
template <typename S>
__global__ void mg_act_grad_kernel(S* dh, const S* __restrict__ Z, long n, int act) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    stv(dh, i, ldv(dh, i) * act_grad(ldv(Z, i), act));
}
__global__ void mg_axpy_kernel(float* y, const float* __restrict__ x, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) y[i] += x[i];
}
// The head's [A+1 x H] weight gradient and [A+1] bias gradient into the flat layout
// (wDec rows, bDec, wVal row, bVal).
__global__ void mg_head_scatter_kernel(const float* __restrict__ gout, const float* __restrict__ gb, int A, int H,
                                       float* gWdec, float* gBdec, float* gWval, float* gBval) {
  const long n = (long)(A + 1) * H;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int k = (int)(i / H);
    const int j = (int)(i - (long)k * H);
    if (k < A)
      gWdec[i] = gout[i];
    else
      gWval[j] = gout[i];
  }
  if (blockIdx.x == 0)
    for (int k = threadIdx.x; k <= A; k += blockDim.x) {
      if (k < A)
        gBdec[k] = gb[k];
      else
        gBval[0] = gb[k];
    }
}

// ---------------------------------------------------------------- replay iterate
__global__ void mg_lastw_kernel(int* lastw, const double* __restrict__ seg, int Bmb) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < Bmb) atomicMax(&lastw[(long)seg[b]], b);
}
// value/ratio of every sampled segment from the BPTT's new value / log-prob; when a segment was
// drawn more than once, the largest b writes (the host loop's last write).
__global__ void mg_iterate_kernel(double* value, double* ratio, const double* __restrict__ logp,
                                  const float* __restrict__ newlp, const float* __restrict__ newval,
                                  const double* __restrict__ seg, const int* __restrict__ lastw, int Bmb, int T) {
  const long n = (long)T * Bmb;
  for (long os = (long)blockIdx.x * blockDim.x + threadIdx.x; os < n; os += (long)gridDim.x * blockDim.x) {
    const int t = (int)(os / Bmb), b = (int)(os - (long)t * Bmb);
    const long e = (long)seg[b];
    if (lastw[e] != b) continue;
    const long si = e * T + t;
    ratio[si] = exp((double)newlp[os] - logp[si]);
    value[si] = (double)newval[os];
  }
}

// ---------------------------------------------------------------- prioritised sampling
// One block: priorities, their sum (fixed tree), probabilities, the prefix sum (per-thread runs
// plus a sequential scan of the run totals), then the draws (splitmix64 state rng + (i+1)*GOLD,
// lower-bound search, importance weight). Deterministic; the sums are ordered differently from the
// host sampler's sequential loop, so a draw can differ from it only when u falls within rounding
// of a cumulative boundary.
// rng_dev (optional): the generator state lives in device memory; it is read here and advanced by
// Bmb * GOLD, so a captured minibatch graph draws a fresh sample on every replay.
__global__ void __launch_bounds__(1024) mg_prio_kernel(const double* __restrict__ l1, long N, long Bmb, double alpha,
                                                       double beta, unsigned long long rng,
                                                       unsigned long long* rng_dev, double* p, double* cum,
                                                       double* seg, double* mbp) {
  __shared__ double sh[1024];
  __shared__ double s_total;
  const int tid = threadIdx.x;
  if (rng_dev) rng = rng_dev[0];
  const long per = (N + 1023) / 1024;
  const long lo = min(N, (long)tid * per), hi = min(N, lo + per);
  double s = 0.0;
  for (long e = lo; e < hi; e++) {
    const double w = exp(alpha * log(l1[e] + 1e-12));
    p[e] = w;
    s += w;
  }
  sh[tid] = s;
  __syncthreads();
  for (int k = 512; k > 0; k >>= 1) {
    if (tid < k) sh[tid] += sh[tid + k];
    __syncthreads();
  }
  const double denom = sh[0] + 1e-6;
  __syncthreads();
  double acc = 0.0;
  for (long e = lo; e < hi; e++) {
    const double q = (p[e] + 1e-6) / denom;
    p[e] = q;
    acc += q;
    cum[e] = acc;
  }
  // exclusive scan of the 1024 run totals: within each warp, then over the 32 warp totals
  const int lane = tid & 31, wid = tid >> 5;
  double inc = acc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) sh[wid] = inc;
  __syncthreads();
  if (wid == 0) {
    double w = sh[lane];
    double winc = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, winc, o);
      if (lane >= o) winc += y;
    }
    sh[32 + lane] = winc - w;  // exclusive offset of warp `lane`
    if (lane == 31) s_total = winc;
  }
  __syncthreads();
  const double off = sh[32 + wid] + (inc - acc);
  for (long e = lo; e < hi; e++) cum[e] += off;
  __syncthreads();
  const double total = s_total;
  for (long i = tid; i < Bmb; i += 1024) {
    unsigned long long z = rng + (unsigned long long)(i + 1) * 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    z ^= z >> 31;
    const double u = (double)(z >> 11) / 9007199254740992.0 * total;
    long a = 0, b = N;
    while (a < b) {
      const long mid = (a + b) >> 1;
      if (cum[mid] >= u)
        b = mid;
      else
        a = mid + 1;
    }
    const long idx = a < N ? a : N - 1;
    seg[i] = (double)idx;
    mbp[i] = exp((-beta) * log((double)N * p[idx] + 1e-12));
  }
  if (rng_dev && tid == 0) rng_dev[0] = rng + (unsigned long long)Bmb * 0x9E3779B97F4A7C15ULL;
}

// ---------------------------------------------------------------- Muon of small matrices
// One CTA does the whole Muon step of one matrix whose short side is at most kSmallSide: Nesterov
// momentum in f64 (the fast tier's nesterov formula), the Frobenius normalisation, every Newton-Schulz
// step in fp32 shared memory (G = X X^T, Pm = b G + c G G, X' = a X + Pm X), and the finalize into the
// f64 master and its bf16 shadow. Replaces a chain of ~18 launches for the action and value heads.
constexpr int kSmallSide = 32;
constexpr int kSmallElems = 16384;  // m * n; two fp32 copies of X stay in shared memory
constexpr int kSmallMaxIters = 16;
struct SmallMat {
  long oW;
  int rows, cols;
  void* Wb;
  long ldw;
  double scale;  // sqrt(max(1, rows/cols))
};
struct SmallMats {
  SmallMat m[4];
  float co[kSmallMaxIters][3];
  int n, iters;
};
__global__ void __launch_bounds__(256) mg_small_muon_kernel(const SmallMats sm, const float* __restrict__ grad,
                                                            const double* __restrict__ cc, double* W, double* mom,
                                                            double mu, double eps, double c1, double lr) {
  extern __shared__ float smf[];
  __shared__ double shd[256];
  const SmallMat& q = sm.m[blockIdx.x];
  const int rows = q.rows, cols = q.cols;
  const bool tr = rows > cols;
  const int m = tr ? cols : rows, n = tr ? rows : cols;
  float* X = smf;
  float* X2 = smf + (long)m * n;
  float* G = X2 + (long)m * n;
  float* Pm = G + m * m;
  const int tid = threadIdx.x;
  const double c = cc[0];
  double s = 0.0;
  for (int i = tid; i < rows * cols; i += 256) {
    const double gi = (double)grad[q.oW + i] * c;
    const double mm = mu * mom[q.oW + i] + gi;
    mom[q.oW + i] = mm;
    const double ui = gi + mu * mm;
    const int r = i / cols, cl = i - r * cols;
    X[tr ? cl * n + r : r * n + cl] = (float)ui;
    s += ui * ui;
  }
  shd[tid] = s;
  __syncthreads();
  for (int k = 128; k > 0; k >>= 1) {
    if (tid < k) shd[tid] += shd[tid + k];
    __syncthreads();
  }
  const float inv = (float)(1.0 / (sqrt(shd[0]) + eps));
  for (int i = tid; i < m * n; i += 256) X[i] *= inv;
  __syncthreads();
  for (int it = 0; it < sm.iters; it++) {
    const float a = sm.co[it][0], bb = sm.co[it][1], cf = sm.co[it][2];
    // G = X X^T: one warp per entry (lanes take every 32nd column, then a fixed shuffle tree), so
    // the long side is not one thread's dependent chain
    for (int e = tid >> 5; e < m * m; e += 8) {
      const int i = e / m, k = e - i * m, ln = tid & 31;
      float acc = 0.f;
      for (int l = ln; l < n; l += 32) acc += X[i * n + l] * X[k * n + l];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (ln == 0) G[e] = acc;
    }
    __syncthreads();
    for (int e = tid; e < m * m; e += 256) {
      const int i = e / m, k = e - i * m;
      float acc = 0.f;
      for (int l = 0; l < m; l++) acc += G[i * m + l] * G[l * m + k];
      Pm[e] = bb * G[e] + cf * acc;
    }
    __syncthreads();
    for (int e = tid; e < m * n; e += 256) {
      const int i = e / n, l = e - i * n;
      float acc = a * X[e];
      for (int k = 0; k < m; k++) acc += Pm[i * m + k] * X[k * n + l];
      X2[e] = acc;
    }
    __syncthreads();
    float* t = X;
    X = X2;
    X2 = t;
  }
  const double c2 = lr * q.scale;
  for (int i = tid; i < rows * cols; i += 256) {
    const int r = i / cols, cl = i - r * cols;
    const double x = (double)X[tr ? cl * n + r : r * n + cl];
    const double w = c1 * W[q.oW + i] + c2 * x;
    W[q.oW + i] = w;
    if (q.Wb) ((__nv_bfloat16*)q.Wb)[r * q.ldw + cl] = __float2bfloat16_rn((float)w);
  }
}
// stepVec of up to four biases in one launch, with their fp32 shadows.
struct BiasList {
  long oB[4];
  int n[4];
  float* shadow[4];
  int count;
};
__global__ void mg_bias_step_kernel(const BiasList bl, const float* __restrict__ grad, const double* __restrict__ cc,
                                    double* W, double* mom, double lr, double wd, double mu) {
  const double c = cc[0];
  for (int q = 0; q < bl.count; q++)
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < bl.n[q]; i += gridDim.x * blockDim.x) {
      const long k = bl.oB[q] + i;
      const double gi = (double)grad[k] * c;
      const double newm = mu * mom[k] + gi;
      const double upd = gi + mu * newm;
      const double nb = W[k] * (1.0 - lr * wd) + lr * upd;
      W[k] = nb;
      mom[k] = newm;
      if (bl.shadow[q]) bl.shadow[q][i] = (float)nb;
    }
}

__global__ void mg_fill_kernel(double* d, double v, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) d[i] = v;
}
__global__ void mg_f64_to_f32_kernel(const double* __restrict__ s, long n, float* d) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    d[i] = (float)s[i];
}

}  // namespace

// ================================================================= session
struct MgShape {
  long D = 0, H = 0, L = 0, A = 0, K = 0;
  int enc_act = 0;
  bool operator==(const MgShape& o) const {
    return D == o.D && H == o.H && L == o.L && A == o.A && K == o.K && enc_act == o.enc_act;
  }
  long P() const { return H * D + H + L * K * H * H + A * H + A + H + 1; }
  long oWenc() const { return 0; }
  long oBenc() const { return H * D; }
  long oLayer(long l) const { return H * D + H + l * K * H * H; }
  long oWdec() const { return H * D + H + L * K * H * H; }
  long oBdec() const { return oWdec() + A * H; }
  long oWval() const { return oBdec() + A; }
  long oBval() const { return oWval() + H; }
};

}  // namespace pl

struct pl_mg {
  int dev = 0;
  long N = 0, T = 0;
  long chain_N = 0, chain_D = 0, chain_LH = 0;  // resident-chaining stamp of the rollout (N = 0: none)
  std::vector<void*> allocs;  // columns and sampling (freed at destroy)
  // resident columns, rows e*T + t (f64)
  double *rew = nullptr, *term = nullptr, *act = nullptr, *logp = nullptr, *val0 = nullptr, *boot = nullptr;
  double *value = nullptr, *ratio = nullptr, *adv = nullptr, *l1 = nullptr;
  bool cols_valid = false;
  // action heads: W = 1 one categorical head; W > 1 multi-discrete heads of sizes hs (act holds W per row)
  int W = 1;
  std::vector<int> hs;
  int* hs_dev = nullptr;
  // obs trajectory
  const float* traj = nullptr;
  float* traj_own = nullptr;
  long trajD = 0;
  bool stamped = false;  // the columns of this update came from pl_mg_stamp_* (read once by pl_mg_take_stamped)
  // prioritised sample
  double *prio_p = nullptr, *prio_cum = nullptr, *seg = nullptr, *mbp = nullptr;
  long seg_cap = 0, prio_B = 0;
  bool prio_fresh = false;
  int* lastw = nullptr;
  // BPTT / Muon workspace (reallocated when the shape, minibatch or tier changes)
  struct Work {
    std::vector<void*> allocs;
    pl::MgShape sh;
    long Bmb = 0, T = 0, R = 0, Dp = 0, Op = 0;
    bool fast = false;
    void* X = nullptr;
    void* Z = nullptr;
    std::vector<void*> h, Y, Os;
    float* Out = nullptr;
    void* dOut = nullptr;
    void* dh[2] = {nullptr, nullptr};
    void* dY = nullptr;
    void* dhn = nullptr;
    int* act_i = nullptr;  // [R x Wact]
    int Wact = 1;
    float *adv_f = nullptr, *ret_f = nullptr, *olp_f = nullptr, *ov_f = nullptr, *term_f = nullptr;
    float *newlp = nullptr, *newval = nullptr, *lossrow = nullptr;
    double* ms = nullptr;
    double* adv_part = nullptr;
    unsigned* adv_counter = nullptr;
    double* obs_in = nullptr;   // host-mode obs upload
    double* scal_in = nullptr;  // host-mode scalars upload
    // weight shadows: fast = bf16 matrices [rows x ld] + fp32 biases; tight = fp32
    void* Wenc = nullptr;
    std::vector<void*> Wl;
    void* Wout = nullptr;
    float *benc = nullptr, *bout = nullptr;
    // gradient and scratch
    float* grad = nullptr;
    float* gout = nullptr;
    float* gbout = nullptr;
    float* colpart = nullptr;
    long colpart_elems = 0;
    float* splitk = nullptr;
    long splitk_elems = 0;
    // Muon
    double* cc = nullptr;
    double* gn_part = nullptr;
    double* g64 = nullptr;
    double* params_in = nullptr;  // host params upload (pl_mg_grad with handle 0)
    pl::NsWork ns, ns2;  // ns2: the Newton-Schulz chains that run on the side stream
    double* exact_ws = nullptr;
  } w;
  cudaStream_t side = nullptr;  // second stream for concurrent Newton-Schulz chains
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  // one minibatch of pl_mg_update captured as a CUDA graph (fast tier), replayed numMB times
  cudaStream_t cap = nullptr;
  cudaGraphExec_t gexec = nullptr;
  std::vector<double> gkey;
  uint64_t gnodes = 0;
  unsigned long long* rng_dev = nullptr;
  bool have_work = false;
  // data parallelism: a communicator from pl_comm_create, this rank and the world size
  void* comm = nullptr;
  int rank = 0, world = 1;
  size_t shadow_src = 0;  // handle whose weights the shadows hold (0 = none / host params)
  bool grad_fresh = false;
  long grad_rows = 0;
  uint64_t launches = 0;
};

namespace pl {
namespace {

template <typename T>
T* mg_alloc(std::vector<void*>& list, size_t n, bool& failed, bool zero = false) {
  void* p = nullptr;
  if (n == 0) n = 1;
  if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) {
    cudaGetLastError();
    failed = true;
    set_error(PL_ERR_NOMEM, "cudaMalloc of %zu bytes failed (MinGRU session)", n * sizeof(T));
    return nullptr;
  }
  if (zero) cudaMemset(p, 0, n * sizeof(T));
  list.push_back(p);
  return (T*)p;
}
void free_list(std::vector<void*>& list) {
  for (void* p : list) cudaFree(p);
  list.clear();
}

int check_net(const pl_mg_net* net) {
  PL_REQUIRE(net != nullptr, PL_ERR_INVALID, "MinGRU: NULL network description");
  PL_REQUIRE(net->D > 0 && net->H > 0 && net->L > 0 && net->A > 0, PL_ERR_INVALID,
             "MinGRU: D, H, L and A must be positive");
  PL_REQUIRE(net->K == 2 || net->K == 3, PL_ERR_INVALID, "MinGRU: K must be 2 or 3 (got %zu)", net->K);
  PL_REQUIRE(net->enc_act == 0 || net->enc_act == 1, PL_ERR_INVALID, "MinGRU: enc_act must be 0 or 1");
  PL_REQUIRE(net->H < (1u << 20) && net->D < (1u << 20) && net->A < 4096 && net->L < 256, PL_ERR_INVALID,
             "MinGRU: network extents out of range");
  return PL_OK;
}
MgShape shape_of(const pl_mg_net* net) {
  MgShape s;
  s.D = (long)net->D;
  s.H = (long)net->H;
  s.L = (long)net->L;
  s.A = (long)net->A;
  s.K = (long)net->K;
  s.enc_act = net->enc_act;
  return s;
}

int ensure_work(pl_mg* s, const MgShape& sh, long Bmb, long T, bool fast) {
  auto& w = s->w;
  if (s->have_work && w.sh == sh && w.Bmb == Bmb && w.T == T && w.fast == fast && w.Wact == s->W) return PL_OK;
  if (fast) PL_REQUIRE(sh.H % 8 == 0, PL_ERR_UNSUPPORTED, "MinGRU bf16 tier needs H %% 8 == 0 (H=%ld)", sh.H);
  free_list(w.allocs);
  s->have_work = false;
  s->shadow_src = 0;
  s->grad_fresh = false;
  w = pl_mg::Work();
  w.sh = sh;
  w.Bmb = Bmb;
  w.T = T;
  w.fast = fast;
  const long R = T * Bmb, H = sh.H, KH = sh.K * sh.H, L = sh.L, A = sh.A;
  w.R = R;
  w.Dp = fast ? rup(sh.D, 64) : sh.D;
  w.Op = fast ? rup(A + 1, 64) : A + 1;
  const size_t es = fast ? 2 : 4;
  bool f = false;
  auto act_buf = [&](long n) -> void* { return (void*)mg_alloc<char>(w.allocs, (size_t)n * es, f); };
  w.X = act_buf(R * w.Dp);
  if (sh.enc_act) w.Z = act_buf(R * H);
  for (long l = 0; l <= L; l++) w.h.push_back(act_buf(R * H));
  for (long l = 0; l < L; l++) {
    w.Y.push_back(act_buf(R * KH));
    w.Os.push_back(act_buf(R * H));
  }
  w.Out = mg_alloc<float>(w.allocs, (size_t)R * w.Op, f);
  w.dOut = act_buf(R * w.Op);
  w.dh[0] = act_buf(R * H);
  w.dh[1] = act_buf(R * H);
  w.dY = act_buf(R * KH);
  if (sh.K == 3) w.dhn = act_buf(R * H);
  w.Wact = s->W;
  w.act_i = mg_alloc<int>(w.allocs, (size_t)R * s->W, f);
  w.adv_f = mg_alloc<float>(w.allocs, R, f);
  w.ret_f = mg_alloc<float>(w.allocs, R, f);
  w.olp_f = mg_alloc<float>(w.allocs, R, f);
  w.ov_f = mg_alloc<float>(w.allocs, R, f);
  w.term_f = mg_alloc<float>(w.allocs, R, f);
  w.newlp = mg_alloc<float>(w.allocs, R, f);
  w.newval = mg_alloc<float>(w.allocs, R, f);
  w.lossrow = mg_alloc<float>(w.allocs, (size_t)R * 8, f);
  w.ms = mg_alloc<double>(w.allocs, 4, f);
  w.adv_part = mg_alloc<double>(w.allocs, kAdvBlocks, f);
  w.adv_counter = mg_alloc<unsigned>(w.allocs, 1, f, true);
  // shadows (zeroed: the padding of the bf16 operands must read as zero)
  w.Wenc = (void*)mg_alloc<char>(w.allocs, (size_t)H * w.Dp * es, f, true);
  for (long l = 0; l < L; l++) w.Wl.push_back((void*)mg_alloc<char>(w.allocs, (size_t)KH * H * es, f, true));
  w.Wout = (void*)mg_alloc<char>(w.allocs, (size_t)w.Op * H * es, f, true);
  w.benc = mg_alloc<float>(w.allocs, H, f, true);
  w.bout = mg_alloc<float>(w.allocs, w.Op, f, true);
  const long P = sh.P();
  w.grad = mg_alloc<float>(w.allocs, P, f);
  w.gout = mg_alloc<float>(w.allocs, (size_t)(A + 1) * H, f);
  w.gbout = mg_alloc<float>(w.allocs, w.Op, f);
  const long chunks = (R + 255) / 256;
  w.colpart_elems = chunks * std::max<long>(H, w.Op);
  // the bf16 tier's last layer-gradient product also leaves per-128-row bias partials of the encoder here
  if (fast) w.colpart_elems = std::max<long>(w.colpart_elems, colsum_scratch_elems((int)((R + 127) / 128), H));
  w.colpart = mg_alloc<float>(w.allocs, w.colpart_elems, f);
  w.splitk_elems = std::max<long>(std::max<long>(8 * KH * H, 64 * (A + 1) * H), 64 * H * std::max<long>(sh.D, 64));
  if (fast) w.splitk = mg_alloc<float>(w.allocs, w.splitk_elems, f);
  w.cc = mg_alloc<double>(w.allocs, 2, f);
  w.gn_part = mg_alloc<double>(w.allocs, 4096, f);
  w.g64 = mg_alloc<double>(w.allocs, P, f);
  w.params_in = mg_alloc<double>(w.allocs, P, f);
  // Muon workspace: every matrix wide-side up (m = min, n = max)
  long mmax = 1, nmax = 1, nprod = 1;
  auto fit = [&](long r, long c) {
    mmax = std::max(mmax, std::min(r, c));
    nmax = std::max(nmax, std::max(r, c));
    nprod = std::max(nprod, r * c);
  };
  fit(H, sh.D);
  fit(KH, H);
  fit(A, H);
  fit(1, H);
  if (fast) {
    const long ldx = rup(nmax, 64), ldg = rup(mmax, 64);
    w.ns.ldx = ldx;
    w.ns.ldg = ldg;
    w.ns.X0 = mg_alloc<bf16>(w.allocs, (size_t)rup(mmax, 128) * ldx, f, true);
    w.ns.X1 = mg_alloc<bf16>(w.allocs, (size_t)rup(mmax, 128) * ldx, f, true);
    w.ns.G = mg_alloc<bf16>(w.allocs, (size_t)rup(mmax, 128) * ldg, f, true);
    w.ns.B = mg_alloc<bf16>(w.allocs, (size_t)rup(mmax, 128) * ldg, f, true);
    w.ns.Xf = mg_alloc<float>(w.allocs, (size_t)mmax * ldx, f);
    w.ns.U = mg_alloc<double>(w.allocs, nprod, f);
    w.ns.part = mg_alloc<double>(w.allocs, 4096, f);
    // the persistent Newton-Schulz chain's per-matrix counters (one matrix per call, each stream its own)
    w.ns.cnt = mg_alloc<unsigned>(w.allocs, (size_t)ns_chain_counter_words(1), f);
    w.ns2 = w.ns;
    w.ns2.cnt = mg_alloc<unsigned>(w.allocs, (size_t)ns_chain_counter_words(1), f);
    w.ns2.X0 = mg_alloc<bf16>(w.allocs, (size_t)rup(mmax, 128) * ldx, f, true);
    w.ns2.X1 = mg_alloc<bf16>(w.allocs, (size_t)rup(mmax, 128) * ldx, f, true);
    w.ns2.G = mg_alloc<bf16>(w.allocs, (size_t)rup(mmax, 128) * ldg, f, true);
    w.ns2.B = mg_alloc<bf16>(w.allocs, (size_t)rup(mmax, 128) * ldg, f, true);
    w.ns2.Xf = mg_alloc<float>(w.allocs, (size_t)mmax * ldx, f);
    w.ns2.U = mg_alloc<double>(w.allocs, nprod, f);
    w.ns2.part = mg_alloc<double>(w.allocs, 4096, f);
    w.ns2.err = nullptr;
  } else {
    size_t ws = std::max(exact_ws_doubles((int)H, (int)sh.D), exact_ws_doubles((int)KH, (int)H));
    ws = std::max(ws, exact_ws_doubles((int)A, (int)H));
    ws = std::max(ws, exact_ws_doubles(1, (int)H));
    w.exact_ws = mg_alloc<double>(w.allocs, ws, f);
  }
  if (f) {
    free_list(w.allocs);
    return PL_ERR_NOMEM;
  }
  PL_CUDA(cudaDeviceSynchronize());  // the zeroing memsets above ran on the legacy stream
  s->have_work = true;
  return PL_OK;
}

// Shadows from f64 params (device): fast = bf16 matrices + fp32 biases, tight = fp32 copies.
int refresh_shadows(pl_mg* s, const double* par, cudaStream_t st) {
  auto& w = s->w;
  const MgShape& sh = w.sh;
  const long H = sh.H, KH = sh.K * sh.H, A = sh.A;
  int rc;
  if (w.fast) {
    rc = launch_w_to_bf16(par + sh.oWenc(), (int)H, (int)sh.D, (bf16*)w.Wenc, w.Dp, st);
    for (long l = 0; !rc && l < sh.L; l++)
      rc = launch_w_to_bf16(par + sh.oLayer(l), (int)KH, (int)H, (bf16*)w.Wl[l], H, st);
    if (!rc) rc = launch_w_to_bf16(par + sh.oWdec(), (int)A, (int)H, (bf16*)w.Wout, H, st);
    if (!rc) rc = launch_w_to_bf16(par + sh.oWval(), 1, (int)H, (bf16*)w.Wout + A * H, H, st);
  } else {
    rc = launch_f64_to_f32(par + sh.oWenc(), H * sh.D, (float*)w.Wenc, st);
    for (long l = 0; !rc && l < sh.L; l++) rc = launch_f64_to_f32(par + sh.oLayer(l), KH * H, (float*)w.Wl[l], st);
    if (!rc) rc = launch_f64_to_f32(par + sh.oWdec(), A * H, (float*)w.Wout, st);
    if (!rc) rc = launch_f64_to_f32(par + sh.oWval(), H, (float*)w.Wout + A * H, st);
  }
  if (!rc) rc = launch_f64_to_f32(par + sh.oBenc(), H, w.benc, st);
  if (!rc) rc = launch_f64_to_f32(par + sh.oBdec(), A, w.bout, st);
  if (!rc) rc = launch_f64_to_f32(par + sh.oBval(), 1, w.bout + A, st);
  return rc;
}

template <typename S>
int colsum(pl_mg* s, const S* M, long R, long ld, int N, float* out, cudaStream_t st) {
  auto& w = s->w;
  const int rows_per = 256;
  const int chunks = (int)((R + rows_per - 1) / rows_per);
  PL_REQUIRE((long)chunks * N <= w.colpart_elems, PL_ERR_INVALID, "MinGRU colsum scratch too small");
  dim3 g1((unsigned)((N + 31) / 32), (unsigned)chunks);
  mg_colsum_part_kernel<S><<<g1, dim3(32, 8), 0, st>>>(M, R, ld, N, rows_per, w.colpart);
  mg_colsum_final_kernel<<<(unsigned)((N + 7) / 8), 256, 0, st>>>(w.colpart, chunks, N, out);
  count_launch(2);
  PL_LAUNCH("mg_colsum_kernel");
  return PL_OK;
}

// Weight gradient C[out x in] (fp32, ld in) = dZ^T Hin over R rows (both MN-major) with split-K
// sized to fill the GPU.
int wgrad_tc(pl_mg* s, const void* dZ, long ldz, int out, const void* Hin, long ldh, int in, long R, float* dst,
             cudaStream_t st) {
  auto& w = s->w;
  Operand A{dZ, R, out, ldz, 1, 0};
  Operand B{Hin, R, in, ldh, 1, 0};
  const int bn = in <= 128 ? 128 : 256;
  const long tiles = ceil_div(out, 128) * ceil_div(in, bn);
  const long kb = ceil_div(R, 64);
  int S = (int)std::min<long>(std::max<long>(1, (2 * 148 + tiles - 1) / tiles), 64);
  while (S > 1 && kb / S < 4) S--;
  while (S > 1 && (long)S * out * in > w.splitk_elems) S--;
  EpiArgs e{};
  e.ldo = in;
  e.out_rows = out;
  e.out_cols = in;
  e.alpha = 1.f;
  if (S == 1) {
    e.out = dst;
    return gemm_launch(bn, EPI_F32, true, true, A, B, out, in, (int)R, 1, e, st);
  }
  e.out = w.splitk;
  e.out_bstride = (long)out * in;
  e.k_splits = S;
  int rc = gemm_launch(bn, EPI_F32, true, true, A, B, out, in, (int)R, 1, e, st);
  if (rc) return rc;
  return launch_splitk_reduce(w.splitk, S, (long)out * in, dst, st);
}

inline int pick_bn_n(long n) { return n <= 64 ? 64 : (n <= 128 ? 128 : 256); }

// Scan launches: the bf16 tier takes two columns per thread and the fast logistic; the fp32 tier
// one column and the accurate one (it is the parity tier).
template <typename S>
int launch_scan_fwd(const void* Y, const void* hin, void* hout, void* Os, const float* term, int B, int H, int T, int K,
                    cudaStream_t st) {
  constexpr bool FAST = std::is_same<S, bf16>::value;
  constexpr int VEC = FAST ? 2 : 1;
  const unsigned nb = (unsigned)(((long)B * (H / VEC) + 255) / 256);
  if (K == 3)
    mg_scan_fwd_kernel<S, 3, VEC, FAST><<<nb, 256, 0, st>>>((const S*)Y, (const S*)hin, (S*)hout, (S*)Os, term, B, H, T);
  else
    mg_scan_fwd_kernel<S, 2, VEC, FAST><<<nb, 256, 0, st>>>((const S*)Y, (const S*)hin, (S*)hout, (S*)Os, term, B, H, T);
  count_launch();
  PL_LAUNCH("mg_scan_fwd_kernel");
  return PL_OK;
}
template <typename S>
int launch_scan_bwd(const void* Y, const void* Os, const void* hin, const void* dh, void* dY, void* dhn,
                    const float* term, int B, int H, int T, int K, cudaStream_t st) {
  constexpr bool FAST = std::is_same<S, bf16>::value;
  constexpr int VEC = FAST ? 2 : 1;
  const unsigned nb = (unsigned)(((long)B * (H / VEC) + 255) / 256);
  if (K == 3)
    mg_scan_bwd_kernel<S, 3, VEC, FAST><<<nb, 256, 0, st>>>((const S*)Y, (const S*)Os, (const S*)hin, (const S*)dh,
                                                             (S*)dY, (S*)dhn, term, B, H, T);
  else
    mg_scan_bwd_kernel<S, 2, VEC, FAST><<<nb, 256, 0, st>>>((const S*)Y, (const S*)Os, (const S*)hin, (const S*)dh,
                                                             (S*)dY, nullptr, term, B, H, T);
  count_launch();
  PL_LAUNCH("mg_scan_bwd_kernel");
  return PL_OK;
}

// The BPTT gradient of the minibatch already gathered into the work buffers (X, act_i, adv_f,
// ret_f, olp_f, ov_f, term_f): forward, PPO head, backward; summed gradient into w.grad.
template <typename S>
int bptt(pl_mg* s, double vf, double ent, double clip, double vfclip, bool losses, cudaStream_t st) {
  auto& w = s->w;
  const MgShape& sh = w.sh;
  const long R = w.R, H = sh.H, KH = sh.K * sh.H, L = sh.L, A = sh.A, D = sh.D;
  const int Bmb = (int)w.Bmb, T = (int)w.T;
  const bool fast = w.fast;
  const int enc_act = sh.enc_act ? 1 : 2;
  float* grad = w.grad;
  int rc;
  // ---- encoder: h0 = enc(X W_enc^T + b_enc)
  if (fast) {
    Operand opA{w.X, R, w.Dp, w.Dp, 1, 0};
    Operand opB{w.Wenc, H, w.Dp, w.Dp, 1, 0};
    EpiArgs e{};
    e.out = w.h[0];
    e.ldo = H;
    e.out_rows = (int)R;
    e.out_cols = (int)H;
    e.bias = w.benc;
    e.act = enc_act;
    e.out2 = sh.enc_act ? w.Z : nullptr;
    e.ldo2 = H;
    rc = gemm_launch(pick_bn_n(H), EPI_FWD, false, false, opA, opB, (int)R, (int)H, (int)w.Dp, 1, e, st);
  } else {
    float* Z = sh.enc_act ? (float*)w.Z : (float*)w.h[0];
    rc = launch_sgemm((int)R, (int)H, (int)D, (const float*)w.X, D, 1, (const float*)w.Wenc, D, 1, Z, H, 1.f, st);
    if (!rc) rc = launch_bias_act_f32(Z, sh.enc_act ? (float*)w.h[0] : nullptr, w.benc, R, (int)H, enc_act, st);
  }
  if (rc) return rc;
  // ---- layers
  for (long l = 0; l < L; l++) {
    if (fast) {
      Operand opA{w.h[l], R, H, H, 1, 0};
      Operand opB{w.Wl[l], KH, H, H, 1, 0};
      EpiArgs e{};
      e.out = w.Y[l];
      e.ldo = KH;
      e.out_rows = (int)R;
      e.out_cols = (int)KH;
      e.alpha = 1.f;
      rc = gemm_launch(256, EPI_BF16, false, false, opA, opB, (int)R, (int)KH, (int)H, 1, e, st);
    } else {
      rc = launch_sgemm((int)R, (int)KH, (int)H, (const float*)w.h[l], H, 1, (const float*)w.Wl[l], H, 1,
                        (float*)w.Y[l], KH, 1.f, st);
    }
    if (rc) return rc;
    rc = launch_scan_fwd<S>(w.Y[l], w.h[l], w.h[l + 1], w.Os[l], w.term_f, Bmb, (int)H, T, (int)sh.K, st);
    if (rc) return rc;
  }
  // ---- heads: Out = h_L W_out^T (bias added by the row kernel)
  if (fast) {
    Operand opA{w.h[L], R, H, H, 1, 0};
    Operand opB{w.Wout, w.Op, H, H, 1, 0};
    EpiArgs e{};
    e.out = w.Out;
    e.ldo = w.Op;
    e.out_rows = (int)R;
    e.out_cols = (int)(A + 1);
    e.alpha = 1.f;
    rc = gemm_launch(128, EPI_F32, false, false, opA, opB, (int)R, (int)(A + 1), (int)H, 1, e, st);
  } else {
    rc = launch_sgemm((int)R, (int)(A + 1), (int)H, (const float*)w.h[L], H, 1, (const float*)w.Wout, H, 1, w.Out,
                      w.Op, 1.f, st);
  }
  if (rc) return rc;
  if (s->W > 1) {
    mg_ppo_rows_md_kernel<S><<<blocks_for(R, 128), 128, 0, st>>>(
        w.Out, (int)w.Op, w.bout, R, (int)A, (int)w.Op, s->W, s->hs_dev, w.act_i, w.adv_f, w.ret_f, w.olp_f, w.ov_f,
        (float)vf, (float)ent, (float)clip, (float)vfclip, (S*)w.dOut, w.newlp, w.newval,
        losses ? w.lossrow : nullptr);
    count_launch();
    PL_LAUNCH("mg_ppo_rows_md_kernel");
  } else {
    mg_ppo_rows_kernel<S><<<blocks_for(R, 128), 128, 0, st>>>(
        w.Out, (int)w.Op, w.bout, R, (int)A, (int)w.Op, w.act_i, w.adv_f, w.ret_f, w.olp_f, w.ov_f, (float)vf,
        (float)ent, (float)clip, (float)vfclip, (S*)w.dOut, w.newlp, w.newval, losses ? w.lossrow : nullptr);
    count_launch();
    PL_LAUNCH("mg_ppo_rows_kernel");
  }
  // ---- head gradients
  rc = colsum<S>(s, (const S*)w.dOut, R, w.Op, (int)(A + 1), w.gbout, st);
  if (rc) return rc;
  if (fast)
    rc = wgrad_tc(s, w.dOut, w.Op, (int)(A + 1), w.h[L], H, (int)H, R, w.gout, st);
  else
    rc = launch_sgemm((int)(A + 1), (int)H, (int)R, (const float*)w.dOut, 1, w.Op, (const float*)w.h[L], 1, H, w.gout,
                      H, 1.f, st);
  if (rc) return rc;
  mg_head_scatter_kernel<<<blocks_for((A + 1) * H), 256, 0, st>>>(w.gout, w.gbout, (int)A, (int)H,
                                                                   grad + sh.oWdec(), grad + sh.oBdec(),
                                                                   grad + sh.oWval(), grad + sh.oBval());
  count_launch();
  PL_LAUNCH("mg_head_scatter_kernel");
  // dh_L = dOut W_out
  int cur = 0;
  if (fast) {
    Operand opA{w.dOut, R, w.Op, w.Op, 1, 0};
    Operand opB{w.Wout, w.Op, H, H, 1, 0};  // MN-major: rows = K (outputs), cols = N (hidden)
    EpiArgs e{};
    e.out = w.dh[cur];
    e.ldo = H;
    e.out_rows = (int)R;
    e.out_cols = (int)H;
    e.alpha = 1.f;
    rc = gemm_launch(256, EPI_BF16, false, true, opA, opB, (int)R, (int)H, (int)w.Op, 1, e, st);
  } else {
    rc = launch_sgemm((int)R, (int)H, (int)(A + 1), (const float*)w.dOut, w.Op, 1, (const float*)w.Wout, 1, H,
                      (float*)w.dh[cur], H, 1.f, st);
  }
  if (rc) return rc;
  // ---- layers, top down
  bool enc_fused = false;
  for (long l = L - 1; l >= 0; l--) {
    rc = launch_scan_bwd<S>(w.Y[l], w.Os[l], w.h[l], w.dh[cur], w.dY, sh.K == 3 ? w.dhn : nullptr, w.term_f, Bmb,
                            (int)H, T, (int)sh.K, st);
    if (rc) return rc;
    // dW_l = dY^T h_l
    if (fast)
      rc = wgrad_tc(s, w.dY, KH, (int)KH, w.h[l], H, (int)H, R, grad + sh.oLayer(l), st);
    else
      rc = launch_sgemm((int)KH, (int)H, (int)R, (const float*)w.dY, 1, KH, (const float*)w.h[l], 1, H,
                        grad + sh.oLayer(l), H, 1.f, st);
    if (rc) return rc;
    // dh_l = dY W_l (+ the highway part)
    const int nxt = cur ^ 1;
    if (fast) {
      Operand opA{w.dY, R, KH, KH, 1, 0};
      Operand opB{w.Wl[l], KH, H, H, 1, 0};  // MN-major: rows = K (= K*H), cols = N (= H)
      EpiArgs e{};
      e.out = w.dh[nxt];
      e.ldo = H;
      e.out_rows = (int)R;
      e.out_cols = (int)H;
      e.alpha = 1.f;
      if (sh.K == 3) {
        e.aux = (const bf16*)w.dhn;
        e.ld_aux = H;
        e.beta = 1.f;
      }
      if (l == 0 && sh.K != 3 && sh.enc_act) {
        // the encoder's data gradient in this product's epilogue: dE = (dY W_0) x GELU'(Z) with the
        // encoder bias partials per 128-row tile (no separate activation and column-sum passes)
        e.aux = (const bf16*)w.Z;
        e.ld_aux = H;
        e.act = 1;
        e.colsum = w.colpart;
        e.ld_colsum = H;
        enc_fused = true;
        rc = gemm_launch(256, EPI_DGRAD, false, true, opA, opB, (int)R, (int)H, (int)KH, 1, e, st);
      } else {
        rc = gemm_launch(256, EPI_BF16, false, true, opA, opB, (int)R, (int)H, (int)KH, 1, e, st);
      }
    } else {
      rc = launch_sgemm((int)R, (int)H, (int)KH, (const float*)w.dY, KH, 1, (const float*)w.Wl[l], 1, H,
                        (float*)w.dh[nxt], H, 1.f, st);
      if (!rc && sh.K == 3) {
        mg_axpy_kernel<<<blocks_for(R * H), 256, 0, st>>>((float*)w.dh[nxt], (const float*)w.dhn, R * H);
        count_launch();
        PL_LAUNCH("mg_axpy_kernel");
      }
    }
    if (rc) return rc;
    cur = nxt;
  }
  // ---- encoder gradients
  if (enc_fused) {
    rc = launch_colsum_reduce(w.colpart, (int)((R + 127) / 128), H, (int)H, grad + sh.oBenc(), st);
  } else {
    if (sh.enc_act) {
      mg_act_grad_kernel<S><<<blocks_for(R * H), 256, 0, st>>>((S*)w.dh[cur], (const S*)w.Z, R * H, 1);
      count_launch();
      PL_LAUNCH("mg_act_grad_kernel");
    }
    rc = colsum<S>(s, (const S*)w.dh[cur], R, H, (int)H, grad + sh.oBenc(), st);
  }
  if (rc) return rc;
  if (fast) {
    // dW_enc [H x D] = dE^T X (X padded to Dp; only D columns are written)
    auto& ww = s->w;
    Operand opA{ww.dh[cur], R, H, H, 1, 0};
    Operand opB{ww.X, R, ww.Dp, ww.Dp, 1, 0};
    const int bn = D <= 128 ? 128 : 256;
    const long tiles = ceil_div(H, 128) * ceil_div(D, bn);
    const long kb = ceil_div(R, 64);
    int Sk = (int)std::min<long>(std::max<long>(1, (2 * 148 + tiles - 1) / tiles), 64);
    while (Sk > 1 && kb / Sk < 4) Sk--;
    while (Sk > 1 && (long)Sk * H * D > ww.splitk_elems) Sk--;
    EpiArgs e{};
    e.ldo = D;
    e.out_rows = (int)H;
    e.out_cols = (int)D;
    e.alpha = 1.f;
    if (Sk == 1) {
      e.out = grad + sh.oWenc();
      rc = gemm_launch(bn, EPI_F32, true, true, opA, opB, (int)H, (int)D, (int)R, 1, e, st);
    } else {
      e.out = ww.splitk;
      e.out_bstride = H * D;
      e.k_splits = Sk;
      rc = gemm_launch(bn, EPI_F32, true, true, opA, opB, (int)H, (int)D, (int)R, 1, e, st);
      if (!rc) rc = launch_splitk_reduce(ww.splitk, Sk, H * D, grad + sh.oWenc(), st);
    }
  } else {
    rc = launch_sgemm((int)H, (int)D, (int)R, (const float*)w.dh[cur], 1, H, (const float*)w.X, 1, D,
                      grad + sh.oWenc(), D, 1.f, st);
  }
  return rc;
}

int run_bptt(pl_mg* s, double vf, double ent, double clip, double vfclip, bool losses, cudaStream_t st) {
  return s->w.fast ? bptt<bf16>(s, vf, ent, clip, vfclip, losses, st) : bptt<float>(s, vf, ent, clip, vfclip, losses, st);
}

// 7-loss channel reduction (the reference's host fold, ffi/puffercuda.cu:5446-5484)
int reduce_losses(pl_mg* s, double vfCoef, double entCoef, double out[7], cudaStream_t st) {
  auto& w = s->w;
  std::vector<float> h((size_t)w.R * 8);
  PL_CUDA(cudaMemcpyAsync(h.data(), w.lossrow, sizeof(float) * h.size(), cudaMemcpyDeviceToHost, st));
  PL_CUDA(cudaStreamSynchronize(st));
  double sPg = 0, sV = 0, sEnt = 0, sOld = 0, sKl = 0, nclip = 0;
  for (long r = 0; r < w.R; r++) {
    const float* q = h.data() + r * 8;
    sPg += q[0];
    sV += q[1];
    sEnt += q[2];
    sOld += q[3];
    sKl += q[4];
    nclip += q[5];
  }
  const double n = (double)w.R;
  out[0] = sPg / n;
  out[1] = sV / n;
  out[2] = sEnt / n;
  out[3] = out[0] + vfCoef * out[1] - entCoef * out[2];
  out[4] = sOld / n;
  out[5] = sKl / n;
  out[6] = nclip / n;
  return PL_OK;
}

int muon_step(pl_mg* s, size_t handle, const double* gClip, double lr, double wd, double mu, double eps,
              double maxGradNorm, double gscale, const double* coeffs, int iters, cudaStream_t st) {
  auto& w = s->w;
  const MgShape& sh = w.sh;
  const long P = sh.P(), H = sh.H, KH = sh.K * sh.H, A = sh.A;
  double* pm = (double*)handle;
  double* mom = pm + P;
  int rc = PL_OK;
  struct Mat {
    long rows, cols, oW;
    void* shadow;
    long ldw;
  };
  struct Bias {
    long n, oB;
    float* shadow;
  };
  std::vector<Mat> mats;
  mats.push_back({H, sh.D, sh.oWenc(), w.Wenc, w.Dp});
  for (long l = 0; l < sh.L; l++) mats.push_back({KH, H, sh.oLayer(l), w.Wl[l], H});
  mats.push_back({A, H, sh.oWdec(), w.Wout, H});
  const size_t es = w.fast ? 2 : 4;
  mats.push_back({1, H, sh.oWval(), (char*)w.Wout + (size_t)A * H * es, H});
  const Bias biases[3] = {{H, sh.oBenc(), w.benc}, {A, sh.oBdec(), w.bout}, {1, sh.oBval(), w.bout + A}};
  if (gClip) {
    // an already clipped host gradient: cc = 1
    if (w.fast) {
      PL_CUDA(cudaMemcpyAsync(w.g64, gClip, sizeof(double) * P, cudaMemcpyHostToDevice, st));
      mg_f64_to_f32_kernel<<<blocks_for(P), 256, 0, st>>>(w.g64, P, w.grad);
      mg_fill_kernel<<<1, 32, 0, st>>>(w.cc, 1.0, 1);
      count_launch(2);
      PL_LAUNCH("mg_gclip_upload");
    }
  } else {
    PL_REQUIRE(s->grad_fresh, PL_ERR_INVALID,
               "MinGRU Muon: no resident gradient (call pl_mg_grad first, or pass a clipped host gradient)");
    rc = launch_gradnorm(w.grad, P, gscale, maxGradNorm, w.gn_part, w.cc, st);
    if (rc) return rc;
  }
  s->grad_fresh = false;
  if (w.fast) {
    // Matrices with a short side of at most kSmallSide take the one-launch fused step; the others run
    // their tensor-core Newton-Schulz chains alternately on the caller's stream and the side stream.
    SmallMats sm{};
    sm.iters = iters;
    const bool small_ok = iters <= kSmallMaxIters;
    for (int i = 0; small_ok && i < iters; i++)
      for (int k = 0; k < 3; k++) sm.co[i][k] = (float)coeffs[3 * i + k];
    std::vector<const Mat*> big;
    size_t small_smem = 0;
    for (const Mat& m : mats) {
      const long mm = std::min(m.rows, m.cols);
      if (small_ok && sm.n < 4 && mm <= kSmallSide && m.rows * m.cols <= kSmallElems) {
        const double r = (double)m.rows / (double)m.cols;
        sm.m[sm.n++] = SmallMat{m.oW, (int)m.rows, (int)m.cols, m.shadow, m.ldw, sqrt(r > 1.0 ? r : 1.0)};
        small_smem = std::max(small_smem, (size_t)(2 * m.rows * m.cols + 2 * mm * mm) * sizeof(float));
      } else {
        big.push_back(&m);
      }
    }
    const bool two = big.size() > 1;
    if (two) {
      if (!s->side) {
        PL_CUDA(cudaStreamCreateWithFlags(&s->side, cudaStreamNonBlocking));
        PL_CUDA(cudaEventCreateWithFlags(&s->ev_fork, cudaEventDisableTiming));
        PL_CUDA(cudaEventCreateWithFlags(&s->ev_join, cudaEventDisableTiming));
      }
      PL_CUDA(cudaEventRecord(s->ev_fork, st));
      PL_CUDA(cudaStreamWaitEvent(s->side, s->ev_fork, 0));
    }
    for (size_t q = 0; q < big.size(); q++) {
      const Mat& m = *big[q];
      const bool on_side = two && (q % 2 == 1);
      cudaStream_t ms = on_side ? s->side : st;
      NsWork& ns = on_side ? w.ns2 : w.ns;
      const long n = m.rows * m.cols;
      const int mm = (int)std::min(m.rows, m.cols), nn = (int)std::max(m.rows, m.cols);
      int nparts = 0;
      rc = launch_nesterov(w.grad + m.oW, w.cc, mom + m.oW, ns.U, mu, n, ns.part, &nparts, ms);
      if (!rc) rc = launch_ns_input(ns.U, ns.part, nparts, (int)m.rows, (int)m.cols, eps, ns.X0, ns.ldx, ms);
      if (!rc) rc = ns_run(mm, nn, coeffs, iters, ns, ns.X0, ns.ldx, ns.Xf, ns.ldx, ms);
      const double r = (double)m.rows / (double)m.cols;
      if (!rc)
        rc = launch_ns_finalize(ns.Xf, ns.ldx, (int)m.rows, (int)m.cols, 1.0 - lr * wd, lr * sqrt(r > 1.0 ? r : 1.0),
                                pm + m.oW, (bf16*)m.shadow, m.ldw, ms);
      if (rc) return rc;
    }
    if (sm.n > 0) {
      PL_CUDA(cudaFuncSetAttribute((const void*)mg_small_muon_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)((2 * kSmallElems + 2 * kSmallSide * kSmallSide) * sizeof(float))));
      mg_small_muon_kernel<<<sm.n, 256, small_smem, st>>>(sm, w.grad, w.cc, pm, mom, mu, eps, 1.0 - lr * wd, lr);
      count_launch();
      PL_LAUNCH("mg_small_muon_kernel");
    }
    BiasList bl{};
    for (const Bias& b : biases) {
      bl.oB[bl.count] = b.oB;
      bl.n[bl.count] = (int)b.n;
      bl.shadow[bl.count] = b.shadow;
      bl.count++;
    }
    mg_bias_step_kernel<<<(unsigned)std::max<long>(1, (H + 255) / 256), 256, 0, st>>>(bl, w.grad, w.cc, pm, mom, lr, wd,
                                                                                      mu);
    count_launch();
    PL_LAUNCH("mg_bias_step_kernel");
    if (two) {
      PL_CUDA(cudaEventRecord(s->ev_join, s->side));
      PL_CUDA(cudaStreamWaitEvent(st, s->ev_join, 0));
    }
  } else {
    double cc = 1.0;
    if (gClip) {
      PL_CUDA(cudaMemcpyAsync(w.g64, gClip, sizeof(double) * P, cudaMemcpyHostToDevice, st));
    } else {
      PL_CUDA(cudaMemcpyAsync(&cc, w.cc, sizeof(double), cudaMemcpyDeviceToHost, st));
      PL_CUDA(cudaStreamSynchronize(st));
      rc = launch_f32_to_f64(w.grad, P, w.g64, st);
      if (rc) return rc;
    }
    rc = set_ns_coeffs(coeffs, iters, st);
    if (rc) return rc;
    for (const Mat& m : mats) {
      rc = muon_mat_exact((int)m.rows, (int)m.cols, pm + m.oW, mom + m.oW, w.g64 + m.oW, cc, lr, wd, mu, eps, iters,
                          w.exact_ws, st);
      if (rc) return rc;
    }
    for (const Bias& b : biases) {
      rc = stepvec_launch(pm + b.oB, mom + b.oB, w.g64 + b.oB, lr, wd, mu, cc, b.n, st);
      if (rc) return rc;
    }
    rc = refresh_shadows(s, pm, st);
    if (rc) return rc;
  }
  s->shadow_src = handle;
  return PL_OK;
}

// Multi-discrete heads must cover the network's A logits exactly.
int check_heads(const pl_mg* s, const pl_mg_net* net) {
  if (s->W <= 1) return PL_OK;
  PL_REQUIRE((int)s->hs.size() == s->W, PL_ERR_INVALID,
             "MinGRU: %d-wide action column but no head sizes (pl_mg_set_heads with the sizes)", s->W);
  long sum = 0;
  for (int v : s->hs) sum += v;
  PL_REQUIRE(sum == (long)net->A, PL_ERR_INVALID, "MinGRU: head sizes sum to %ld, the network has A = %zu logits", sum,
             net->A);
  return PL_OK;
}

int alloc_columns(pl_mg* s) {
  bool f = false;
  const size_t NT = (size_t)s->N * s->T;
  s->rew = mg_alloc<double>(s->allocs, NT, f);
  s->term = mg_alloc<double>(s->allocs, NT, f);
  s->act = mg_alloc<double>(s->allocs, NT, f);
  s->logp = mg_alloc<double>(s->allocs, NT, f);
  s->val0 = mg_alloc<double>(s->allocs, NT, f);
  s->boot = mg_alloc<double>(s->allocs, s->N, f);
  s->value = mg_alloc<double>(s->allocs, NT, f);
  s->ratio = mg_alloc<double>(s->allocs, NT, f);
  s->adv = mg_alloc<double>(s->allocs, NT, f);
  s->l1 = mg_alloc<double>(s->allocs, s->N, f);
  s->prio_p = mg_alloc<double>(s->allocs, s->N, f);
  s->prio_cum = mg_alloc<double>(s->allocs, s->N, f);
  s->lastw = mg_alloc<int>(s->allocs, s->N, f);
  s->rng_dev = mg_alloc<unsigned long long>(s->allocs, 1, f);
  return f ? PL_ERR_NOMEM : PL_OK;
}

int ensure_sample(pl_mg* s, long Bmb) {
  if (Bmb <= s->seg_cap) return PL_OK;
  bool f = false;
  s->seg = mg_alloc<double>(s->allocs, Bmb, f);
  s->mbp = mg_alloc<double>(s->allocs, Bmb, f);
  if (f) return PL_ERR_NOMEM;
  s->seg_cap = Bmb;
  return PL_OK;
}

// exact: the reference's sequential f64 order (bit-identical, one thread per segment); otherwise the
// warp-parallel f64 scan (coalesced, about 1e-15 relative), which the bf16 tier's update uses.
int mg_vtrace_dev(pl_mg* s, double gamma, double lam, double rho, double c, cudaStream_t st, bool exact = true) {
  PL_REQUIRE(s->cols_valid, PL_ERR_INVALID, "MinGRU: no columns (call pl_mg_set_columns first)");
  if (!exact)
    return pl_vtrace_f64_scan_dev(s->rew, s->value, s->term, s->ratio, s->boot, (size_t)s->N, (size_t)s->T, gamma,
                                  lam, rho, c, s->adv, s->l1, st);
  return pl_vtrace_f64_dev(s->rew, s->value, s->term, s->ratio, s->boot, (size_t)s->N, (size_t)s->T, gamma, lam, rho,
                           c, s->adv, s->l1, st);
}

}  // namespace
}  // namespace pl

// ================================================================= C API
extern "C" {

size_t pl_mg_param_count(const pl_mg_net* net) {
  if (pl::check_net(net)) return 0;
  return (size_t)pl::shape_of(net).P();
}

int pl_mg_create(size_t N, size_t T, pl_mg** out) {
  using namespace pl;
  PL_REQUIRE(out != nullptr, PL_ERR_INVALID, "pl_mg_create: NULL out");
  *out = nullptr;
  PL_REQUIRE(N > 0 && T > 0 && N < (1u << 30) && T < (1u << 20) && N * T < (1ull << 31), PL_ERR_INVALID,
             "pl_mg_create: bad extents N=%zu T=%zu", N, T);
  int rc = require_device();
  if (rc) return rc;
  pl_mg* s = new pl_mg();
  PL_CUDA(cudaGetDevice(&s->dev));
  s->N = (long)N;
  s->T = (long)T;
  rc = alloc_columns(s);
  if (rc) {
    free_list(s->allocs);
    delete s;
    return rc;
  }
  *out = s;
  return PL_OK;
}

int pl_mg_destroy(pl_mg* s) {
  if (!s) return PL_OK;
  cudaDeviceSynchronize();
  pl::free_list(s->w.allocs);
  pl::free_list(s->allocs);
  if (s->traj_own) cudaFree(s->traj_own);
  if (s->gexec) cudaGraphExecDestroy(s->gexec);
  if (s->cap) cudaStreamDestroy(s->cap);
  if (s->side) cudaStreamDestroy(s->side);
  if (s->ev_fork) cudaEventDestroy(s->ev_fork);
  if (s->ev_join) cudaEventDestroy(s->ev_join);
  delete s;
  return PL_OK;
}

static int mg_set_columns_impl(pl_mg* s, const double* rew, const double* term, const double* act, const double* logp,
                               const double* val, const double* boot, cudaMemcpyKind kind, cudaStream_t st) {
  using namespace pl;
  PL_REQUIRE(s && rew && term && act && logp && val && boot, PL_ERR_INVALID, "pl_mg_set_columns: NULL argument");
  const size_t NT = (size_t)s->N * s->T;
  PL_CUDA(cudaMemcpyAsync(s->rew, rew, NT * 8, kind, st));
  PL_CUDA(cudaMemcpyAsync(s->term, term, NT * 8, kind, st));
  PL_CUDA(cudaMemcpyAsync(s->act, act, NT * (size_t)s->W * 8, kind, st));
  PL_CUDA(cudaMemcpyAsync(s->logp, logp, NT * 8, kind, st));
  PL_CUDA(cudaMemcpyAsync(s->val0, val, NT * 8, kind, st));
  PL_CUDA(cudaMemcpyAsync(s->boot, boot, (size_t)s->N * 8, kind, st));
  PL_CUDA(cudaMemcpyAsync(s->value, s->val0, NT * 8, cudaMemcpyDeviceToDevice, st));
  mg_fill_kernel<<<blocks_for((long)NT), 256, 0, st>>>(s->ratio, 1.0, (long)NT);
  count_launch();
  PL_LAUNCH("mg_fill_kernel");
  s->cols_valid = true;
  s->prio_fresh = false;
  s->stamped = false;
  return PL_OK;
}

int pl_mg_set_columns(pl_mg* s, const double* rew, const double* term, const double* act, const double* logp,
                      const double* val, const double* boot) {
  int rc = mg_set_columns_impl(s, rew, term, act, logp, val, boot, cudaMemcpyHostToDevice, 0);
  if (rc) return rc;
  PL_CUDA(cudaStreamSynchronize(0));
  return PL_OK;
}

int pl_mg_set_columns_dev(pl_mg* s, const double* rew, const double* term, const double* act, const double* logp,
                          const double* val, const double* boot, void* stream) {
  return mg_set_columns_impl(s, rew, term, act, logp, val, boot, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
}

int pl_mg_set_heads(pl_mg* s, size_t W, const double* head_sizes) {
  using namespace pl;
  PL_REQUIRE(s != nullptr && W >= 1 && W <= 4096, PL_ERR_INVALID, "pl_mg_set_heads: bad width %zu", W);
  if ((int)W != s->W) {
    // the action column changes width: reallocate it; the columns must be set again
    bool f = false;
    s->act = mg_alloc<double>(s->allocs, (size_t)s->N * s->T * W, f);
    if (f) return PL_ERR_NOMEM;
    s->W = (int)W;
    s->cols_valid = false;
    s->prio_fresh = false;
    s->hs.clear();
    s->hs_dev = W > 1 ? mg_alloc<int>(s->allocs, W, f) : nullptr;
    if (f) return PL_ERR_NOMEM;
  }
  if (W > 1 && head_sizes) {
    std::vector<int> hv(W);
    for (size_t i = 0; i < W; i++) {
      hv[i] = (int)head_sizes[i];
      PL_REQUIRE(hv[i] >= 1, PL_ERR_INVALID, "pl_mg_set_heads: head %zu has size %d", i, hv[i]);
    }
    if (hv != s->hs) {
      PL_CUDA(cudaMemcpy(s->hs_dev, hv.data(), sizeof(int) * W, cudaMemcpyHostToDevice));
      s->hs = hv;
    }
  }
  return PL_OK;
}

int pl_mg_set_comm(pl_mg* s, void* comm, int rank, int world) {
  using namespace pl;
  PL_REQUIRE(s != nullptr && world >= 1 && rank >= 0 && rank < world, PL_ERR_INVALID,
             "pl_mg_set_comm: bad rank %d / world %d", rank, world);
  PL_REQUIRE(world == 1 || comm != nullptr, PL_ERR_INVALID, "pl_mg_set_comm: world %d needs a communicator", world);
  PL_REQUIRE(world == 1 || pl_comm_aborted(comm) == 0, PL_ERR_INVALID,
             "pl_mg_set_comm: not a live communicator from pl_comm_create");
  s->comm = world > 1 ? comm : nullptr;
  s->rank = rank;
  s->world = world;
  return PL_OK;
}

int pl_mg_set_obs(pl_mg* s, const double* obs, size_t D) {
  using namespace pl;
  PL_REQUIRE(s && obs && D > 0, PL_ERR_INVALID, "pl_mg_set_obs: bad argument");
  const size_t n = (size_t)s->N * s->T * D;
  if (s->traj_own && s->trajD != (long)D) {
    cudaFree(s->traj_own);
    s->traj_own = nullptr;
  }
  if (!s->traj_own) {
    if (cudaMalloc(&s->traj_own, n * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      s->traj_own = nullptr;
      return set_error(PL_ERR_NOMEM, "pl_mg_set_obs: cudaMalloc of %zu bytes failed", n * sizeof(float));
    }
  }
  double* tmp = (double*)scratch(20, n * sizeof(double));
  if (!tmp) return PL_ERR_NOMEM;
  PL_CUDA(cudaMemcpy(tmp, obs, n * sizeof(double), cudaMemcpyHostToDevice));
  mg_f64_to_f32_kernel<<<blocks_for((long)n), 256>>>(tmp, (long)n, s->traj_own);
  count_launch();
  PL_LAUNCH("mg_f64_to_f32_kernel");
  PL_CUDA(cudaDeviceSynchronize());
  s->traj = s->traj_own;
  s->trajD = (long)D;
  return PL_OK;
}

// ---------------------------------------------------------------- rollout-side column producer
static int mg_own_traj(pl_mg* s, size_t D) {
  using namespace pl;
  const size_t n = (size_t)s->N * s->T * D;
  if (s->traj_own && s->trajD != (long)D) {
    cudaFree(s->traj_own);
    s->traj_own = nullptr;
  }
  if (!s->traj_own) {
    if (cudaMalloc(&s->traj_own, n * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      s->traj_own = nullptr;
      return set_error(PL_ERR_NOMEM, "MinGRU obs trajectory: cudaMalloc of %zu bytes failed", n * sizeof(float));
    }
  }
  s->traj = s->traj_own;
  s->trajD = (long)D;
  return PL_OK;
}

int pl_mg_stamp_step(pl_mg* s, size_t step, size_t e0, size_t ne, const double* act, const double* logp,
                     const double* val, const float* obs, size_t D, void* stream) {
  using namespace pl;
  PL_REQUIRE(s && act && logp && val, PL_ERR_INVALID, "pl_mg_stamp_step: NULL argument");
  PL_REQUIRE(step < (size_t)s->T && e0 + ne <= (size_t)s->N, PL_ERR_INVALID,
             "pl_mg_stamp_step: step %zu / envs [%zu, %zu) outside %ld x %ld", step, e0, e0 + ne, s->N, s->T);
  cudaStream_t st = (cudaStream_t)stream;
  int rc = launch_stamp_rows_f64(s->act, s->W, s->T, (long)step, (long)e0, (long)ne, act, st);
  if (!rc) rc = launch_stamp_rows_f64(s->logp, 1, s->T, (long)step, (long)e0, (long)ne, logp, st);
  if (!rc) rc = launch_stamp_rows_f64(s->val0, 1, s->T, (long)step, (long)e0, (long)ne, val, st);
  if (!rc) rc = launch_stamp_rows_f64(s->value, 1, s->T, (long)step, (long)e0, (long)ne, val, st);
  if (!rc && obs) {
    PL_REQUIRE(D > 0, PL_ERR_INVALID, "pl_mg_stamp_step: obs without its width D");
    rc = mg_own_traj(s, D);
    if (!rc) rc = launch_stamp_rows_f32(s->traj_own, (long)D, s->T, (long)step, (long)e0, (long)ne, obs, st);
  }
  s->cols_valid = false;  // complete once pl_mg_stamp_finish has the reward / terminal planes
  s->prio_fresh = false;
  return rc;
}

int pl_mg_stamp_finish(pl_mg* s, const double* rew, const double* term, const double* boot, void* stream) {
  using namespace pl;
  PL_REQUIRE(s && rew && term && boot, PL_ERR_INVALID, "pl_mg_stamp_finish: NULL argument");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = launch_stamp_plane(s->rew, s->N, s->T, rew, st);
  if (!rc) rc = launch_stamp_plane(s->term, s->N, s->T, term, st);
  if (rc) return rc;
  PL_CUDA(cudaMemcpyAsync(s->boot, boot, (size_t)s->N * 8, cudaMemcpyDeviceToDevice, st));
  const long NT = s->N * s->T;
  mg_fill_kernel<<<blocks_for(NT), 256, 0, st>>>(s->ratio, 1.0, NT);
  count_launch();
  PL_LAUNCH("mg_fill_kernel");
  s->cols_valid = true;
  s->prio_fresh = false;
  s->stamped = true;
  return PL_OK;
}

int pl_mg_take_stamped(pl_mg* s, int* stamped) {
  using namespace pl;
  PL_REQUIRE(s && stamped, PL_ERR_INVALID, "pl_mg_take_stamped: NULL argument");
  *stamped = (s->stamped && s->cols_valid) ? 1 : 0;
  s->stamped = false;
  return PL_OK;
}

int pl_mg_chain_stamp(pl_mg* s, size_t N, size_t D, size_t LH) {
  using namespace pl;
  PL_REQUIRE(s != nullptr, PL_ERR_INVALID, "pl_mg_chain_stamp: NULL session");
  s->chain_N = (long)N;
  s->chain_D = N ? (long)D : 0;
  s->chain_LH = N ? (long)LH : 0;
  return PL_OK;
}

int pl_mg_chain_ready(pl_mg* s, size_t N, size_t D, size_t LH, int* ready) {
  using namespace pl;
  PL_REQUIRE(s && ready, PL_ERR_INVALID, "pl_mg_chain_ready: NULL argument");
  *ready = (s->chain_N > 0 && s->chain_N == (long)N && s->chain_D == (long)D && s->chain_LH == (long)LH) ? 1 : 0;
  return PL_OK;
}

int pl_mg_set_obs_dev(pl_mg* s, const float* traj, size_t D) {
  using namespace pl;
  PL_REQUIRE(s && traj && D > 0, PL_ERR_INVALID, "pl_mg_set_obs_dev: bad argument");
  s->traj = traj;
  s->trajD = (long)D;
  return PL_OK;
}

int pl_mg_vtrace(pl_mg* s, double gamma, double lam, double rhoClip, double cClip, double* advL1, void* stream) {
  using namespace pl;
  PL_REQUIRE(s != nullptr, PL_ERR_INVALID, "pl_mg_vtrace: NULL session");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = mg_vtrace_dev(s, gamma, lam, rhoClip, cClip, st);
  if (rc) return rc;
  if (advL1) {
    PL_CUDA(cudaMemcpyAsync(advL1, s->l1, sizeof(double) * s->N, cudaMemcpyDeviceToHost, st));
    PL_CUDA(cudaStreamSynchronize(st));
  }
  return PL_OK;
}

static int mg_vtrace_prio_impl(pl_mg* s, double gamma, double lam, double rhoClip, double cClip, size_t mbSegs,
                               double prioAlpha, double annealBeta, uint64_t rng, bool rng_on_device,
                               cudaStream_t st, bool exact = true) {
  using namespace pl;
  PL_REQUIRE(s != nullptr && mbSegs > 0 && mbSegs < (1u << 30), PL_ERR_INVALID, "pl_mg_vtrace_prio: bad argument");
  int rc = mg_vtrace_dev(s, gamma, lam, rhoClip, cClip, st, exact);
  if (rc) return rc;
  rc = ensure_sample(s, (long)mbSegs);
  if (rc) return rc;
  mg_prio_kernel<<<1, 1024, 0, st>>>(s->l1, s->N, (long)mbSegs, prioAlpha, annealBeta, (unsigned long long)rng,
                                     rng_on_device ? s->rng_dev : nullptr, s->prio_p, s->prio_cum, s->seg, s->mbp);
  count_launch();
  PL_LAUNCH("mg_prio_kernel");
  s->prio_B = (long)mbSegs;
  s->prio_fresh = true;
  return PL_OK;
}

int pl_mg_vtrace_prio(pl_mg* s, double gamma, double lam, double rhoClip, double cClip, size_t mbSegs,
                      double prioAlpha, double annealBeta, uint64_t rng, void* stream) {
  return mg_vtrace_prio_impl(s, gamma, lam, rhoClip, cClip, mbSegs, prioAlpha, annealBeta, rng, false,
                             (cudaStream_t)stream);
}

int pl_mg_grad(pl_mg* s, const pl_mg_net* net, size_t handle, const double* params, const double* segIdx,
               const double* mbPrio, size_t Bmb, double vfCoef, double entCoef, double clipEps, double vfClip,
               uint8_t bf16f, void* stream) {
  using namespace pl;
  PL_REQUIRE(s != nullptr, PL_ERR_INVALID, "pl_mg_grad: NULL session");
  int rc = check_net(net);
  if (rc) return rc;
  PL_REQUIRE((handle != 0) != (params != nullptr), PL_ERR_INVALID,
             "pl_mg_grad: pass exactly one of a policy handle and host params");
  PL_REQUIRE((segIdx == nullptr) == (mbPrio == nullptr), PL_ERR_INVALID,
             "pl_mg_grad: segIdx and mbPrio are both host arrays or both NULL (the resident sample)");
  PL_REQUIRE(Bmb > 0 && Bmb < (1u << 24), PL_ERR_INVALID, "pl_mg_grad: bad minibatch size %zu", Bmb);
  PL_REQUIRE(s->cols_valid, PL_ERR_INVALID, "pl_mg_grad: no columns (call pl_mg_set_columns first)");
  rc = check_heads(s, net);
  if (rc) return rc;
  PL_REQUIRE(s->traj && s->trajD == (long)net->D, PL_ERR_INVALID,
             "pl_mg_grad: no obs trajectory of width D=%zu (call pl_mg_set_obs first)", net->D);
  if (!segIdx)
    PL_REQUIRE(s->prio_fresh && s->prio_B == (long)Bmb, PL_ERR_INVALID,
               "pl_mg_grad: no resident sample of %zu segments (call pl_mg_vtrace_prio first)", Bmb);
  cudaStream_t st = (cudaStream_t)stream;
  const MgShape sh = shape_of(net);
  const uint64_t l0 = pl_kernel_launch_count();
  rc = ensure_work(s, sh, (long)Bmb, s->T, bf16f != 0);
  if (rc) return rc;
  rc = ensure_sample(s, (long)Bmb);
  if (rc) return rc;
  auto& w = s->w;
  if (segIdx) {
    PL_CUDA(cudaMemcpyAsync(s->seg, segIdx, sizeof(double) * Bmb, cudaMemcpyHostToDevice, st));
    PL_CUDA(cudaMemcpyAsync(s->mbp, mbPrio, sizeof(double) * Bmb, cudaMemcpyHostToDevice, st));
  }
  s->prio_fresh = false;
  // weights
  if (params) {
    PL_CUDA(cudaMemcpyAsync(w.params_in, params, sizeof(double) * sh.P(), cudaMemcpyHostToDevice, st));
    rc = refresh_shadows(s, w.params_in, st);
    s->shadow_src = 0;
  } else if (s->shadow_src != handle) {
    rc = refresh_shadows(s, (const double*)handle, st);
    s->shadow_src = handle;
  }
  if (rc) return rc;
  // gather
  const int Bi = (int)Bmb, T = (int)s->T;
  if (s->world > 1) {
    // the advantage statistics are those of the all-rank minibatch
    const double nall = (double)w.R * s->world;
    for (int sq = 0; sq < 2; sq++) {
      mg_adv_ms_kernel<<<kAdvBlocks, 256, 0, st>>>(s->adv, s->seg, Bi, T, sq, w.ms, w.adv_part, w.adv_counter, 1);
      count_launch();
      PL_LAUNCH("mg_adv_ms_kernel");
      rc = comm_allreduce_f64(s->comm, w.ms + 2 + sq, 1, st);
      if (rc) return rc;
      mg_adv_final_kernel<<<1, 32, 0, st>>>(w.ms, nall, sq);
      count_launch();
      PL_LAUNCH("mg_adv_final_kernel");
    }
  } else {
    mg_adv_ms_kernel<<<kAdvBlocks, 256, 0, st>>>(s->adv, s->seg, Bi, T, 0, w.ms, w.adv_part, w.adv_counter, 0);
    mg_adv_ms_kernel<<<kAdvBlocks, 256, 0, st>>>(s->adv, s->seg, Bi, T, 1, w.ms, w.adv_part, w.adv_counter, 0);
    count_launch();
  }
  mg_gather_scal_kernel<<<blocks_for(w.R), 256, 0, st>>>(s->act, s->logp, s->term, s->adv, s->value, s->seg, s->mbp,
                                                         w.ms, Bi, T, s->W, w.act_i, w.adv_f, w.ret_f, w.olp_f,
                                                         w.ov_f, w.term_f);
  if (w.fast)
    mg_gather_obs_kernel<__nv_bfloat16><<<blocks_for(w.R * w.Dp), 256, 0, st>>>(s->traj, s->seg, Bi, T, (int)sh.D,
                                                                               (int)w.Dp, (__nv_bfloat16*)w.X);
  else
    mg_gather_obs_kernel<float><<<blocks_for(w.R * w.Dp), 256, 0, st>>>(s->traj, s->seg, Bi, T, (int)sh.D, (int)w.Dp,
                                                                        (float*)w.X);
  count_launch(3);
  PL_LAUNCH("mg_gather_kernels");
  const bool losses = loss_channel_on();
  rc = run_bptt(s, vfCoef, entCoef, clipEps, vfClip, losses, st);
  if (rc) return rc;
  // data parallel: the summed gradient of the all-rank minibatch on every rank
  if (s->world > 1) {
    rc = comm_allreduce_f32(s->comm, w.grad, (size_t)sh.P(), st);
    if (rc) return rc;
  }
  // replay iterate
  PL_CUDA(cudaMemsetAsync(s->lastw, 0xFF, sizeof(int) * s->N, st));
  mg_lastw_kernel<<<(unsigned)((Bi + 255) / 256), 256, 0, st>>>(s->lastw, s->seg, Bi);
  mg_iterate_kernel<<<blocks_for(w.R), 256, 0, st>>>(s->value, s->ratio, s->logp, w.newlp, w.newval, s->seg, s->lastw,
                                                     Bi, T);
  count_launch(2);
  PL_LAUNCH("mg_iterate_kernel");
  if (losses) {
    double lo[7];
    rc = reduce_losses(s, vfCoef, entCoef, lo, st);
    if (rc) return rc;
    loss_channel_store(lo);
  }
  s->grad_fresh = true;
  s->grad_rows = w.R;
  s->launches = pl_kernel_launch_count() - l0;
  return PL_OK;
}

int pl_mg_grad_download(pl_mg* s, double* grad, double* newlp, double* newval) {
  using namespace pl;
  PL_REQUIRE(s && s->have_work, PL_ERR_INVALID, "pl_mg_grad_download: no gradient");
  auto& w = s->w;
  const long P = w.sh.P();
  PL_CUDA(cudaDeviceSynchronize());
  if (grad) {
    std::vector<float> g((size_t)P);
    PL_CUDA(cudaMemcpy(g.data(), w.grad, sizeof(float) * P, cudaMemcpyDeviceToHost));
    for (long i = 0; i < P; i++) grad[i] = (double)g[i];
  }
  std::vector<float> t((size_t)w.R);
  if (newlp) {
    PL_CUDA(cudaMemcpy(t.data(), w.newlp, sizeof(float) * w.R, cudaMemcpyDeviceToHost));
    for (long i = 0; i < w.R; i++) newlp[i] = (double)t[i];
  }
  if (newval) {
    PL_CUDA(cudaMemcpy(t.data(), w.newval, sizeof(float) * w.R, cudaMemcpyDeviceToHost));
    for (long i = 0; i < w.R; i++) newval[i] = (double)t[i];
  }
  return device_error_check();
}

int pl_mg_muon(pl_mg* s, const pl_mg_net* net, size_t handle, const double* gClip, double lr, double wd, double mu,
               double eps, double maxGradNorm, double gscale, const double* coeffs, size_t iters, uint8_t bf16f,
               void* stream) {
  using namespace pl;
  PL_REQUIRE(s != nullptr && handle != 0, PL_ERR_INVALID, "pl_mg_muon: NULL session or handle");
  int rc = check_net(net);
  if (rc) return rc;
  if (!coeffs) {
    coeffs = &kMuonCoeffs[0][0];
    iters = 5;
  }
  PL_REQUIRE(iters > 0 && iters <= 64, PL_ERR_INVALID, "pl_mg_muon: 1..64 Newton-Schulz steps");
  const MgShape sh = shape_of(net);
  const long Bmb = s->have_work ? s->w.Bmb : 1;
  if (!(s->have_work && s->w.sh == sh && s->w.fast == (bf16f != 0))) {
    PL_REQUIRE(gClip != nullptr, PL_ERR_INVALID,
               "pl_mg_muon: no resident gradient for this network and tier (call pl_mg_grad first)");
    rc = ensure_work(s, sh, Bmb, s->T, bf16f != 0);
    if (rc) return rc;
  }
  const uint64_t l0 = pl_kernel_launch_count();
  rc = muon_step(s, handle, gClip, lr, wd, mu, eps, maxGradNorm, gscale, coeffs, (int)iters, (cudaStream_t)stream);
  s->launches += pl_kernel_launch_count() - l0;
  return rc;
}

int pl_mg_read_state(pl_mg* s, double* value, double* ratio, double* adv) {
  using namespace pl;
  PL_REQUIRE(s != nullptr, PL_ERR_INVALID, "pl_mg_read_state: NULL session");
  const size_t NT = (size_t)s->N * s->T;
  PL_CUDA(cudaDeviceSynchronize());
  if (value) PL_CUDA(cudaMemcpy(value, s->value, NT * 8, cudaMemcpyDeviceToHost));
  if (ratio) PL_CUDA(cudaMemcpy(ratio, s->ratio, NT * 8, cudaMemcpyDeviceToHost));
  if (adv) PL_CUDA(cudaMemcpy(adv, s->adv, NT * 8, cudaMemcpyDeviceToHost));
  return device_error_check();
}

static int mg_minibatch(pl_mg* s, const pl_mg_net* net, size_t handle, const pl_mg_hyper* h, size_t mbSegs,
                        uint64_t rng, bool rng_on_device, double lr, cudaStream_t st) {
  const double gscale = 1.0 / ((double)mbSegs * (double)s->T * (double)s->world);
  int rc = mg_vtrace_prio_impl(s, h->gamma, h->lam, h->rhoClip, h->cClip, mbSegs, h->prioAlpha, h->annealBeta, rng,
                               rng_on_device, st, /*exact=*/h->bf16 == 0);
  if (rc) return rc;
  rc = pl_mg_grad(s, net, handle, nullptr, nullptr, nullptr, mbSegs, h->vfCoef, h->entCoef, h->clipEps, h->vfClip,
                  h->bf16, st);
  if (rc) return rc;
  return pl_mg_muon(s, net, handle, nullptr, lr, h->wd, h->mu, h->eps, h->maxGradNorm, gscale, h->ns_coeffs,
                    h->ns_coeffs ? h->ns_iters : 5, h->bf16, st);
}

// The fast tier runs the first minibatch of the update eagerly (which also performs every one-time
// set-up outside any capture) and replays a captured graph of the same minibatch for the other
// numMB - 1: the sampler's generator state advances in device memory, every other argument of the
// chain is fixed for the update. The graph is captured again when the network, handle,
// hyperparameters, minibatch size or lr change.
static int mg_update_graph(pl_mg* s, const pl_mg_net* net, size_t handle, const pl_mg_hyper* h, size_t numMB,
                           size_t mbSegs, uint64_t* rng, double lr, cudaStream_t st) {
  using namespace pl;
  std::vector<double> key = {(double)net->D, (double)net->H, (double)net->L, (double)net->A, (double)net->K,
                             (double)net->enc_act, (double)handle, h->gamma, h->lam, h->rhoClip, h->cClip,
                             h->prioAlpha, h->annealBeta, h->wd, h->mu, h->eps, h->vfCoef, h->entCoef, h->clipEps,
                             h->vfClip, h->maxGradNorm, (double)mbSegs, lr, (double)h->ns_iters, (double)s->W};
  for (int v : s->hs) key.push_back((double)v);
  if (h->ns_coeffs)
    for (size_t i = 0; i < 3 * h->ns_iters; i++) key.push_back(h->ns_coeffs[i]);
  // everything that allocates or reads back happens before the capture
  const MgShape sh = shape_of(net);
  int rc = ensure_work(s, sh, (long)mbSegs, s->T, true);
  if (!rc) rc = ensure_sample(s, (long)mbSegs);
  if (rc) return rc;
  if (s->shadow_src != handle) {
    rc = refresh_shadows(s, (const double*)handle, st);
    if (rc) return rc;
    s->shadow_src = handle;
  }
  PL_CUDA(cudaMemcpyAsync(s->rng_dev, rng, sizeof(uint64_t), cudaMemcpyHostToDevice, st));
  rc = mg_minibatch(s, net, handle, h, mbSegs, 0, true, lr, st);
  if (rc) return rc;
  if (!s->gexec || key != s->gkey) {
    if (s->gexec) {
      cudaGraphExecDestroy(s->gexec);
      s->gexec = nullptr;
    }
    if (!s->cap) PL_CUDA(cudaStreamCreateWithFlags(&s->cap, cudaStreamNonBlocking));
    const uint64_t c0 = pl_kernel_launch_count();
    PL_CUDA(cudaStreamBeginCapture(s->cap, cudaStreamCaptureModeThreadLocal));
    rc = mg_minibatch(s, net, handle, h, mbSegs, 0, true, lr, s->cap);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(s->cap, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return check_cuda(e, "cudaStreamEndCapture (MinGRU minibatch)");
    const cudaError_t e2 = cudaGraphInstantiate(&s->gexec, g, 0);
    cudaGraphDestroy(g);
    if (e2 != cudaSuccess) {
      s->gexec = nullptr;
      return check_cuda(e2, "cudaGraphInstantiate (MinGRU minibatch)");
    }
    s->gkey = key;
    s->gnodes = pl_kernel_launch_count() - c0;
  }
  for (size_t mb = 1; mb < numMB; mb++) {
    PL_CUDA(cudaGraphLaunch(s->gexec, st));
    count_launch(s->gnodes);
  }
  *rng += (uint64_t)numMB * (uint64_t)mbSegs * 0x9E3779B97F4A7C15ULL;
  s->prio_fresh = false;
  s->grad_fresh = false;
  s->shadow_src = handle;
  return PL_OK;
}

int pl_mg_update(pl_mg* s, const pl_mg_net* net, size_t handle, const pl_mg_hyper* h, size_t numMB, size_t mbSegs,
                 uint64_t* rng, double lr, void* stream) {
  using namespace pl;
  PL_REQUIRE(s && net && h && rng && handle, PL_ERR_INVALID, "pl_mg_update: NULL argument");
  PL_REQUIRE(!s->comm || pl_comm_aborted(s->comm) == 0, PL_ERR_COMM,
             "pl_mg_update: the communicator was aborted (or is not one of this library)");
  int rc = check_net(net);
  if (!rc) rc = check_heads(s, net);
  if (rc) return rc;
  PL_REQUIRE(mbSegs > 0 && mbSegs < (1u << 24), PL_ERR_INVALID, "pl_mg_update: bad minibatch size %zu", mbSegs);
  PL_REQUIRE(s->cols_valid && s->traj && s->trajD == (long)net->D, PL_ERR_INVALID,
             "pl_mg_update: set the columns and the obs trajectory first");
  const uint64_t l0 = pl_kernel_launch_count();
  if (h->bf16 && !loss_channel_on() && numMB > 1) {  // data parallel too: the collectives are captured
    rc = mg_update_graph(s, net, handle, h, numMB, mbSegs, rng, lr, (cudaStream_t)stream);
    s->launches = pl_kernel_launch_count() - l0;
    return rc;
  }
  for (size_t mb = 0; mb < numMB; mb++) {
    rc = mg_minibatch(s, net, handle, h, mbSegs, *rng, false, lr, (cudaStream_t)stream);
    if (rc) return rc;
    *rng += (uint64_t)mbSegs * 0x9E3779B97F4A7C15ULL;
  }
  s->launches = pl_kernel_launch_count() - l0;
  return PL_OK;
}

uint64_t pl_mg_last_launches(const pl_mg* s) { return s ? s->launches : 0; }

// Host-mode gradient: one cached session per device carries the workspace between calls.
int pl_mingru_ppo_grad(const double* params, const double* obs, const double* scal, size_t B, size_t T,
                       const pl_mg_net* net, double vfCoef, double entCoef, double clipEps, double vfClip,
                       uint8_t bf16f, double* out) {
  return pl_mingru_ppo_grad_md(params, obs, scal, B, T, net, 1, nullptr, vfCoef, entCoef, clipEps, vfClip, bf16f, out);
}

int pl_mingru_ppo_grad_md(const double* params, const double* obs, const double* scal, size_t B, size_t T,
                          const pl_mg_net* net, size_t W, const double* head_sizes, double vfCoef, double entCoef,
                          double clipEps, double vfClip, uint8_t bf16f, double* out) {
  using namespace pl;
  PL_REQUIRE(W >= 1 && (W == 1 || head_sizes), PL_ERR_INVALID, "pl_mingru_ppo_grad_md: %zu heads need their sizes",
             W);
  int rc = check_net(net);
  if (rc) return rc;
  PL_REQUIRE(params && obs && scal && out, PL_ERR_INVALID, "pl_mingru_ppo_grad: NULL argument");
  PL_REQUIRE(B > 0 && T > 0 && B * T < (1u << 28), PL_ERR_INVALID, "pl_mingru_ppo_grad: bad extents B=%zu T=%zu", B,
             T);
  rc = require_device();
  if (rc) return rc;
  static std::mutex mu;
  static pl_mg* cache[64] = {nullptr};
  std::lock_guard<std::mutex> g(mu);
  int dev = 0;
  PL_CUDA(cudaGetDevice(&dev));
  PL_REQUIRE(dev >= 0 && dev < 64, PL_ERR_UNSUPPORTED, "device index out of range");
  if (!cache[dev] || cache[dev]->T != (long)T || cache[dev]->N != (long)B) {
    if (cache[dev]) pl_mg_destroy(cache[dev]);
    cache[dev] = nullptr;
    rc = pl_mg_create(B, T, &cache[dev]);
    if (rc) return rc;
  }
  pl_mg* s = cache[dev];
  rc = pl_mg_set_heads(s, W, W > 1 ? head_sizes : nullptr);
  if (!rc) rc = check_heads(s, net);
  if (rc) return rc;
  const MgShape sh = shape_of(net);
  rc = ensure_work(s, sh, (long)B, (long)T, bf16f != 0);
  if (rc) return rc;
  auto& w = s->w;
  const long R = w.R, P = sh.P();
  double* obs_d = (double*)scratch(21, sizeof(double) * R * sh.D);
  double* scal_d = (double*)scratch(22, sizeof(double) * (W + 5) * R);
  if (!obs_d || !scal_d) return PL_ERR_NOMEM;
  PL_CUDA(cudaMemcpy(obs_d, obs, sizeof(double) * R * sh.D, cudaMemcpyHostToDevice));
  PL_CUDA(cudaMemcpy(scal_d, scal, sizeof(double) * (W + 5) * R, cudaMemcpyHostToDevice));
  PL_CUDA(cudaMemcpy(w.params_in, params, sizeof(double) * P, cudaMemcpyHostToDevice));
  rc = refresh_shadows(s, w.params_in, 0);
  if (rc) return rc;
  s->shadow_src = 0;
  if (w.fast)
    mg_obs_rows_kernel<__nv_bfloat16><<<blocks_for(R * w.Dp), 256>>>(obs_d, R, (int)sh.D, (int)w.Dp,
                                                                     (__nv_bfloat16*)w.X);
  else
    mg_obs_rows_kernel<float><<<blocks_for(R * w.Dp), 256>>>(obs_d, R, (int)sh.D, (int)w.Dp, (float*)w.X);
  mg_scal_rows_kernel<<<blocks_for(R), 256>>>(scal_d, R, (int)W, w.act_i, w.adv_f, w.ret_f, w.olp_f, w.ov_f,
                                              w.term_f);
  count_launch(2);
  PL_LAUNCH("mg_host_rows");
  rc = run_bptt(s, vfCoef, entCoef, clipEps, vfClip, false, 0);
  if (rc) return rc;
  s->grad_fresh = true;
  rc = pl_mg_grad_download(s, out, out + P, out + P + R);
  return rc;
}

}  // extern "C"
