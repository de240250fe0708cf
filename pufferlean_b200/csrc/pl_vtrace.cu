// Advantage scans over B segments x T steps (row-major, row b holds segment b's horizon).
//
//  * exact tier (f64): the reference's sequential backward scan with its IEEE op order, every
//    product and sum rounded on its own (__dmul_rn / __dadd_rn, no fused multiply-add), so the
//    result is bit-identical to ffi/puffercuda.cu:69-90 (vector form) and :146-167 (MinGRU form).
//  * fast tier (fp32, and an f64 form for the recurrent update's bf16 tier): one warp per segment.
//    Each lane owns a contiguous run of T/32 steps, loaded with vector loads; the recurrence
//    A_t = delta_t + k_t * A_{t+1} is a composition of affine maps, so each lane folds its run into
//    one map (k, delta), a 5-step shuffle suffix scan composes the maps of the lanes to its right,
//    and the lane then replays its run backwards from the scanned boundary value. sum_t |A_t| per
//    segment falls out of the same registers.
#include "pl_common.cuh"
#include "pl_runtime.h"

namespace pl {

// ---------------------------------------------------------------- exact f64
template <bool MINGRU>
__global__ void vtrace_f64_kernel(const double* __restrict__ rew, const double* __restrict__ val,
                                  const double* __restrict__ term, const double* __restrict__ imp,
                                  const double* __restrict__ bootv, double* __restrict__ adv,
                                  double* __restrict__ adv_l1, int B, int T, double gamma, double lam,
                                  double rhoClip, double cClip) {
  const int seg = blockIdx.x * blockDim.x + threadIdx.x;
  if (seg >= B) return;
  const long off = (long)seg * T;
  const double* reward = rew + off;
  const double* value = val + off;
  const double* done = term + off;
  const double* ratio = imp + off;
  double* out = adv + off;
  const double gamma_lambda = __dmul_rn(gamma, lam);
  double carry = 0.0;  // A[t+1] of the backward recurrence
  if (!MINGRU) {
    if (T > 0) out[T - 1] = 0.0;
    for (int t = T - 2; t >= 0; t--) {
      const double alive = (done[t] != 0.0) ? 0.0 : 1.0;
      const double w = ratio[t];
      const double rho_t = w < rhoClip ? w : rhoClip;
      const double c_t = w < cClip ? w : cClip;
      const double r_raw = reward[t];
      const double r_t = r_raw > 1.0 ? 1.0 : (r_raw < -1.0 ? -1.0 : r_raw);  // NaN passes through
      // rho * (r + gamma*V[t+1]*alive - V[t])
      const double td =
          __dmul_rn(rho_t, __dsub_rn(__dadd_rn(r_t, __dmul_rn(__dmul_rn(gamma, value[t + 1]), alive)), value[t]));
      // td + gamma*lambda*c*A[t+1]*alive
      carry = __dadd_rn(td, __dmul_rn(__dmul_rn(__dmul_rn(gamma_lambda, c_t), carry), alive));
      out[t] = carry;
    }
  } else {
    for (int t = T - 1; t >= 0; t--) {
      const double alive = (done[t] > 0.5) ? 0.0 : 1.0;
      const double v_next = (t + 1 < T) ? value[t + 1] : bootv[seg];
      const double w = ratio[t];
      const double rho_t = w < rhoClip ? w : rhoClip;
      const double c_t = w < cClip ? w : cClip;
      const double r_raw = reward[t];
      const double r_t = r_raw > 1.0 ? 1.0 : (r_raw < -1.0 ? -1.0 : r_raw);  // NaN passes through
      // rho*r + gamma*v_next*alive - V[t]
      const double td = __dsub_rn(__dadd_rn(__dmul_rn(rho_t, r_t), __dmul_rn(__dmul_rn(gamma, v_next), alive)), value[t]);
      carry = __dadd_rn(td, __dmul_rn(__dmul_rn(__dmul_rn(gamma_lambda, c_t), carry), alive));
      out[t] = carry;
    }
  }
  if (adv_l1) {
    double s = 0.0;
    for (int t = 0; t < T; t++) s = __dadd_rn(s, fabs(out[t]));
    adv_l1[seg] = s;
  }
}

// ---------------------------------------------------------------- warp-per-segment scan (fp32 / f64)
template <int EPL, typename F>
__device__ __forceinline__ void load_run(const F* __restrict__ p, int t0, int T, bool vec, F (&x)[EPL], F fill) {
  if (vec && t0 + EPL <= T) {
    if constexpr (sizeof(F) == 4 && EPL == 2) {
      const float2 q = *reinterpret_cast<const float2*>(p + t0);
      x[0] = q.x;
      x[1] = q.y;
      return;
    } else if constexpr (sizeof(F) == 4 && EPL % 4 == 0) {
#pragma unroll
      for (int i = 0; i < EPL; i += 4) {
        const float4 q = *reinterpret_cast<const float4*>(p + t0 + i);
        x[i] = q.x;
        x[i + 1] = q.y;
        x[i + 2] = q.z;
        x[i + 3] = q.w;
      }
      return;
    } else if constexpr (sizeof(F) == 8 && EPL % 2 == 0) {
#pragma unroll
      for (int i = 0; i < EPL; i += 2) {
        const double2 q = *reinterpret_cast<const double2*>(p + t0 + i);
        x[i] = q.x;
        x[i + 1] = q.y;
      }
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < EPL; e++) x[e] = (t0 + e < T) ? p[t0 + e] : fill;
}
template <int EPL, typename F>
__device__ __forceinline__ void store_run(F* __restrict__ p, int t0, int T, bool vec, const F (&x)[EPL]) {
  if (vec && t0 + EPL <= T) {
    if constexpr (sizeof(F) == 4 && EPL == 2) {
      *reinterpret_cast<float2*>(p + t0) = make_float2(x[0], x[1]);
      return;
    } else if constexpr (sizeof(F) == 4 && EPL % 4 == 0) {
#pragma unroll
      for (int i = 0; i < EPL; i += 4)
        *reinterpret_cast<float4*>(p + t0 + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
      return;
    } else if constexpr (sizeof(F) == 8 && EPL % 2 == 0) {
#pragma unroll
      for (int i = 0; i < EPL; i += 2) *reinterpret_cast<double2*>(p + t0 + i) = make_double2(x[i], x[i + 1]);
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < EPL; e++)
    if (t0 + e < T) p[t0 + e] = x[e];
}

// Programmatic dependent launch: a scan may be launched before the kernel ahead of it in the stream has
// finished (its launch and set-up overlap that kernel's tail); it waits for that kernel's results
// before its first load and lets the next one start once its loads are done. Both are no-ops for a
// plain launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// One warp per segment; lane l owns steps [l EPL, (l + 1) EPL) of the horizon. The backward recurrence
// A_t = delta_t + k_t A_{t+1} is a chain of affine maps: each lane folds its run into one map, a 5-step
// shuffle suffix scan composes the maps to its right, and the lane replays its run from the scanned
// boundary value. Not the reference's sequential operation order (the f64 form agrees with it to
// rounding, about 1e-15 relative; the exact tier is vtrace_f64_kernel).
template <typename F, int EPL, bool MINGRU>
__global__ void __launch_bounds__(256) vtrace_warp_kernel(const F* __restrict__ rew, const F* __restrict__ val,
                                                          const F* __restrict__ term, const F* __restrict__ imp,
                                                          const F* __restrict__ bootv, F* __restrict__ adv,
                                                          F* __restrict__ adv_l1, int B, int T, F gamma, F lam,
                                                          F rhoClip, F cClip) {
  const int lane = threadIdx.x & 31;
  const long seg = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_wait();
  if (seg >= B) {  // warp-uniform
    pdl_release();
    return;
  }
  const long base = seg * T;
  const int t0 = lane * EPL;
  // vector loads need every row start aligned to the run width
  constexpr uintptr_t ALIGN = EPL * sizeof(F) >= 16 ? 16 : EPL * sizeof(F);
  const uintptr_t orp = (uintptr_t)(rew + base) | (uintptr_t)(val + base) | (uintptr_t)(term + base) |
                        (imp ? (uintptr_t)(imp + base) : 0) | (uintptr_t)(adv + base);
  const bool vec = EPL > 1 && (T % EPL) == 0 && (orp % ALIGN) == 0;
  F r[EPL], v[EPL], d[EPL], im[EPL];
  load_run<EPL, F>(rew + base, t0, T, vec, r, F(0));
  load_run<EPL, F>(val + base, t0, T, vec, v, F(0));
  load_run<EPL, F>(term + base, t0, T, vec, d, F(0));
  if (imp)
    load_run<EPL, F>(imp + base, t0, T, vec, im, F(1));
  else {
#pragma unroll
    for (int e = 0; e < EPL; e++) im[e] = F(1);  // no importance ratios: rho = c = min(1, clip)
  }
  const F boot = MINGRU ? bootv[seg] : F(0);
  pdl_release();
  // value one step past this lane's run: the first value of the next lane (or the bootstrap)
  const F v_after = __shfl_down_sync(0xffffffffu, v[0], 1);
  const F gl = gamma * lam;
  F k[EPL], dl[EPL];
#pragma unroll
  for (int e = 0; e < EPL; e++) {
    const int t = t0 + e;
    const F vn = (e + 1 < EPL) ? v[e + 1] : v_after;
    const F rc = r[e] > F(1) ? F(1) : (r[e] < F(-1) ? F(-1) : r[e]);
    const F rho = im[e] < rhoClip ? im[e] : rhoClip;
    const F c = im[e] < cClip ? im[e] : cClip;
    if (t >= T) {  // past the horizon: identity map
      k[e] = F(1);
      dl[e] = F(0);
    } else if (!MINGRU) {
      const F nnt = (d[e] != F(0)) ? F(0) : F(1);
      if (t == T - 1) {  // A[T-1] = 0
        k[e] = F(0);
        dl[e] = F(0);
      } else {
        dl[e] = rho * (rc + gamma * vn * nnt - v[e]);
        k[e] = gl * c * nnt;
      }
    } else {
      const F nnt = (d[e] > F(0.5)) ? F(0) : F(1);
      const F vnx = (t == T - 1) ? boot : vn;
      dl[e] = rho * rc + gamma * vnx * nnt - v[e];
      k[e] = (t == T - 1) ? F(0) : gl * c * nnt;  // A_T enters as 0
    }
  }
  // fold this lane's run into one affine map F(x) = KK*x + DD (applied to A at the run's end)
  F KK = F(1), DD = F(0);
#pragma unroll
  for (int e = EPL - 1; e >= 0; e--) {
    DD = dl[e] + k[e] * DD;
    KK = k[e] * KK;
  }
  // inclusive suffix scan of maps over lanes: lane l -> F_l o F_{l+1} o ... o F_31
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const F K2 = __shfl_down_sync(0xffffffffu, KK, off);
    const F D2 = __shfl_down_sync(0xffffffffu, DD, off);
    if (lane + off < 32) {
      DD = DD + KK * D2;
      KK = KK * K2;
    }
  }
  F A = __shfl_down_sync(0xffffffffu, DD, 1);  // value entering this run from the right
  if (lane == 31) A = F(0);
  F out[EPL];
  F l1 = F(0);
#pragma unroll
  for (int e = EPL - 1; e >= 0; e--) {
    A = dl[e] + k[e] * A;
    out[e] = A;
    if (t0 + e < T) l1 += A < F(0) ? -A : A;
  }
  store_run<EPL, F>(adv + base, t0, T, vec, out);
  if (adv_l1) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    if (lane == 0) adv_l1[seg] = l1;
  }
}

// Launch of the warp scan with programmatic stream serialisation allowed (see pdl_wait).
template <typename F, int EPL, bool MINGRU>
static cudaError_t launch_warp(dim3 grid, dim3 block, cudaStream_t st, const F* rew, const F* val, const F* term,
                               const F* imp, const F* bootv, F* adv, F* l1, int B, int T, F g, F l, F rho, F c) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, vtrace_warp_kernel<F, EPL, MINGRU>, rew, val, term, imp, bootv, adv, l1, B, T, g, l,
                            rho, c);
}

template <typename F, bool MINGRU>
static int launch_scan(const F* rew, const F* val, const F* term, const F* imp, const F* bootv, int B, int T, F g,
                       F l, F rho, F c, F* adv, F* l1, cudaStream_t st) {
  const int warps = 8;
  dim3 grid((unsigned)ceil_div(B, warps)), block(32 * warps);
  cudaError_t e;
  if (T <= 32)
    e = launch_warp<F, 1, MINGRU>(grid, block, st, rew, val, term, imp, bootv, adv, l1, B, T, g, l, rho, c);
  else if (T <= 64)
    e = launch_warp<F, 2, MINGRU>(grid, block, st, rew, val, term, imp, bootv, adv, l1, B, T, g, l, rho, c);
  else if (T <= 128)
    e = launch_warp<F, 4, MINGRU>(grid, block, st, rew, val, term, imp, bootv, adv, l1, B, T, g, l, rho, c);
  else if (T <= 256)
    e = launch_warp<F, 8, MINGRU>(grid, block, st, rew, val, term, imp, bootv, adv, l1, B, T, g, l, rho, c);
  else
    return set_error(PL_ERR_UNSUPPORTED, "the V-trace scan supports horizons up to 256 (T=%d)", T);
  if (e != cudaSuccess) return check_cuda(e, "vtrace_warp_kernel launch");
  count_launch();
  PL_LAUNCH("vtrace_warp_kernel");
  return PL_OK;
}

int vtrace_f64_launch(const double* rew, const double* val, const double* term, const double* imp,
                      const double* bootv, int B, int T, double g, double l, double rho, double c, double* adv,
                      double* l1, cudaStream_t st) {
  dim3 grid((unsigned)ceil_div(B, 128)), block(128);
  if (bootv)
    vtrace_f64_kernel<true><<<grid, block, 0, st>>>(rew, val, term, imp, bootv, adv, l1, B, T, g, l, rho, c);
  else
    vtrace_f64_kernel<false><<<grid, block, 0, st>>>(rew, val, term, imp, bootv, adv, l1, B, T, g, l, rho, c);
  count_launch();
  PL_LAUNCH("vtrace_f64_kernel");
  return PL_OK;
}

int vtrace_f32_launch(const float* rew, const float* val, const float* term, const float* imp, const float* bootv,
                      int B, int T, double g, double l, double rho, double c, float* adv, float* l1,
                      cudaStream_t st) {
  if (bootv)
    return launch_scan<float, true>(rew, val, term, imp, bootv, B, T, (float)g, (float)l, (float)rho, (float)c, adv,
                                    l1, st);
  return launch_scan<float, false>(rew, val, term, imp, bootv, B, T, (float)g, (float)l, (float)rho, (float)c, adv,
                                   l1, st);
}

int vtrace_f64_scan_launch(const double* rew, const double* val, const double* term, const double* imp,
                           const double* bootv, int B, int T, double g, double l, double rho, double c, double* adv,
                           double* l1, cudaStream_t st) {
  if (bootv) return launch_scan<double, true>(rew, val, term, imp, bootv, B, T, g, l, rho, c, adv, l1, st);
  return launch_scan<double, false>(rew, val, term, imp, bootv, B, T, g, l, rho, c, adv, l1, st);
}

static int vtrace_host(const double* rew, const double* val, const double* term, const double* imp,
                       const double* bootv, size_t B, size_t T, double g, double l, double rho, double c,
                       double* adv) {
  int rc = require_device();
  if (rc) return rc;
  PL_REQUIRE(rew && val && term && imp && adv, PL_ERR_INVALID, "V-trace: NULL buffer");
  const size_t n = B * T;
  if (n == 0) return PL_OK;
  double* d = (double*)scratch(0, sizeof(double) * (5 * n + B));
  if (!d) return PL_ERR_NOMEM;
  double *dR = d, *dV = d + n, *dT = d + 2 * n, *dI = d + 3 * n, *dA = d + 4 * n, *dB = d + 5 * n;
  PL_CUDA(cudaMemcpy(dR, rew, 8 * n, cudaMemcpyHostToDevice));
  PL_CUDA(cudaMemcpy(dV, val, 8 * n, cudaMemcpyHostToDevice));
  PL_CUDA(cudaMemcpy(dT, term, 8 * n, cudaMemcpyHostToDevice));
  PL_CUDA(cudaMemcpy(dI, imp, 8 * n, cudaMemcpyHostToDevice));
  if (bootv) PL_CUDA(cudaMemcpy(dB, bootv, 8 * B, cudaMemcpyHostToDevice));
  rc = vtrace_f64_launch(dR, dV, dT, dI, bootv ? dB : nullptr, (int)B, (int)T, g, l, rho, c, dA, nullptr, 0);
  if (rc) return rc;
  PL_CUDA(cudaMemcpy(adv, dA, 8 * n, cudaMemcpyDeviceToHost));
  return PL_OK;
}

}  // namespace pl

extern "C" {

int pl_vtrace(const double* rew, const double* val, const double* term, const double* imp, size_t B, size_t T,
              double gamma, double lam, double rhoClip, double cClip, double* adv) {
  return pl::vtrace_host(rew, val, term, imp, nullptr, B, T, gamma, lam, rhoClip, cClip, adv);
}

int pl_vtrace_mingru(const double* rew, const double* val, const double* term, const double* imp,
                     const double* bootv, size_t B, size_t T, double gamma, double lam, double rhoClip, double cClip,
                     double* adv) {
  PL_REQUIRE(bootv || B * T == 0, PL_ERR_INVALID, "V-trace MinGRU form needs bootv");
  return pl::vtrace_host(rew, val, term, imp, bootv, B, T, gamma, lam, rhoClip, cClip, adv);
}

int pl_vtrace_f32_dev(const float* rew, const float* val, const float* term, const float* imp, const float* bootv,
                      size_t B, size_t T, double gamma, double lam, double rhoClip, double cClip, float* adv,
                      float* adv_l1, void* stream) {
  if (B * T == 0) return PL_OK;
  PL_REQUIRE(B < (1u << 31) && T < (1u << 31), PL_ERR_INVALID, "V-trace extents too large");
  return pl::vtrace_f32_launch(rew, val, term, imp, bootv, (int)B, (int)T, gamma, lam, rhoClip, cClip, adv, adv_l1,
                               (cudaStream_t)stream);
}

int pl_vtrace_f64_scan_dev(const double* rew, const double* val, const double* term, const double* imp,
                           const double* bootv, size_t B, size_t T, double gamma, double lam, double rhoClip,
                           double cClip, double* adv, double* adv_l1, void* stream) {
  if (B * T == 0) return PL_OK;
  PL_REQUIRE(B < (1u << 31) && T < (1u << 31), PL_ERR_INVALID, "V-trace extents too large");
  return pl::vtrace_f64_scan_launch(rew, val, term, imp, bootv, (int)B, (int)T, gamma, lam, rhoClip, cClip, adv,
                                    adv_l1, (cudaStream_t)stream);
}

int pl_vtrace_f64_dev(const double* rew, const double* val, const double* term, const double* imp,
                      const double* bootv, size_t B, size_t T, double gamma, double lam, double rhoClip,
                      double cClip, double* adv, double* adv_l1, void* stream) {
  if (B * T == 0) return PL_OK;
  PL_REQUIRE(B < (1u << 31) && T < (1u << 31), PL_ERR_INVALID, "V-trace extents too large");
  return pl::vtrace_f64_launch(rew, val, term, imp, bootv, (int)B, (int)T, gamma, lam, rhoClip, cClip, adv, adv_l1,
                               (cudaStream_t)stream);
}

}  // extern "C"
