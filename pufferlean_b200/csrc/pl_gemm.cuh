// Warp-specialised tcgen05 GEMM for sm_100a with fused epilogues for the PPO+Muon update.
//
//   D[M x N] = sum_k A[m,k] * B[n,k]            (bf16 operands, fp32 accumulate in TMEM)
//
// A and B each arrive either K-major (row m / n holds its K values contiguously) or MN-major
// (row k holds the M / N values contiguously); the choice is a template flag per operand, so the
// forward (X W^T), data-gradient (dZ W) and weight-gradient (dZ^T X) products of every layer all
// read the tensors where they already lie, with no transposed copies.
//
// CTA = 10 warps: warp 0 issues TMA tile loads into a STAGES-deep shared-memory ring, warp 1 owns
// two TMEM accumulators (128 lanes x BN fp32 columns each) and issues tcgen05.mma from one thread,
// warps 2-9 drain TMEM through tcgen05.ld and run the epilogue while the next tile accumulates.
// Tiles are BM=128 x BN, BK=64 (one 128-byte swizzle atom of bf16 per row); the kernel is
// persistent, one CTA per SM.
#pragma once
#include "pl_common.cuh"
#include "pl_tc.cuh"

namespace pl {

enum EpiKind : int {
  EPI_F32 = 0,    // out(f32)  = alpha*acc (+ beta*aux) (+ diag*I)  [wgrad, split-K partials, tests]
  EPI_BF16 = 1,   // out(bf16) = alpha*acc (+ beta*aux) (+ diag*I)  [Newton-Schulz chain]
  EPI_FWD = 2,    // z = acc + bias; out(bf16) = act(z); out2(bf16) = z (GELU only)
  EPI_DGRAD = 3,  // out(bf16) = acc * act'(aux); column partial sums of it  [bias grads]
  EPI_PPO = 4,    // logits+value = acc + bias -> PPO objective gradient dOut(bf16) + column sums
};

struct EpiArgs {
  void* out;
  long ldo;          // elements
  long out_bstride;  // elements per blockIdx.z (batch or split-K slice)
  int out_rows, out_cols;  // stores are masked to rows < out_rows, cols < out_cols
  float alpha, beta;
  const __nv_bfloat16* aux;
  long ld_aux, aux_bstride;
  const float* bias;
  void* out2;
  long ldo2;
  float* colsum;  // [gridDim.y][ld_colsum] per-CTA column partial sums (fixed-order reduced later)
  long ld_colsum;
  int act;        // 0 ReLU, 1 GELU (tanh form), 2 identity
  // PPO head (EPI_PPO): one row per thread, per-row columns of the minibatch
  const int* act_idx;
  const float* adv;
  const double* adv_ms;  // optional [mean, std+1e-8]: adv is then normalised in the epilogue
  const float* ret;
  const float* olp;
  const float* ov;  // NULL = unclipped value loss
  int A;
  float vf, ent, clip, vfclip;
  float* newlp;
  float* newval;
  float* loss_part;  // [gridDim.y][8] optional per-CTA loss partials
  unsigned* err;
  int k_splits;      // >1: the z index of a tile is its split-K slice; else its batch index
  int nbatch;        // number of stacked matrices (z extent when k_splits <= 1)
  int tma_out;       // bf16 outputs leave through shared memory and TMA bulk stores (host-checked)
  float diag;        // EPI_F32 / EPI_BF16: added on the diagonal (row == column) of every matrix
  const float* alpha_b;  // EPI_F32 / EPI_BF16, optional: per-matrix factor on alpha (indexed by batch)
  // EPI_BF16 with aux, optional (the Newton-Schulz polynomial of step 0 on an unnormalised input): aux is
  // G = X X^T of the raw X; the epilogue takes s = 1 / (sqrt(trace G) + fold_eps) from G's bf16 diagonal
  // (a fixed-order fold in f64), scales alpha by s^4 and beta by s^2, and writes (float) s to
  // fold_scale[batch] for the next product. Every warp computes the same s.
  float* fold_scale;
  double fold_eps;
};

// s = 1 / (sqrt(sum_i diag_i) + eps) over the m bf16 diagonal entries of a matrix (leading dimension
// ld): lane l folds i = l, l + 32, ... in f64, then a fixed butterfly; the same bits in every warp.
__device__ __forceinline__ double ns_trace_inv(const __nv_bfloat16* g, long ld, int m, double eps, int lane) {
  double t = 0.0;
  for (int i = lane; i < m; i += 32) t += (double)__bfloat162float(__ldcg(g + (long)i * ld + i));
#pragma unroll
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return 1.0 / (sqrt(t) + eps);
}

// Activation codes: 0 ReLU, 1 GELU (tanh form), 2 identity (a linear layer with bias).
__device__ __forceinline__ float act_fwd(float z, int act) {
  if (act == 0) return z > 0.f ? z : 0.f;
  if (act == 2) return z;
  float u = 0.7978845608028654f * (z + 0.044715f * z * z * z);
  return 0.5f * z * (1.f + tanhf(u));
}
__device__ __forceinline__ float act_grad(float z, int act) {
  if (act == 0) return z > 0.f ? 1.f : 0.f;
  if (act == 2) return 1.f;
  float u = 0.7978845608028654f * (z + 0.044715f * z * z * z);
  float t = tanhf(u);
  return 0.5f * (1.f + t) + 0.5f * z * (1.f - t * t) * 0.7978845608028654f * (1.f + 3.f * 0.044715f * z * z);
}

// One level of warp_colsum16's butterfly: lanes with `hi` set keep the upper half of x and send the
// lower half to lane ^ off (the others the reverse); the additions go two values at a time (two-lane
// fp32 adds, each rounded as the scalar add).
template <int HALF>
__device__ __forceinline__ void colsum_level(const float (&x)[2 * HALF], int off, bool hi, float (&y)[HALF]) {
#pragma unroll
  for (int j = 0; j < HALF; j += 2) {
    float2 keep, recv;
    keep.x = hi ? x[j + HALF] : x[j];
    keep.y = hi ? x[j + 1 + HALF] : x[j + 1];
    recv.x = __shfl_xor_sync(0xffffffffu, hi ? x[j] : x[j + HALF], off);
    recv.y = __shfl_xor_sync(0xffffffffu, hi ? x[j + 1] : x[j + 1 + HALF], off);
    const float2 r = __fadd2_rn(keep, recv);
    y[j] = r.x;
    y[j + 1] = r.y;
  }
}
// Sums each of 16 per-lane values over the 32 lanes of a warp with 16 shuffles (a butterfly that
// halves the live values each step). Lane L returns the total of column (L >> 1). Fixed order.
__device__ __forceinline__ float warp_colsum16(const float (&v)[16], int lane) {
  float a[8], b[4], c[2];
  colsum_level<8>(v, 16, lane & 16, a);
  colsum_level<4>(a, 8, lane & 8, b);
  colsum_level<2>(b, 4, lane & 4, c);
  bool hi = lane & 2;
  float send = hi ? c[0] : c[1], keep = hi ? c[1] : c[0];
  float d = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  return d + __shfl_xor_sync(0xffffffffu, d, 1);
}

__device__ __forceinline__ void store_row16_bf16(__nv_bfloat16* p, const float (&v)[16], int nvalid, bool vec) {
  if (vec && nvalid == 16 && ((uintptr_t)p & 15) == 0) {
    uint4 w[2];
    uint32_t* u = reinterpret_cast<uint32_t*>(w);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      u[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    reinterpret_cast<uint4*>(p)[0] = w[0];
    reinterpret_cast<uint4*>(p)[1] = w[1];
  } else {
    for (int j = 0; j < nvalid; j++) p[j] = __float2bfloat16_rn(v[j]);
  }
}
__device__ __forceinline__ void store_row16_f32(float* p, const float (&v)[16], int nvalid, bool vec) {
  if (vec && nvalid == 16 && ((uintptr_t)p & 15) == 0) {
#pragma unroll
    for (int j = 0; j < 4; j++) reinterpret_cast<float4*>(p)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    for (int j = 0; j < nvalid; j++) p[j] = v[j];
  }
}
__device__ __forceinline__ void load_row16_bf16(const __nv_bfloat16* p, float (&v)[16], int nvalid, bool vec) {
  if (vec && nvalid == 16 && ((uintptr_t)p & 15) == 0) {
    uint4 w[2];
    w[0] = reinterpret_cast<const uint4*>(p)[0];
    w[1] = reinterpret_cast<const uint4*>(p)[1];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(w);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      float2 f = __bfloat1622float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; j++) v[j] = (j < nvalid) ? __bfloat162float(p[j]) : 0.f;
  }
}

// tanh on the SFU (tanh.approx.f32, relative error about 2^-11): used where the result is
// rounded to bf16 anyway.
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Activation over a register row with the (warp-uniform) activation code tested once per row,
// so the per-element code is branch-free: v = act(z), or v = acc * act'(z) for the gradient.
// Both in fused multiply-adds with the constants folded (the epilogues are instruction-bound):
//   u = z (k + k c z^2), k = sqrt(2 / pi), c = 0.044715, t = tanh u;
//   GELU(z) = z (1/2 + t/2);  GELU'(z) = (1/2 + t/2) + (1 - t^2) z (k/2 + 3 k c z^2 / 2).
__device__ __forceinline__ float gelu_fast(float z) {
  constexpr float k = 0.7978845608028654f, kc = 0.7978845608028654f * 0.044715f;
  const float z2 = z * z;
  const float t = tanh_fast(z * __fmaf_rn(kc, z2, k));
  return z * __fmaf_rn(0.5f, t, 0.5f);
}
__device__ __forceinline__ float gelu_grad_fast(float z) {
  constexpr float k = 0.7978845608028654f, kc = 0.7978845608028654f * 0.044715f;
  constexpr float h = 0.5f * 0.7978845608028654f, h3 = 1.5f * 0.7978845608028654f * 0.044715f;
  const float z2 = z * z;
  const float t = tanh_fast(z * __fmaf_rn(kc, z2, k));
  return __fmaf_rn(__fmaf_rn(-t, t, 1.f), z * __fmaf_rn(h3, z2, h), __fmaf_rn(0.5f, t, 0.5f));
}
// The same operations two lanes at a time: sm_100's two-lane fp32 instructions round each lane as the
// scalar instruction does, so these are bit-identical to gelu_fast / gelu_grad_fast in half the
// arithmetic instructions (the epilogues that evaluate them are issue-bound).
__device__ __forceinline__ float2 gelu_fast2(float2 z) {
  constexpr float k = 0.7978845608028654f, kc = 0.7978845608028654f * 0.044715f;
  const float2 z2 = __fmul2_rn(z, z);
  const float2 u = __fmul2_rn(z, __ffma2_rn(make_float2(kc, kc), z2, make_float2(k, k)));
  const float2 t = make_float2(tanh_fast(u.x), tanh_fast(u.y));
  return __fmul2_rn(z, __ffma2_rn(make_float2(0.5f, 0.5f), t, make_float2(0.5f, 0.5f)));
}
__device__ __forceinline__ float2 gelu_grad_fast2(float2 z) {
  constexpr float k = 0.7978845608028654f, kc = 0.7978845608028654f * 0.044715f;
  constexpr float h = 0.5f * 0.7978845608028654f, h3 = 1.5f * 0.7978845608028654f * 0.044715f;
  const float2 z2 = __fmul2_rn(z, z);
  const float2 u = __fmul2_rn(z, __ffma2_rn(make_float2(kc, kc), z2, make_float2(k, k)));
  const float2 t = make_float2(tanh_fast(u.x), tanh_fast(u.y));
  const float2 s = __ffma2_rn(make_float2(-t.x, -t.y), t, make_float2(1.f, 1.f));
  const float2 w = __fmul2_rn(z, __ffma2_rn(make_float2(h3, h3), z2, make_float2(h, h)));
  return __ffma2_rn(s, w, __ffma2_rn(make_float2(0.5f, 0.5f), t, make_float2(0.5f, 0.5f)));
}
__device__ __forceinline__ float act_fwd_fast(float z, int act) {
  if (act == 0) return z > 0.f ? z : 0.f;
  if (act == 2) return z;
  return gelu_fast(z);
}
__device__ __forceinline__ float act_grad_fast(float z, int act) {
  if (act == 0) return z > 0.f ? 1.f : 0.f;
  if (act == 2) return 1.f;
  return gelu_grad_fast(z);
}
template <int N>
__device__ __forceinline__ void act_fwd_row(const float (&z)[N], float (&v)[N], int act) {
  static_assert(N % 2 == 0, "rows of an even number of values");
  if (act == 1) {
#pragma unroll
    for (int j = 0; j < N; j += 2) {
      const float2 g = gelu_fast2(make_float2(z[j], z[j + 1]));
      v[j] = g.x;
      v[j + 1] = g.y;
    }
  } else if (act == 0) {
#pragma unroll
    for (int j = 0; j < N; j++) v[j] = z[j] > 0.f ? z[j] : 0.f;
  } else {
#pragma unroll
    for (int j = 0; j < N; j++) v[j] = z[j];
  }
}
template <int N>
__device__ __forceinline__ void act_grad_row(float (&v)[N], const float (&z)[N], int act) {
  static_assert(N % 2 == 0, "rows of an even number of values");
  if (act == 1) {
#pragma unroll
    for (int j = 0; j < N; j += 2) {
      const float2 g = __fmul2_rn(make_float2(v[j], v[j + 1]), gelu_grad_fast2(make_float2(z[j], z[j + 1])));
      v[j] = g.x;
      v[j + 1] = g.y;
    }
  } else if (act == 0) {
#pragma unroll
    for (int j = 0; j < N; j++) v[j] = z[j] > 0.f ? v[j] : 0.f;
  }
}

// Shared memory: 1 KB alignment slack, the TMA ring, the epilogue area (bf16 staging tiles for the
// TMA bulk stores: per epilogue warp STG_BUFS sets of one 32 x 32 tile per output, 1 KB aligned for
// the 64-byte swizzle; then the column reduction scratch [4][BN] + per-warp loss partials), then the
// barriers. The ring takes what is left of 227 KB. The Newton-Schulz products (EPI_BF16) stage into
// two alternating sets, so a chunk never waits for the previous chunk's store to finish reading.
//
// AT (aux through TMA, the data gradient of a short-K product such as the head's, K <= 128): the ring
// keeps 2 stages and the space goes to two aux tiles (128 x BN bf16, 128-byte swizzle) that the
// producer loads with each tile's operands, so the epilogue reads its aux from shared memory instead of
// waiting on DRAM chunk by chunk.
template <int BN, int EPI, bool AT = false>
struct GemmSmem {
  static constexpr int BM = 128, BK = 64;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NOUT = EPI == EPI_FWD ? 2 : ((EPI == EPI_DGRAD || EPI == EPI_BF16) ? 1 : 0);
  static constexpr int STG_BUFS = (EPI == EPI_BF16 || AT) ? 2 : 1;
  static constexpr uint32_t STG_ONE = NOUT * 32 * 32 * 2;
  static constexpr uint32_t STG_WARP = STG_BUFS * STG_ONE;
  static constexpr uint32_t STG_BYTES = 8 * STG_WARP;
  static constexpr uint32_t RED_BYTES =
      (EPI == EPI_DGRAD || EPI == EPI_PPO) ? (4 * BN * 4 + 4 * 8 * 4 + (EPI == EPI_PPO ? 128 * 8 * 4 : 0)) : 0;
  static constexpr uint32_t AUX_TILE = AT ? 128u * BN * 2u : 0u;
  static constexpr uint32_t AUX_BYTES = 2 * AUX_TILE;
  static constexpr uint32_t FIXED = 1024 + 256 + STG_BYTES + RED_BYTES + AUX_BYTES;
  static constexpr int FIT = (int)((232448 - FIXED) / STAGE_BYTES);
  static constexpr int STAGES = AT ? 2 : (FIT > 8 ? 8 : FIT);
  static constexpr uint32_t TOTAL = FIXED + STAGES * STAGE_BYTES;
  static_assert(STAGES >= 2 && FIT >= STAGES, "shared memory budget");
};

// Tile coordinates of linear tile t: n fastest (consecutive tiles share the A row-panel, which
// the CTAs running at the same time then read once from HBM), then m, then the z slice.
struct TileIdx {
  int n, m, z;
};
__device__ __forceinline__ TileIdx tile_of(int t, int num_n, int num_m) {
  TileIdx r;
  r.n = t % num_n;
  const int q = t / num_n;
  r.m = q % num_m;
  r.z = q / num_m;
  return r;
}

// Epilogue of one 128 x BN accumulator tile held in TMEM columns [tcol, tcol + BN).
// Runs on the 4 epilogue warps; warp `sub` owns TMEM lanes / tile rows [32 sub, 32 sub + 32).
// Writes this lane's 32 bf16 values (its row of a 32 x 32 tile) into a staging tile in the TMA
// 64-byte swizzle (16-byte piece c of row r at position c ^ ((r >> 1) & 3); the store map reads it
// back in order): the 8 lanes of each store phase then cover all 32 banks, and every register index
// is static.
__device__ __forceinline__ void stage_row32(uint8_t* tile, int lane, const float (&v)[32]) {
  uint8_t* row = tile + lane * 64;
  const int x = (lane >> 1) & 3;
#pragma unroll
  for (int c = 0; c < 4; c++) {
    uint32_t u[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[8 * c + 2 * k], v[8 * c + 2 * k + 1]);
      u[k] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(row + ((c ^ x) << 4)) = make_uint4(u[0], u[1], u[2], u[3]);
  }
}

// alpha * acc + beta * aux, one rounding per operation in this order. The Newton-Schulz polynomial
// is formed with it in the GEMM epilogue and in the fused small-matrix kernel, so the two agree bit
// for bit; the diagonal term is then one more rounded add on the diagonal only.
__device__ __forceinline__ float axpb(float alpha, float acc, float beta, float aux) {
  return __fmaf_rn(alpha, acc, __fmul_rn(beta, aux));
}

// The 32 bf16 aux values of one row at columns [nc, nc + 32) (zero past cols), as four 16-byte words.
// Read through L2 only: in the persistent Newton-Schulz chain the aux matrix is rewritten by other
// CTAs between the reads of one SM, so a line kept in L1 could be stale.
__device__ __forceinline__ void aux_load32(const __nv_bfloat16* aux_row, int nc, int cols, uint4 (&pre)[4]) {
  if (nc + 32 <= cols) {
#pragma unroll
    for (int i = 0; i < 4; i++) pre[i] = __ldcg(reinterpret_cast<const uint4*>(aux_row + nc) + i);
  } else {
    __align__(16) __nv_bfloat16 t[32];
    for (int q = 0; q < 32; q++) t[q] = (nc + q < cols) ? __ldcg(aux_row + nc + q) : __float2bfloat16_rn(0.f);
#pragma unroll
    for (int i = 0; i < 4; i++) pre[i] = reinterpret_cast<const uint4*>(t)[i];
  }
}

// The 32 bf16 aux values of tile row rl at tile columns [c32, c32 + 32), from an aux tile that TMA wrote
// into shared memory as {64-column, 128-row} boxes in the 128-byte swizzle (16-byte piece q of row r at
// q ^ (r & 7)). The 8 lanes of each 16-byte load phase read 8 consecutive rows: all 32 banks.
__device__ __forceinline__ void aux_smem32(const uint8_t* aux_sm, int rl, int c32, uint4 (&o)[4]) {
  const uint8_t* base = aux_sm + (c32 >> 6) * (128 * 128) + rl * 128;
  const int q0 = (c32 & 63) >> 3;
#pragma unroll
  for (int i = 0; i < 4; i++) o[i] = *reinterpret_cast<const uint4*>(base + (((q0 + i) ^ (rl & 7)) << 4));
}

template <int BN, int EPI, int NB_ = GemmSmem<BN, EPI>::STG_BUFS>
__device__ __forceinline__ void epilogue_tile(const EpiArgs& ep, uint32_t t_row, int m_tile, int n_tile, int bz,
                                              int batch, bool have_acc, int sub, int half, int lane, float* red,
                                              float* rowscr, uint8_t* stg, const CUtensorMap* tmC,
                                              const CUtensorMap* tmC2, uint32_t& seq,
                                              const uint8_t* aux_sm = nullptr) {
  constexpr int BM = 128;
  const int row = m_tile * BM + sub * 32 + lane;
  const bool row_ok = row < ep.out_rows;
  float alpha = ep.alpha_b ? ep.alpha * __ldcg(ep.alpha_b + batch) : ep.alpha;
  float beta = ep.beta;
  if constexpr (EPI == EPI_BF16) {
    if (ep.fold_scale && ep.aux) {
      const double inv = ns_trace_inv(ep.aux + (long)batch * ep.aux_bstride, ep.ld_aux, ep.out_rows, ep.fold_eps, lane);
      alpha = ep.alpha * (float)(inv * inv * inv * inv);
      beta = ep.beta * (float)(inv * inv);
      // a (near-)zero X with a tiny eps: s^4 beyond float range multiplies a G that is zero; keep Pm = a I
      if (!isfinite(alpha)) alpha = 0.f;
      if (!isfinite(beta)) beta = 0.f;
      if (lane == 0) ep.fold_scale[batch] = (float)inv;
    }
  }
  if constexpr (EPI == EPI_PPO) {
    // one minibatch row per TMEM lane; BN covers every logit + the value column
    const int A = ep.A;
    int a = 0;
    float adv = 0.f, ret = 0.f, olp = 0.f, vold = 0.f;
    if (row_ok) {
      a = ep.act_idx[row];
      adv = ep.adv[row];
      if (ep.adv_ms) adv = (float)(((double)adv - ep.adv_ms[0]) / ep.adv_ms[1]);
      ret = ep.ret[row];
      olp = ep.olp[row];
      if (ep.ov) vold = ep.ov[row];
    }
    if constexpr (BN >= 80) {
      if (A + 1 <= 80) {
        // ---- heads of up to 79 actions + the value: the two warps of a row group split its 80 columns
        // (the first group columns [0, 48), the second [48, 80)); each folds its share of the row's
        // max, exp sum and probability-weighted logit sum, the shares meet through shared memory
        // (xch: per row the two maxima, the action logit, the value, the two exp sums and the two
        // weighted sums), and each writes the gradient of its own columns
        const int q0 = half ? 3 : 0, nq = half ? 2 : 3;
        const int rl = sub * 32 + lane;
        float* xr = rowscr + 32 + rl * 8;
        uint32_t r5[3][16];
#pragma unroll
        for (int q = 0; q < 3; q++)
          if (q < nq) tc::tmem_ld16(t_row + 16 * (q0 + q), r5[q]);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 3; q++) tc::tmem_tie16(r5[q]);
        float x[48];
#pragma unroll
        for (int i = 0; i < 48; i++) {
          const int k = 16 * q0 + i;
          x[i] = (i < 16 * nq) ? (have_acc ? __uint_as_float(r5[i >> 4][i & 15]) : 0.f) + (k <= A ? __ldg(ep.bias + k) : 0.f)
                               : 0.f;
        }
        float pm = -INFINITY, xa_own = 0.f, v_own = 0.f;
#pragma unroll
        for (int i = 0; i < 48; i++) {
          const int k = 16 * q0 + i;
          if (i < 16 * nq && k < A) pm = fmaxf(pm, x[i]);
          if (i < 16 * nq && k == a) xa_own = x[i];
          if (i < 16 * nq && k == A) v_own = x[i];
        }
        xr[half] = pm;
        if (half == (a < 48 ? 0 : 1)) xr[2] = xa_own;  // the action's logit (0 past the 80 columns)
        if (half == (A < 48 ? 0 : 1)) xr[3] = v_own;   // the value column
        tc::named_bar_sync(1, 256);
        const float mx = fmaxf(xr[0], xr[1]), xa = xr[2], vnew = xr[3];
        float pse = 0.f, psx = 0.f;
#pragma unroll
        for (int i = 0; i < 48; i++) {
          const int k = 16 * q0 + i;
          if (i < 16 * nq && k < A) {
            const float e = __expf(x[i] - mx);
            pse += e;
            psx += e * x[i];
          }
        }
        xr[4 + half] = pse;
        xr[6 + half] = psx;
        tc::named_bar_sync(1, 256);
        const float se = xr[4] + xr[5], sx = xr[6] + xr[7];
        const float lse = mx + logf(se), pout = sx / se;
        const float logpA = xa - lse;
        const float ratio = expf(logpA - olp);
        const float lo = 1.f - ep.clip, hi = 1.f + ep.clip;
        const float ratioC = ratio < lo ? lo : (ratio > hi ? hi : ratio);
        const float surr1 = adv * ratio, surr2 = adv * ratioC;
        const float dPol = surr1 <= surr2 ? adv * ratio : adv * ((lo < ratio && ratio < hi) ? 1.f : 0.f) * ratio;
        float dv = vnew - ret;
        if (ep.ov && ep.vfclip > 0.f) {
          const float dd = vnew - vold;
          const float vc = vold + (dd < -ep.vfclip ? -ep.vfclip : (dd > ep.vfclip ? ep.vfclip : dd));
          const float du = (vnew - ret) * (vnew - ret), cc = (vc - ret) * (vc - ret);
          if (!(du >= cc) && !(dd > -ep.vfclip && dd < ep.vfclip)) dv = 0.f;
        }
        const float dval = -ep.vf * dv;
        if (row_ok && !half) {
          if (ep.newlp) ep.newlp[row] = logpA;
          if (ep.newval) ep.newval[row] = vnew;
        }
        if (ep.loss_part && !half) {
          const float ent_row = lse - pout;
          float lt[6] = {row_ok ? -fminf(surr1, surr2) : 0.f, row_ok ? 0.5f * (vnew - ret) * (vnew - ret) : 0.f,
                         row_ok ? ent_row : 0.f, row_ok ? (ratio - 1.f) - logf(ratio) : 0.f,
                         row_ok ? -logf(ratio) : 0.f, row_ok ? (fabsf(ratio - 1.f) > ep.clip ? 1.f : 0.f) : 0.f};
#pragma unroll
          for (int q = 0; q < 6; q++) {
            float v = lt[q];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) rowscr[sub * 8 + q] = v;
          }
        }
        __nv_bfloat16* outp = (__nv_bfloat16*)ep.out + (long)row * ep.ldo;
        const bool vec = (ep.ldo % 8) == 0;
#pragma unroll
        for (int q = 0; q < 3; q++) {
          if (q < nq) {
            const int cq = 16 * (q0 + q);
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; j++) {
              const int k = cq + j;
              const float xk = x[16 * q + j];
              const float pk = __expf(xk - lse);
              const float d = k < A ? dPol * ((k == a ? 1.f : 0.f) - pk) + ep.ent * pk * (pout - xk) : (k == A ? dval : 0.f);
              v[j] = row_ok ? d : 0.f;
            }
            if (row_ok && cq < ep.ldo) store_row16_bf16(outp + cq, v, min(16, (int)(ep.ldo - cq)), vec);
            const float cs = warp_colsum16(v, lane);
            if ((lane & 1) == 0) red[sub * BN + cq + (lane >> 1)] = cs;
          }
        }
        if (row_ok && !half) {
          float z[16];
#pragma unroll
          for (int j = 0; j < 16; j++) z[j] = 0.f;
          for (int c0 = 80; c0 < BN && c0 < ep.ldo; c0 += 16) store_row16_bf16(outp + c0, z, min(16, (int)(ep.ldo - c0)), vec);
        }
        tc::named_bar_sync(1, 256);
        const int t = threadIdx.x - 64;
        for (int c = t; c < BN; c += 256) {
          if (c < ep.out_cols)
            ep.colsum[(long)m_tile * ep.ld_colsum + c] = ((red[c] + red[BN + c]) + red[2 * BN + c]) + red[3 * BN + c];
        }
        if (ep.loss_part && t < 6)
          ep.loss_part[(long)m_tile * 8 + t] = ((rowscr[t] + rowscr[8 + t]) + rowscr[16 + t]) + rowscr[24 + t];
        tc::named_bar_sync(1, 256);  // scratch is reused by the next tile
        return;
      }
    }
    // ---- wider heads: one thread per row; the second group of epilogue warps only joins the barriers
    if (half) {
      tc::named_bar_sync(1, 256);
      tc::named_bar_sync(1, 256);
      return;
    }
    float mx = -INFINITY, se = 0.f, xa = 0.f, vnew = 0.f;
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t r[16];
      tc::tmem_ld16(t_row + c0, r);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const int k = c0 + j;
        const float x = (have_acc ? __uint_as_float(r[j]) : 0.f) + (k < ep.out_cols ? ep.bias[k] : 0.f);
        if (k < A) {
          if (x > mx) {
            se = se * expf(mx - x) + 1.f;
            mx = x;
          } else {
            se += expf(x - mx);
          }
          if (k == a) xa = x;
        }
        if (k == A) vnew = x;
      }
    }
    const float lse = mx + logf(se);
    float pout = 0.f;
    for (int c0 = 0; c0 < BN && c0 < A; c0 += 16) {
      uint32_t r[16];
      tc::tmem_ld16(t_row + c0, r);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const int k = c0 + j;
        if (k < A) {
          const float x = (have_acc ? __uint_as_float(r[j]) : 0.f) + ep.bias[k];
          pout += expf(x - lse) * x;
        }
      }
    }
    const float logpA = xa - lse;
    const float ratio = expf(logpA - olp);
    const float lo = 1.f - ep.clip, hi = 1.f + ep.clip;
    const float ratioC = ratio < lo ? lo : (ratio > hi ? hi : ratio);
    const float surr1 = adv * ratio, surr2 = adv * ratioC;
    float dPol;
    if (surr1 <= surr2)
      dPol = adv * ratio;
    else
      dPol = adv * ((lo < ratio && ratio < hi) ? 1.f : 0.f) * ratio;
    float dv = vnew - ret;
    if (ep.ov && ep.vfclip > 0.f) {
      const float dd = vnew - vold;
      const float vc = vold + (dd < -ep.vfclip ? -ep.vfclip : (dd > ep.vfclip ? ep.vfclip : dd));
      const float du = (vnew - ret) * (vnew - ret), cc = (vc - ret) * (vc - ret);
      if (!(du >= cc) && !(dd > -ep.vfclip && dd < ep.vfclip)) dv = 0.f;
    }
    const float dval = -ep.vf * dv;
    if (row_ok) {
      if (ep.newlp) ep.newlp[row] = logpA;
      if (ep.newval) ep.newval[row] = vnew;
    }
    if (ep.loss_part) {
      // per-row loss terms (PufferLib decomposition): pg loss, value loss, entropy, kl, old kl, clipfrac
      const float ent_row = lse - pout;
      float lt[6] = {row_ok ? -fminf(surr1, surr2) : 0.f, row_ok ? 0.5f * (vnew - ret) * (vnew - ret) : 0.f,
                     row_ok ? ent_row : 0.f, row_ok ? (ratio - 1.f) - logf(ratio) : 0.f,
                     row_ok ? -logf(ratio) : 0.f, row_ok ? (fabsf(ratio - 1.f) > ep.clip ? 1.f : 0.f) : 0.f};
#pragma unroll
      for (int q = 0; q < 6; q++) {
        float v = lt[q];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) rowscr[sub * 8 + q] = v;
      }
    }
    __nv_bfloat16* outp = (__nv_bfloat16*)ep.out + (long)row * ep.ldo;
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t r[16];
      tc::tmem_ld16(t_row + c0, r);
      tc::tmem_wait_ld();
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const int k = c0 + j;
        float d = 0.f;
        if (row_ok) {
          if (k < A) {
            const float x = (have_acc ? __uint_as_float(r[j]) : 0.f) + ep.bias[k];
            const float p = expf(x - lse);
            d = dPol * ((k == a ? 1.f : 0.f) - p) + ep.ent * p * (pout - x);
          } else if (k == A) {
            d = dval;
          }
        }
        v[j] = d;
      }
      if (row_ok) {
        const int nvalid = min(16, (int)(ep.ldo - c0));
        if (nvalid > 0) store_row16_bf16(outp + c0, v, nvalid, (ep.ldo % 8) == 0);
      }
      const float cs = warp_colsum16(v, lane);
      if ((lane & 1) == 0) red[sub * BN + c0 + (lane >> 1)] = cs;
    }
    tc::named_bar_sync(1, 256);
    const int t = threadIdx.x - 64;
    for (int c = t; c < BN; c += 128) {
      if (c < ep.out_cols)
        ep.colsum[(long)m_tile * ep.ld_colsum + c] = ((red[c] + red[BN + c]) + red[2 * BN + c]) + red[3 * BN + c];
    }
    if (ep.loss_part && t < 6)
      ep.loss_part[(long)m_tile * 8 + t] = ((rowscr[t] + rowscr[8 + t]) + rowscr[16 + t]) + rowscr[24 + t];
    tc::named_bar_sync(1, 256);  // scratch is reused by the next tile
  } else {
    const int n_base = n_tile * BN;
    const bool do_colsum = (EPI == EPI_DGRAD) && ep.colsum != nullptr;
    // this warp's half of the tile's columns, drained 32 at a time (two TMEM loads per wait)
    const int cb = half * (BN / 2), ce = cb + BN / 2;
    uint32_t rr[2][16];
    constexpr bool STAGED_OK = (EPI == EPI_FWD || EPI == EPI_DGRAD || EPI == EPI_BF16);
    if (STAGED_OK && ep.tma_out) {
      // ---- staged path: 32 x 32 tiles through shared memory, TMA bulk stores (rows/cols past the
      // logical extent are clipped by the tensor map). Pipelined per warp: chunk c + 1's TMEM load is
      // issued once chunk c is staged (its registers are free then) and overlaps chunk c's fence and
      // store; chunk c + 1's bf16 aux piece (Z for act', X for the Newton-Schulz axpby) is loaded
      // before chunk c's math, so its latency hides under a whole chunk.
      const int row0 = m_tile * 128 + sub * 32;
      constexpr bool HAS_AUX = (EPI == EPI_DGRAD || EPI == EPI_BF16);
      constexpr int NCH = BN / 64;  // 32-column chunks in this warp's half of the tile
      constexpr int NB = NB_;
      const bool use_aux = HAS_AUX && ep.aux != nullptr && row_ok;
      const __nv_bfloat16* aux_row =
          use_aux ? ep.aux + (long)batch * ep.aux_bstride + (long)row * ep.ld_aux : nullptr;
      const int left = ep.out_cols - (n_base + cb);
      const int nch = left <= 0 ? 0 : min(NCH, (left + 31) >> 5);
      uint4 pre[4];
      if (nch > 0) {
        tc::tmem_ld16(t_row + cb, rr[0]);
        tc::tmem_ld16(t_row + cb + 16, rr[1]);
        if (use_aux && !aux_sm) aux_load32(aux_row, n_base + cb, ep.out_cols, pre);
      }
#pragma unroll 1
      for (int ch = 0; ch < nch; ch++) {  // nch is warp-uniform
        const int c32 = cb + 32 * ch;
        const int n0 = n_base + c32;
        const bool full = n0 + 32 <= ep.out_cols;
        uint4 cur[4];
        if (use_aux && aux_sm) {  // the tile's aux is already in shared memory (zero past the extents)
          aux_smem32(aux_sm, sub * 32 + lane, c32, cur);
        } else {
#pragma unroll
          for (int i = 0; i < 4; i++) cur[i] = use_aux ? pre[i] : make_uint4(0u, 0u, 0u, 0u);
          if (use_aux && ch + 1 < nch) aux_load32(aux_row, n0 + 32, ep.out_cols, pre);
        }
        const __nv_bfloat16* auxh = reinterpret_cast<const __nv_bfloat16*>(cur);
        float bz[32];
        if constexpr (EPI == EPI_FWD) {
          if (full && ((reinterpret_cast<uintptr_t>(ep.bias + n0) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
              const float4 t = __ldg(reinterpret_cast<const float4*>(ep.bias + n0) + i);
              bz[4 * i] = t.x;
              bz[4 * i + 1] = t.y;
              bz[4 * i + 2] = t.z;
              bz[4 * i + 3] = t.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; j++) bz[j] = (n0 + j) < ep.out_cols ? ep.bias[n0 + j] : 0.f;
          }
        }
        tc::tmem_wait_ld_tie(rr[0], rr[1]);
        float v[32], z[32];
        if (!have_acc) {  // an empty split-K slice: the accumulator was never written
#pragma unroll
          for (int j = 0; j < 16; j++) rr[0][j] = rr[1][j] = 0u;
        }
        // warp-uniform variants, each a branch-free loop
        if constexpr (EPI == EPI_FWD) {
#pragma unroll
          for (int j = 0; j < 32; j++) z[j] = __uint_as_float(rr[j >> 4][j & 15]) + bz[j];
        } else if constexpr (EPI == EPI_DGRAD) {
          if (row_ok && full) {
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = __uint_as_float(rr[j >> 4][j & 15]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; j++)
              v[j] = (row_ok && n0 + j < ep.out_cols) ? __uint_as_float(rr[j >> 4][j & 15]) : 0.f;
          }
        } else if (use_aux) {
#pragma unroll
          for (int j = 0; j < 32; j++)
            v[j] = axpb(alpha, __uint_as_float(rr[j >> 4][j & 15]), beta, __bfloat162float(auxh[j]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; j++) v[j] = __fmul_rn(alpha, __uint_as_float(rr[j >> 4][j & 15]));
        }
        if constexpr (EPI == EPI_BF16) {
          if (n0 == row0) {  // this chunk's columns are the warp's rows: the diagonal passes through it
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = j == lane ? __fadd_rn(v[j], ep.diag) : v[j];
          }
        }
        if constexpr (EPI == EPI_FWD) act_fwd_row(z, v, ep.act);
        if constexpr (EPI == EPI_DGRAD) {
          float aux[32];
#pragma unroll
          for (int j = 0; j < 32; j++) aux[j] = __bfloat162float(auxh[j]);
          act_grad_row(v, aux, ep.act);
        }
        uint8_t* st = stg + (NB == 2 ? (seq & 1u) * GemmSmem<BN, EPI>::STG_ONE : 0u);
        seq++;
        if (lane == 0) tc::bulk_wait_read<NB - 1>();  // the store that last read this tile is done with it
        __syncwarp();
        stage_row32(st, lane, v);
        if constexpr (EPI == EPI_FWD) {
          if (ep.out2) stage_row32(st + 2048, lane, z);
        }
        if (ch + 1 < nch) {  // the registers were consumed above: the next chunk's load reuses them
          tc::tmem_ld16(t_row + c32 + 32, rr[0]);
          tc::tmem_ld16(t_row + c32 + 48, rr[1]);
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tc::tma_store_3d(tmC, st, n0, row0, batch);
          if constexpr (EPI == EPI_FWD) {
            if (ep.out2) tc::tma_store_3d(tmC2, st + 2048, n0, row0, batch);
          }
          tc::bulk_commit();
        }
        if constexpr (EPI == EPI_DGRAD) {
          if (do_colsum) {
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
              float w16[16];
#pragma unroll
              for (int j = 0; j < 16; j++) w16[j] = v[16 * hh + j];
              const float cs = warp_colsum16(w16, lane);
              if ((lane & 1) == 0) red[sub * BN + c32 + 16 * hh + (lane >> 1)] = cs;
            }
          }
        }
      }
    } else
    for (int c32 = cb; c32 < ce; c32 += 32) {
      if (n_base + c32 >= ep.out_cols) break;  // warp-uniform
      tc::tmem_ld16(t_row + c32, rr[0]);
      tc::tmem_ld16(t_row + c32 + 16, rr[1]);
      tc::tmem_wait_ld();
#pragma unroll
     for (int hh = 0; hh < 2; hh++) {
      const int c0 = c32 + 16 * hh;
      const int n0 = n_base + c0;
      if (n0 >= ep.out_cols) break;  // warp-uniform
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; j++) v[j] = have_acc ? __uint_as_float(rr[hh][j]) : 0.f;
      const int nvalid = min(16, ep.out_cols - n0);
      if constexpr (EPI == EPI_F32 || EPI == EPI_BF16) {
        if (row_ok) {
          float x[16];
          if (ep.aux) {
            load_row16_bf16(ep.aux + (long)batch * ep.aux_bstride + (long)row * ep.ld_aux + n0, x, nvalid,
                            (ep.ld_aux % 8) == 0);
          }
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const float t = ep.aux ? axpb(alpha, v[j], beta, x[j]) : __fmul_rn(alpha, v[j]);
            v[j] = row == n0 + j ? __fadd_rn(t, ep.diag) : t;
          }
          const long off = (long)bz * ep.out_bstride + (long)row * ep.ldo + n0;
          if constexpr (EPI == EPI_F32)
            store_row16_f32((float*)ep.out + off, v, nvalid, (ep.ldo % 4) == 0);
          else
            store_row16_bf16((__nv_bfloat16*)ep.out + off, v, nvalid, (ep.ldo % 8) == 0);
        }
      } else if constexpr (EPI == EPI_FWD) {
        if (row_ok) {
          float z[16], h[16];
#pragma unroll
          for (int j = 0; j < 16; j++) {
            z[j] = v[j] + ((n0 + j) < ep.out_cols ? ep.bias[n0 + j] : 0.f);
            h[j] = act_fwd_fast(z[j], ep.act);
          }
          store_row16_bf16((__nv_bfloat16*)ep.out + (long)row * ep.ldo + n0, h, nvalid, (ep.ldo % 8) == 0);
          if (ep.out2)
            store_row16_bf16((__nv_bfloat16*)ep.out2 + (long)row * ep.ldo2 + n0, z, nvalid, (ep.ldo2 % 8) == 0);
        }
      } else if constexpr (EPI == EPI_DGRAD) {
        float x[16];
        if (row_ok) {
          load_row16_bf16(ep.aux + (long)row * ep.ld_aux + n0, x, nvalid, (ep.ld_aux % 8) == 0);
#pragma unroll
          for (int j = 0; j < 16; j++) v[j] = (j < nvalid) ? v[j] * act_grad_fast(x[j], ep.act) : 0.f;
          store_row16_bf16((__nv_bfloat16*)ep.out + (long)row * ep.ldo + n0, v, nvalid, (ep.ldo % 8) == 0);
        } else {
#pragma unroll
          for (int j = 0; j < 16; j++) v[j] = 0.f;
        }
        if (do_colsum) {
          const float cs = warp_colsum16(v, lane);
          if ((lane & 1) == 0) red[sub * BN + c0 + (lane >> 1)] = cs;
        }
      }
     }
    }
    if (do_colsum) {
      tc::named_bar_sync(1, 256);
      const int t = threadIdx.x - 64;
      for (int c = t; c < BN; c += 256) {
        const int n = n_base + c;
        if (n < ep.out_cols)
          ep.colsum[(long)m_tile * ep.ld_colsum + n] = ((red[c] + red[BN + c]) + red[2 * BN + c]) + red[3 * BN + c];
      }
      tc::named_bar_sync(1, 256);  // scratch is reused by the next tile
    }
  }
}

// Persistent kernel: gridDim.x CTAs (at most one per SM) walk the linear tile list. The TMEM holds
// two 128 x BN fp32 accumulators, so the MMA warp fills one while the epilogue warps drain the
// other: the epilogue of tile j overlaps the main loop of tile j+1.
// AT: the aux tile of each output tile comes through TMA (tmC2 is then its {64, 128}-box operand map) into
// one of two shared-memory buffers, loaded by the producer with the tile's operands; aux_full / aux_empty
// hand the buffers between the producer and the epilogue warps.
template <int BN, bool A_MN, bool B_MN, int EPI, bool AT = false>
__global__ void __launch_bounds__(320, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2, int M, int N,
                   int K, EpiArgs ep) {
  static_assert(!AT || EPI == EPI_DGRAD, "aux through TMA is the data gradient's");
  using S = GemmSmem<BN, EPI, AT>;
  constexpr int BM = S::BM, BK = S::BK, STAGES = S::STAGES;
  constexpr uint32_t IDESC = tc::idesc_bf16(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
  constexpr uint32_t TMEM_COLS = 2 * BN;  // 128, 256 or 512: a power of two
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint8_t* sAux = smem + STAGES * S::STAGE_BYTES;        // [2][128 x BN] (AT), 1 KB aligned
  uint8_t* stg_base = sAux + S::AUX_BYTES;               // [8 warps][STG_WARP], 1 KB aligned
  float* red = (float*)(stg_base + S::STG_BYTES);        // [4][BN]
  float* rowscr = red + 4 * BN;                          // [4 warps][8]
  uint64_t* full = (uint64_t*)(stg_base + S::STG_BYTES + S::RED_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* epi_done = acc_empty + 2;   // the 8 epilogue warps have finished with TMEM and their stores
  uint64_t* aux_full = epi_done + 1;    // [2] (AT)
  uint64_t* aux_empty = aux_full + 2;   // [2] (AT)
  uint32_t* tmem_slot = (uint32_t*)(aux_empty + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_n = (N + BN - 1) / BN, num_m = (M + BM - 1) / BM;
  const int num_z = ep.k_splits > 1 ? ep.k_splits : (ep.nbatch > 1 ? ep.nbatch : 1);
  const int total_tiles = num_n * num_m * num_z;
  const int total_kb = (K + BK - 1) / BK;
  const int per_split = ep.k_splits > 1 ? (total_kb + ep.k_splits - 1) / ep.k_splits : total_kb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], 8);  // one arrival per epilogue warp
    }
    tc::mbar_init(epi_done, 8);
    if (AT)
      for (int b = 0; b < 2; b++) {
        tc::mbar_init(&aux_full[b], 1);
        tc::mbar_init(&aux_empty[b], 8);  // one arrival per epilogue warp
      }
    *abort_flag = 0;
    tc::fence_mbar_init();
    tc::tma_prefetch_desc(&tmA);
    tc::tma_prefetch_desc(&tmB);
    if (AT) tc::tma_prefetch_desc(&tmC2);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto kb_range = [&](int z, int& b0, int& b1) {
    if (ep.k_splits > 1) {
      b0 = z * per_split;
      b1 = min(total_kb, b0 + per_split);
      if (b1 < b0) b1 = b0;
    } else {
      b0 = 0;
      b1 = total_kb;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: one ring across all tiles of this CTA
      long it = 0;
      long ja = 0;  // aux tiles issued (AT)
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        const TileIdx ti = tile_of(t, num_n, num_m);
        const int batch = ep.k_splits > 1 ? 0 : ti.z;
        int b0, b1;
        kb_range(ti.z, b0, b1);
        if (AT) {  // this tile's aux, into the buffer the epilogue released two tiles ago
          const int ab = (int)(ja & 1);
          if (ja >= 2 &&
              !tc::mbar_wait(&aux_empty[ab], (uint32_t)(((ja >> 1) - 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 10)) {
            *abort_flag = 1;
            break;
          }
          tc::mbar_expect_tx(&aux_full[ab], S::AUX_TILE);
#pragma unroll
          for (int h = 0; h < BN / 64; h++)
            tc::tma_load_3d(sAux + ab * S::AUX_TILE + h * (128 * 128), &tmC2, &aux_full[ab], ti.n * BN + 64 * h,
                            ti.m * BM, batch);
          ja++;
        }
        for (int kb = b0; kb < b1; kb++, it++) {
          const int s = (int)(it % STAGES);
          if (it >= STAGES &&
              !tc::mbar_wait(&empty[s], (uint32_t)(((it / STAGES) - 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 1)) {
            *abort_flag = 1;
            break;
          }
          const int k0 = kb * BK;
          tc::mbar_expect_tx(&full[s], S::STAGE_BYTES);
          uint8_t* a = sA + s * S::A_BYTES;
          uint8_t* b = sB + s * S::B_BYTES;
          if (!A_MN) {
            tc::tma_load_3d(a, &tmA, &full[s], k0, ti.m * BM, batch);
          } else {
            tc::tma_load_3d(a, &tmA, &full[s], ti.m * BM, k0, batch);
            tc::tma_load_3d(a + 8192, &tmA, &full[s], ti.m * BM + 64, k0, batch);
          }
          if (!B_MN) {
            tc::tma_load_3d(b, &tmB, &full[s], k0, ti.n * BN, batch);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; j++)
              tc::tma_load_3d(b + j * 8192, &tmB, &full[s], ti.n * BN + 64 * j, k0, batch);
          }
        }
      }
      // Drain: every load issued must have landed before the CTA retires.
      for (long i = it - STAGES > 0 ? it - STAGES : 0; i < it; i++)
        tc::mbar_wait(&full[i % STAGES], (uint32_t)((i / STAGES) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 2);
      if (AT)
        for (long i = ja - 2 > 0 ? ja - 2 : 0; i < ja; i++)
          tc::mbar_wait(&aux_full[i & 1], (uint32_t)((i >> 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 11);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer (one thread)
      long it = 0;
      int j = 0;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x, j++) {
        const TileIdx ti = tile_of(t, num_n, num_m);
        int b0, b1;
        kb_range(ti.z, b0, b1);
        const int buf = j & 1;
        if (j >= 2 &&
            !tc::mbar_wait(&acc_empty[buf], (uint32_t)(((j >> 1) - 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 3)) {
          *abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        for (int kb = b0; kb < b1; kb++, it++) {
          const int s = (int)(it % STAGES);
          if (!tc::mbar_wait(&full[s], (uint32_t)((it / STAGES) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 4)) {
            *abort_flag = 1;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a_addr = tc::smem_u32(sA + s * S::A_BYTES);
          const uint32_t b_addr = tc::smem_u32(sB + s * S::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; kk++) {
            // K-major: the 16-element K slice is 32 bytes further along the swizzled row;
            // MN-major: it is 16 rows (2 groups of 8 rows x 128 B) further down.
            const uint64_t ad = A_MN ? tc::sw128_desc(a_addr + kk * 2048, 8192, 1024)
                                     : tc::sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? tc::sw128_desc(b_addr + kk * 2048, 8192, 1024)
                                     : tc::sw128_desc(b_addr + kk * 32, 16, 1024);
            tc::umma_bf16(d_tmem, ad, bd, IDESC, (kb > b0 || kk > 0) ? 1u : 0u);
          }
          tc::umma_commit(&empty[s]);
        }
        tc::umma_commit(&acc_full[buf]);  // also when the slice is empty: the epilogue then writes zeros
      }
      // every MMA this thread issued must complete before TMEM is released
      if (j > 0) tc::mbar_wait(&acc_full[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 5);
    }
  } else {
    // ---------------- epilogue warps 2..9: warp w reads TMEM lanes 32 (w % 4) .. +32 (its rows);
    // warps w and w + 4 share those rows and split the tile's columns
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;
    uint32_t stg_seq = 0;  // chunks this warp has staged: picks the staging tile
    int j = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, j++) {
      const TileIdx ti = tile_of(t, num_n, num_m);
      int b0, b1;
      kb_range(ti.z, b0, b1);
      const int buf = j & 1;
      const bool ok = tc::mbar_wait(&acc_full[buf], (uint32_t)((j >> 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 6) &&
                      (!AT || tc::mbar_wait(&aux_full[buf], (uint32_t)((j >> 1) & 1), ep.err,
                                            PL_ERR_MBAR_TIMEOUT | 12));
      if (!ok || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      tc::tc_fence_after();
      const uint32_t t_row = tmem_base + (uint32_t)(buf * BN) + ((uint32_t)(sub * 32) << 16);
      epilogue_tile<BN, EPI, S::STG_BUFS>(ep, t_row, ti.m, ti.n, ti.z, ep.k_splits > 1 ? 0 : ti.z, b1 > b0, sub, half,
                                          lane, red, rowscr, stg_base + (warp - 2) * S::STG_WARP, &tmC, &tmC2,
                                          stg_seq, AT ? sAux + buf * S::AUX_TILE : nullptr);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(&acc_empty[buf])) : "memory");
        if (AT) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(&aux_empty[buf])) : "memory");
      }
    }
    // bulk stores must finish reading shared memory (and land) before the CTA retires
    if (lane == 0) tc::bulk_wait<0>();
    tc::tc_fence_before();
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(epi_done)) : "memory");
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // TMEM is released only after every epilogue warp has signalled that its reads and stores are done
    // (an explicit handshake: warps 0 and 1 reach the CTA barrier with lane 0 still in its role loop)
    if (lane == 0) tc::mbar_wait(epi_done, 0, ep.err, PL_ERR_MBAR_TIMEOUT | 7);
    __syncwarp();
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- CTA-pair variant
// The same GEMM on clusters of two CTAs (the two SMs of a pair) with cta_group::2 MMAs: a pair tile is
// 256 x BN, CTA r of the pair holds A rows [128 r, 128 r + 128) and B rows (the N side)
// [BN/2 r, BN/2 r + BN/2) of every k-block, and receives accumulator rows [128 r, 128 r + 128) in its
// own TMEM. Per SM that is BN/2 instead of BN B rows per k-block, so each SM moves a third fewer
// operand bytes per flop and its shared-memory ring covers more k-blocks in flight.
//   barriers: full[s] lives in the even CTA (armed there with both halves' bytes; both CTAs' loads
//   report to it); empty[s] and acc_full[b] exist in both CTAs and are released by the even CTA's MMA
//   thread, which commits to each; acc_empty[b] lives in the even CTA and counts the epilogue warps
//   of both CTAs.
template <int BN, int EPI>
struct GemmPairSmem {
  static constexpr int BM = 128, BK = 64;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = (BN / 2) * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t FIXED = GemmSmem<BN, EPI>::FIXED;
  static constexpr int FIT = (int)((232448 - FIXED) / STAGE_BYTES);
  static constexpr int STAGES = FIT > 10 ? 10 : FIT;
  static constexpr uint32_t TOTAL = FIXED + STAGES * STAGE_BYTES;
  static_assert(STAGES >= 2, "shared memory budget");
};

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2, int M,
                        int N, int K, EpiArgs ep) {
  static_assert(EPI != EPI_PPO, "the PPO head runs on single CTAs");
  static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");
  using S = GemmPairSmem<BN, EPI>;
  constexpr int BM = S::BM, BK = S::BK, STAGES = S::STAGES, BNH = BN / 2;
  constexpr uint32_t IDESC = tc::idesc_bf16(2 * BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
  constexpr uint32_t TMEM_COLS = 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint8_t* stg_base = smem + STAGES * S::STAGE_BYTES;  // 1 KB aligned
  float* red = (float*)(stg_base + GemmSmem<BN, EPI>::STG_BYTES);
  float* rowscr = red + 4 * BN;
  uint64_t* full = (uint64_t*)(stg_base + GemmSmem<BN, EPI>::STG_BYTES + GemmSmem<BN, EPI>::RED_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_slot = (uint32_t*)(acc_empty + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_n = (N + BN - 1) / BN, num_m = (M + 2 * BM - 1) / (2 * BM);
  const int num_z = ep.k_splits > 1 ? ep.k_splits : (ep.nbatch > 1 ? ep.nbatch : 1);
  const int total_tiles = num_n * num_m * num_z;
  const int total_kb = (K + BK - 1) / BK;
  const int per_split = ep.k_splits > 1 ? (total_kb + ep.k_splits - 1) / ep.k_splits : total_kb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], 16);  // one arrival per epilogue warp of both CTAs
    }
    *abort_flag = 0;
    tc::fence_mbar_init();
    tc::tma_prefetch_desc(&tmA);
    tc::tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tc::tmem_relinquish_pair();
  }
  tc::tc_fence_before();
  __syncwarp();
  __syncthreads();
  tc::cluster_sync();  // both CTAs' barriers are initialised before either signals the other
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto kb_range = [&](int z, int& b0, int& b1) {
    if (ep.k_splits > 1) {
      b0 = z * per_split;
      b1 = min(total_kb, b0 + per_split);
      if (b1 < b0) b1 = b0;
    } else {
      b0 = 0;
      b1 = total_kb;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer of this CTA's halves; the even CTA arms full[s] for both
      long it = 0;
      for (int t = pair; t < total_tiles && !*abort_flag; t += npairs) {
        const TileIdx ti = tile_of(t, num_n, num_m);
        const int batch = ep.k_splits > 1 ? 0 : ti.z;
        const int arow = ti.m * 2 * BM + (int)rank * BM;
        const int brow = ti.n * BN + (int)rank * BNH;
        int b0, b1;
        kb_range(ti.z, b0, b1);
        for (int kb = b0; kb < b1; kb++, it++) {
          const int s = (int)(it % STAGES);
          if (it >= STAGES &&
              !tc::mbar_wait(&empty[s], (uint32_t)(((it / STAGES) - 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 1)) {
            *abort_flag = 1;
            break;
          }
          const int k0 = kb * BK;
          if (rank == 0) tc::mbar_expect_tx(&full[s], 2 * S::STAGE_BYTES);
          const uint32_t fb = tc::cluster_addr(tc::smem_u32(&full[s]), 0);
          uint8_t* a = sA + s * S::A_BYTES;
          uint8_t* b = sB + s * S::B_BYTES;
          if (!A_MN) {
            tc::tma_load_3d_pair(a, &tmA, fb, k0, arow, batch);
          } else {
            tc::tma_load_3d_pair(a, &tmA, fb, arow, k0, batch);
            tc::tma_load_3d_pair(a + 8192, &tmA, fb, arow + 64, k0, batch);
          }
          if (!B_MN) {
            tc::tma_load_3d_pair(b, &tmB, fb, k0, brow, batch);
          } else {
#pragma unroll
            for (int j = 0; j < BNH / 64; j++) tc::tma_load_3d_pair(b + j * 8192, &tmB, fb, brow + 64 * j, k0, batch);
          }
        }
      }
      // The even CTA's ring drains here: every phase it armed has received both CTAs' bytes.
      if (rank == 0)
        for (long i = it - STAGES > 0 ? it - STAGES : 0; i < it; i++)
          tc::mbar_wait(&full[i % STAGES], (uint32_t)((i / STAGES) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 2);
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer of the pair (even CTA, one thread)
      long it = 0;
      int j = 0;
      for (int t = pair; t < total_tiles && !*abort_flag; t += npairs, j++) {
        const TileIdx ti = tile_of(t, num_n, num_m);
        int b0, b1;
        kb_range(ti.z, b0, b1);
        const int buf = j & 1;
        if (j >= 2 &&
            !tc::mbar_wait(&acc_empty[buf], (uint32_t)(((j >> 1) - 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 3)) {
          *abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        for (int kb = b0; kb < b1; kb++, it++) {
          const int s = (int)(it % STAGES);
          if (!tc::mbar_wait(&full[s], (uint32_t)((it / STAGES) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 4)) {
            *abort_flag = 1;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a_addr = tc::smem_u32(sA + s * S::A_BYTES);
          const uint32_t b_addr = tc::smem_u32(sB + s * S::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; kk++) {
            const uint64_t ad = A_MN ? tc::sw128_desc(a_addr + kk * 2048, 8192, 1024)
                                     : tc::sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? tc::sw128_desc(b_addr + kk * 2048, 8192, 1024)
                                     : tc::sw128_desc(b_addr + kk * 32, 16, 1024);
            tc::umma_bf16_pair(d_tmem, ad, bd, IDESC, (kb > b0 || kk > 0) ? 1u : 0u);
          }
          // stage s is free in both CTAs once these MMAs complete
          const uint32_t e = tc::smem_u32(&empty[s]);
          tc::umma_commit_pair(tc::cluster_addr(e, 0));
          tc::umma_commit_pair(tc::cluster_addr(e, 1));
        }
        const uint32_t f = tc::smem_u32(&acc_full[buf]);
        tc::umma_commit_pair(tc::cluster_addr(f, 0));
        tc::umma_commit_pair(tc::cluster_addr(f, 1));
      }
      if (j > 0) tc::mbar_wait(&acc_full[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 5);
    }
  } else {
    // ---------------- epilogue warps 2..9 of each CTA drain its 128 accumulator rows
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;
    uint32_t stg_seq = 0;  // chunks this warp has staged: picks the staging tile
    int j = 0;
    for (int t = pair; t < total_tiles; t += npairs, j++) {
      const TileIdx ti = tile_of(t, num_n, num_m);
      int b0, b1;
      kb_range(ti.z, b0, b1);
      const int buf = j & 1;
      const int m_blk = ti.m * 2 + (int)rank;
      const bool ok = tc::mbar_wait(&acc_full[buf], (uint32_t)((j >> 1) & 1), ep.err, PL_ERR_MBAR_TIMEOUT | 6);
      if (!ok || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      tc::tc_fence_after();
      const uint32_t t_row = tmem_base + (uint32_t)(buf * BN) + ((uint32_t)(sub * 32) << 16);
      // a 128-row block wholly past M (odd CTA, M not a multiple of 256) has nothing to write: its
      // column partials would fall outside the ceil(M / 128) rows the caller provides
      if (m_blk * BM < M)
        epilogue_tile<BN, EPI>(ep, t_row, m_blk, ti.n, ti.z, ep.k_splits > 1 ? 0 : ti.z, b1 > b0, sub, half, lane, red,
                               rowscr, stg_base + (warp - 2) * GemmSmem<BN, EPI>::STG_WARP, &tmC, &tmC2, stg_seq);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_remote(tc::cluster_addr(tc::smem_u32(&acc_empty[buf]), 0));
    }
    if (lane == 0) tc::bulk_wait<0>();
    __syncwarp();
  }
  tc::tc_fence_before();
  __syncwarp();
  __syncthreads();
  tc::cluster_sync();  // no CTA leaves while the pair's MMAs or loads may still touch its memory
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
struct Operand {
  const void* ptr;  // bf16
  long rows, cols;  // storage: rows x cols, cols contiguous (cols = the inner dimension)
  long ld;          // elements between rows (>= cols, multiple of 8)
  long batch;       // number of stacked matrices (>= 1)
  long bstride;     // elements between stacked matrices
};

// 3-D bf16 operand map {cols, rows, batch} with a {64, box_rows, 1} box in the 128-byte swizzle.
int gemm_operand_map(CUtensorMap* map, const Operand& op, uint32_t box_rows);
// Store map of a bf16 output for the staged epilogue ({32, 32, 1} box, 64-byte swizzle); false when
// the output's alignment rules TMA stores out.
bool gemm_store_map(CUtensorMap* map, const void* ptr, long rows, long cols, long ld, long batch, long bstride);
// C[M x N] = A * B^T with operands given by their storage; a_mn / b_mn say whether the operand is
// stored MN-major (storage rows = K) or K-major (storage rows = M or N).
int gemm_launch(int bn, int epi, bool a_mn, bool b_mn, const Operand& A, const Operand& B, int M, int N, int K,
                int batch, const EpiArgs& ep, cudaStream_t st);
// 0 = single-CTA tiles only, 1 = CTA pairs where eligible, 2 = CTA pairs for the products whose two
// operands are MN-major (the weight gradients; the default); a negative mode only queries. Returns the
// previous mode.
int gemm_set_pair_mode(int mode);

}  // namespace pl
