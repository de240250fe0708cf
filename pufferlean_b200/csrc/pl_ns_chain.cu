// Persistent Newton-Schulz chain: every product of every quintic step of a batch of matrices in one
// launch.
//
// The per-step form (ns_run_batched) launches three GEMMs per step -- G = X X^T, Pm = a I + b G + c G G,
// X' = Pm X -- and each launch pays its ramp (barrier set-up, TMEM allocation, the first tile's main
// loop before any epilogue) and its tail (the last, often partial, wave of tiles) on top of the launch
// itself. Here one cooperative launch of one CTA per SM walks a single job list -- step by step,
// product by product, matrix by matrix, tile by tile -- with the warp roles, shared-memory ring,
// double-buffered TMEM accumulators and epilogue of tc_gemm_kernel. A job waits only for what it
// reads: per matrix, three counters count the finished tile parts of G, Pm and X'. Each of a tile's
// 8 epilogue warps waits for its own TMA stores to complete, fences them to the generic proxy and
// bumps the counter behind a GPU-scope fence (8 parts make a tile; no barrier inside the CTA, so no
// warp ever waits for another here). The producer warp polls the counter a job needs with acquire
// loads, then fences to the async proxy before the job's TMA loads.
// Matrix i's Pm tiles can therefore run while matrix j's G tiles are still in flight, and no SM idles
// at a product boundary.
//
// Deadlock freedom: each CTA takes its jobs in increasing list order and every job depends only on
// jobs earlier in the list, so the earliest unfinished job always has its inputs; the launch is
// cooperative, so all CTAs are resident together. Every wait is bounded: a counter wait that runs out
// sets the device error word and an abort word the other waiters watch, and the CTA drains and
// returns like the GEMM does on a barrier timeout.
//
// Symmetry: G = X X^T and Pm = a I + b G + c G G are symmetric, so only their tiles (mt, nt) with
// 128 mt < 256 (nt + 1) -- on or above the diagonal band of 128 x 256 tiles -- are computed (a quarter
// fewer G and Pm jobs at m = 512). A product that reads G or Pm takes each 64-wide k-block of its
// operand rows from where it lies: K-major from the stored tile when that tile exists, otherwise the
// transposed block of the stored upper tile read MN-major (the instruction descriptor's major bit is
// chosen per k-block). Nothing is mirrored and nothing reads the lower band, which is never written.
//
// Buffers: iterate 0 is the input, iterate s >= 1 lives in buffer s & 1; G and Pm have one buffer each. Overwrites are safe by the
// chain itself: G(s, i) rewrites G only after X'(s-1, i) finished, which needed all of Pm(s-1, i), the
// last reader of G(s-1, i); Pm(s, i) needs G(s, i), which needed X'(s-1, i), the last reader of Pm; and
// X'(s, i) rewrites xbuf[(s+1) & 1] only after Pm(s, i), which transitively needed X'(s-1, i) and
// G(s-1, i), the last readers of iterate s-1.
#include "pl_gemm.cuh"
#include "pl_mlp.cuh"
#include "pl_runtime.h"

namespace pl {

namespace {

constexpr int kChainBN = 256;
constexpr int kChainMaxIters = 16;
constexpr unsigned kParts = 8;  // epilogue warps per tile, each publishing its own part

constexpr int kChainMaxGroups = kNsChainMaxGroups;

// Tensor maps of one group (a batch of same-shape matrices).
struct NsChainMaps {
  CUtensorMap xk[3];  // iterate buffers 0, 1 and the input as K-major operands ({64, 128} boxes)
  CUtensorMap xn[3];  // the same as MN-major operands ({64, 64} boxes)
  CUtensorMap xs[3];  // store maps of iterate buffers 0, 1 and of the final bf16 output
  CUtensorMap gk, gs, gn;  // G: K-major operand, store, MN-major operand ({64, 64} boxes) maps
  CUtensorMap pk, ps, pn;  // Pm
  CUtensorMap xk256[3], gk256;  // K-major B views with 256-row boxes
};
struct NsChainMapSet {
  NsChainMaps g[kChainMaxGroups];
};

// Shape, buffers and counters of one group.
struct NsChainGroup {
  int m, n, batch;
  int nG, nX, TG, TX, kbG, kbM;  // tile columns of G / X', tiles per matrix, k-blocks of G / the rest
  int TS;  // G / Pm tiles computed per matrix (the upper band: (mt, nt) with mt < 2 nt + 2)
  int final_kind;  // 0: the last iterate into buffer iters & 1; 1: into the final bf16 output; 2: fp32
  float* scale0;  // optional per-matrix factor of an unnormalised input: [batch] s, [batch] s^2
  double fold_eps;  // >= 0: s comes from trace G of step 0 (written by its Pm epilogue), not from scale0
  const __nv_bfloat16* G;  // aux of the Pm epilogue
  long ldg, gbs;
  float* out_f32;
  long ld_out, obs;
  unsigned* cnt;  // [3][batch] finished tile parts (8 per tile) of G, Pm, X' (zeroed before launch)
};

struct NsChainArgs {
  int ngroups, iters;
  long pjobs[3];   // jobs of each product over all groups, per step
  long step_jobs;  // their sum
  unsigned* abort_word;  // zeroed before launch
  unsigned* err;
  float coef[3 * kChainMaxIters];
  NsChainGroup g[kChainMaxGroups];
};

struct ChainJob {
  int s, p, g, i, mt, nt;
};

// Whether the 64-wide k-block at column k0 of the operand rows starting at row0 (a multiple of 128)
// lies in a computed tile of a symmetric product: tile (row0 / 128, k0 / 256) exists when
// row0 / 128 < 2 (k0 / 256) + 2. For a 256-row B block (row0 = 256 nt) both of its 128-row halves give
// the same answer.
__device__ __forceinline__ bool sym_stored(int row0, int k0) { return (row0 >> 7) < 2 * (k0 >> 8) + 2; }

// Job J of the list: step, product (0 G, 1 Pm, 2 X'), group, matrix, then tile (n fastest; for G and
// Pm only the upper band, row by row from nt = mt / 2).
__device__ __forceinline__ ChainJob chain_job(long J, const NsChainArgs& a) {
  ChainJob j;
  j.s = (int)(J / a.step_jobs);
  long r = J - (long)j.s * a.step_jobs;
  j.p = 0;
  while (j.p < 2 && r >= a.pjobs[j.p]) r -= a.pjobs[j.p++];
  j.g = 0;
  int per = j.p == 2 ? a.g[0].TX : a.g[0].TS;
  while (j.g + 1 < a.ngroups && r >= (long)a.g[j.g].batch * per) {
    r -= (long)a.g[j.g].batch * per;
    j.g++;
    per = j.p == 2 ? a.g[j.g].TX : a.g[j.g].TS;
  }
  j.i = (int)(r / per);
  int t = (int)(r - (long)j.i * per);
  if (j.p == 2) {
    const int nn = a.g[j.g].nX;
    j.nt = t % nn;
    j.mt = t / nn;
  } else {
    const int nn = a.g[j.g].nG;
    int mt = 0;
    while (t >= nn - (mt >> 1)) t -= nn - (mt >> 1), mt++;
    j.mt = mt;
    j.nt = (mt >> 1) + t;
  }
  return j;
}

// Target of the counter job `jb` waits on (0 = none), and the counter itself.
__device__ __forceinline__ unsigned chain_dep(const ChainJob& jb, const NsChainGroup& gp, const unsigned** c) {
  if (jb.p == 0) {  // G(s) reads iterate s: all of X'(s-1)
    *c = gp.cnt + 2L * gp.batch + jb.i;
    return kParts * (unsigned)(jb.s * gp.TX);
  }
  if (jb.p == 1) {  // Pm(s) reads G(s)
    *c = gp.cnt + jb.i;
    return kParts * (unsigned)((jb.s + 1) * gp.TS);
  }
  *c = gp.cnt + (long)gp.batch + jb.i;  // X'(s) reads Pm(s) (and iterate s, finished before G(s))
  return kParts * (unsigned)((jb.s + 1) * gp.TS);
}

// Bounded acquire-poll of a tile counter. Gives up early when another CTA has raised the abort word.
__device__ bool chain_wait(const unsigned* c, unsigned target, unsigned* abort_word, unsigned* err) {
  for (uint32_t it = 0; it < (1u << 22); it++) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
    if (v >= target) return true;
    if (*(volatile unsigned*)abort_word) return false;
    __nanosleep(64);
  }
  atomicOr(err, PL_ERR_MBAR_TIMEOUT | 9);
  atomicExch(abort_word, 1u);
  return false;
}

template <int BN>
__global__ void __launch_bounds__(320, 1)
    ns_chain_kernel(const __grid_constant__ NsChainMapSet ms, const __grid_constant__ NsChainArgs a) {
  using S = GemmSmem<BN, EPI_BF16>;
  constexpr int BM = S::BM, BK = S::BK, STAGES = S::STAGES;
  constexpr uint32_t IDESC_KK = tc::idesc_bf16(BM, BN, 0, 0);
  constexpr uint32_t IDESC_KN = tc::idesc_bf16(BM, BN, 0, 1);
  constexpr uint32_t IDESC_NK = tc::idesc_bf16(BM, BN, 1, 0);
  constexpr uint32_t IDESC_NN = tc::idesc_bf16(BM, BN, 1, 1);
  constexpr uint32_t TMEM_COLS = 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint8_t* stg_base = smem + STAGES * S::STAGE_BYTES;  // [8 warps][STG_WARP], 1 KB aligned
  uint64_t* full = (uint64_t*)(stg_base + S::STG_BYTES + S::RED_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* epi_done = acc_empty + 2;
  uint32_t* tmem_slot = (uint32_t*)(epi_done + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long total = (long)a.iters * a.step_jobs;
  unsigned* abort_word = a.abort_word;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      tc::mbar_init(&acc_full[b], 1);
      tc::mbar_init(&acc_empty[b], 8);
    }
    tc::mbar_init(epi_done, 8);
    *abort_flag = 0;
    tc::fence_mbar_init();
    tc::tma_prefetch_desc(&ms.g[0].xk[2]);
    tc::tma_prefetch_desc(&ms.g[0].gk);
    tc::tma_prefetch_desc(&ms.g[0].pk);
    tc::tma_prefetch_desc(&ms.g[0].xn[2]);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: waits for each job's inputs, then one ring across all jobs
      long it = 0;
      for (long J = blockIdx.x; J < total && !*abort_flag; J += gridDim.x) {
        const ChainJob jb = chain_job(J, a);
        const NsChainGroup& gp = a.g[jb.g];
        const NsChainMaps& maps = ms.g[jb.g];
        const unsigned* c;
        const unsigned target = chain_dep(jb, gp, &c);
        if (target > 0 && !chain_wait(c, target, abort_word, a.err)) {
          *abort_flag = 1;
          break;
        }
        tc::fence_proxy_async_global();
        const int xi = jb.s == 0 ? 2 : (jb.s & 1);  // where iterate s lives
        const CUtensorMap* mA = jb.p == 0 ? &maps.xk[xi] : (jb.p == 1 ? &maps.gk : &maps.pk);
        const CUtensorMap* mAn = jb.p == 1 ? &maps.gn : &maps.pn;  // A's transposed blocks (G or Pm)
        const CUtensorMap* mB = jb.p == 0 ? &maps.xk256[xi] : (jb.p == 1 ? &maps.gk256 : &maps.xn[xi]);
        const int nkb = jb.p == 0 ? gp.kbG : gp.kbM;
        bool ok = true;
        for (int kb = 0; kb < nkb; kb++, it++) {
          const int s = (int)(it % STAGES);
          if (it >= STAGES &&
              !tc::mbar_wait(&empty[s], (uint32_t)(((it / STAGES) - 1) & 1), a.err, PL_ERR_MBAR_TIMEOUT | 1)) {
            ok = false;
            break;
          }
          const int k0 = kb * BK;
          tc::mbar_expect_tx(&full[s], S::STAGE_BYTES);
          uint8_t* pa = sA + s * S::A_BYTES;
          uint8_t* pb = sB + s * S::B_BYTES;
          if (jb.p == 0 || sym_stored(jb.mt * BM, k0)) {  // A K-major: one 128-row box
            tc::tma_load_3d(pa, mA, &full[s], k0, jb.mt * BM, jb.i);
          } else {  // the transposed block of the stored upper tile, MN-major: two 64-row chunks
            tc::tma_load_3d(pa, mAn, &full[s], jb.mt * BM, k0, jb.i);
            tc::tma_load_3d(pa + 8192, mAn, &full[s], jb.mt * BM + 64, k0, jb.i);
          }
          if (jb.p == 0 || (jb.p == 1 && sym_stored(jb.nt * BN, k0))) {  // B K-major: one BN-row box
            tc::tma_load_3d(pb, mB, &full[s], k0, jb.nt * BN, jb.i);
          } else {  // B read MN-major (the iterate, or G's transposed block): 64-column chunks 8 KB apart
            const CUtensorMap* mBn = jb.p == 1 ? &maps.gn : mB;
#pragma unroll
            for (int h = 0; h < BN / 64; h++)
              tc::tma_load_3d(pb + h * 8192, mBn, &full[s], jb.nt * BN + 64 * h, k0, jb.i);
          }
        }
        if (!ok) {
          *abort_flag = 1;
          atomicExch(abort_word, 1u);
          break;
        }
      }
      // every load issued must have landed before the CTA retires
      for (long i = it - STAGES > 0 ? it - STAGES : 0; i < it; i++)
        tc::mbar_wait(&full[i % STAGES], (uint32_t)((i / STAGES) & 1), a.err, PL_ERR_MBAR_TIMEOUT | 2);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer (one thread)
      long it = 0;
      int j = 0;
      for (long J = blockIdx.x; J < total && !*abort_flag; J += gridDim.x, j++) {
        const ChainJob jb = chain_job(J, a);
        const int nkb = jb.p == 0 ? a.g[jb.g].kbG : a.g[jb.g].kbM;
        const int buf = j & 1;
        if (j >= 2 &&
            !tc::mbar_wait(&acc_empty[buf], (uint32_t)(((j >> 1) - 1) & 1), a.err, PL_ERR_MBAR_TIMEOUT | 3)) {
          *abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        for (int kb = 0; kb < nkb; kb++, it++) {
          const int s = (int)(it % STAGES);
          if (!tc::mbar_wait(&full[s], (uint32_t)((it / STAGES) & 1), a.err, PL_ERR_MBAR_TIMEOUT | 4)) {
            *abort_flag = 1;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a_addr = tc::smem_u32(sA + s * S::A_BYTES);
          const uint32_t b_addr = tc::smem_u32(sB + s * S::B_BYTES);
          // operand majors of this k-block, as the producer loaded it
          const int k0 = kb * BK;
          const bool amn = jb.p != 0 && !sym_stored(jb.mt * BM, k0);
          const bool bmn = jb.p == 2 || (jb.p == 1 && !sym_stored(jb.nt * BN, k0));
          const uint32_t idesc = amn ? (bmn ? IDESC_NN : IDESC_NK) : (bmn ? IDESC_KN : IDESC_KK);
#pragma unroll
          for (int kk = 0; kk < BK / 16; kk++) {
            const uint64_t ad = amn ? tc::sw128_desc(a_addr + kk * 2048, 8192, 1024)
                                    : tc::sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = bmn ? tc::sw128_desc(b_addr + kk * 2048, 8192, 1024)
                                    : tc::sw128_desc(b_addr + kk * 32, 16, 1024);
            tc::umma_bf16(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc::umma_commit(&empty[s]);
        }
        tc::umma_commit(&acc_full[buf]);
      }
      if (j > 0) tc::mbar_wait(&acc_full[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1), a.err, PL_ERR_MBAR_TIMEOUT | 5);
    }
  } else {
    // ---------------- epilogue warps 2..9 (rows 32 (w % 4) .., columns split between w and w + 4)
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stg = stg_base + (warp - 2) * S::STG_WARP;
    uint32_t seq = 0;
    int j = 0;
    for (long J = blockIdx.x; J < total; J += gridDim.x, j++) {
      const ChainJob jb = chain_job(J, a);
      const NsChainGroup& gp = a.g[jb.g];
      const NsChainMaps& maps = ms.g[jb.g];
      const int m = gp.m, n = gp.n, B = gp.batch;
      const int buf = j & 1;
      if (!tc::mbar_wait(&acc_full[buf], (uint32_t)((j >> 1) & 1), a.err, PL_ERR_MBAR_TIMEOUT | 6)) {
        *abort_flag = 1;
        break;
      }
      tc::tc_fence_after();
      const uint32_t t_row = tmem_base + (uint32_t)(buf * BN) + ((uint32_t)(sub * 32) << 16);
      const bool last = jb.s + 1 == a.iters;
      EpiArgs e{};
      e.err = a.err;
      e.k_splits = 1;
      e.nbatch = B;
      e.tma_out = 1;
      e.out_rows = m;
      e.alpha = 1.f;
      const CUtensorMap* tmC;
      if (jb.p == 0) {
        e.out_cols = m;
        if (jb.s == 0 && gp.scale0 && gp.fold_eps < 0.0) e.alpha_b = gp.scale0 + B;
        tmC = &maps.gs;
      } else if (jb.p == 1) {
        e.out_cols = m;
        e.alpha = a.coef[3 * jb.s + 2];
        e.beta = a.coef[3 * jb.s + 1];
        if (jb.s == 0 && gp.scale0 && gp.fold_eps >= 0.0) {
          e.fold_scale = gp.scale0;
          e.fold_eps = gp.fold_eps;
        }
        e.diag = a.coef[3 * jb.s];
        e.aux = gp.G;
        e.ld_aux = gp.ldg;
        e.aux_bstride = gp.gbs;
        tmC = &maps.ps;
      } else {
        e.out_cols = n;
        if (jb.s == 0 && gp.scale0) e.alpha_b = gp.scale0;
        tmC = (last && gp.final_kind == 1) ? &maps.xs[2] : &maps.xs[(jb.s + 1) & 1];
      }
      if (jb.p == 2 && last && gp.final_kind == 2) {
        e.out = gp.out_f32;
        e.ldo = gp.ld_out;
        e.out_bstride = gp.obs;
        e.tma_out = 0;
        epilogue_tile<BN, EPI_F32>(e, t_row, jb.mt, jb.nt, jb.i, jb.i, true, sub, half, lane, nullptr, nullptr, stg,
                                   tmC, tmC, seq);
      } else {
        epilogue_tile<BN, EPI_BF16>(e, t_row, jb.mt, jb.nt, jb.i, jb.i, true, sub, half, lane, nullptr, nullptr,
                                    stg, tmC, tmC, seq);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(&acc_empty[buf])) : "memory");
        // publish this warp's part: its stores have completed, are ordered before generic accesses,
        // and the count is bumped after a GPU-scope fence (fp32 output is written by every lane: the
        // warp's lanes were ordered before lane 0 by the epilogue's last __syncwarp)
        tc::bulk_wait<0>();
        tc::fence_proxy_async_global();
        __threadfence();
        atomicAdd(gp.cnt + (long)jb.p * B + jb.i, 1u);
      }
      __syncwarp();
    }
    if (lane == 0) tc::bulk_wait<0>();
    tc::tc_fence_before();
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(epi_done)) : "memory");
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) tc::mbar_wait(epi_done, 0, a.err, PL_ERR_MBAR_TIMEOUT | 7);
    __syncwarp();
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

static int g_ns_chain = 1;  // 0: every batch takes the per-step launches (tests compare the two)
int ns_set_chain_mode(int mode) {
  const int prev = g_ns_chain;
  if (mode >= 0) g_ns_chain = mode ? 1 : 0;
  return prev;
}
// 1: the cooperative chain launch is also recorded into a stream capture (a cooperative kernel node; the
// MinGRU minibatch graph takes it: 3,443 -> 2,561 launches per configs[3] update, 42.9 -> 42.6 ms)
static int g_ns_chain_capture = 1;
int ns_set_chain_capture(int mode) {
  const int prev = g_ns_chain_capture;
  if (mode >= 0) g_ns_chain_capture = mode ? 1 : 0;
  return prev;
}

long ns_chain_counter_words(long batch) { return 3 * batch + 1; }

// Maps and kernel-side description of one group; returns 1 (nothing launched) when its buffers
// cannot take the chain's TMA maps.
static int chain_group(const NsChainGroupHost& h, int iters, NsChainMaps& mp, NsChainGroup& g) {
  const int m = h.m, n = h.n;
  if (h.ldx % 8 || h.xbs % 8 || h.ldg % 8 || !aligned16(h.X) || !aligned16(h.xbuf[0]) || !aligned16(h.xbuf[1]) ||
      !aligned16(h.G) || !aligned16(h.B) || (h.final_bf16 && !aligned16(h.final_bf16)))
    return 1;
  memset(&mp, 0, sizeof(mp));
  __nv_bfloat16* xb[3] = {h.xbuf[0], h.xbuf[1], h.X};
  const long gbs = (long)h.ldg * m;
  for (int b = 0; b < 3; b++) {
    Operand op{xb[b], m, n, h.ldx, h.batch, h.xbs};
    int rc = gemm_operand_map(&mp.xk[b], op, 128);
    if (!rc) rc = gemm_operand_map(&mp.xk256[b], op, 256);
    if (!rc) rc = gemm_operand_map(&mp.xn[b], op, 64);
    if (rc) return rc;
    if (b < 2 && !gemm_store_map(&mp.xs[b], xb[b], m, n, h.ldx, h.batch, h.xbs)) return 1;
  }
  mp.xs[2] = mp.xs[0];
  if (h.final_bf16 && !gemm_store_map(&mp.xs[2], h.final_bf16, m, n, h.ldx, h.batch, h.xbs)) return 1;
  Operand og{h.G, m, m, h.ldg, h.batch, gbs}, opm{h.B, m, m, h.ldg, h.batch, gbs};
  int rc = gemm_operand_map(&mp.gk, og, 128);
  if (!rc) rc = gemm_operand_map(&mp.gk256, og, 256);
  if (!rc) rc = gemm_operand_map(&mp.gn, og, 64);
  if (!rc) rc = gemm_operand_map(&mp.pk, opm, 128);
  if (!rc) rc = gemm_operand_map(&mp.pn, opm, 64);
  if (rc) return rc;
  if (!gemm_store_map(&mp.gs, h.G, m, m, h.ldg, h.batch, gbs) || !gemm_store_map(&mp.ps, h.B, m, m, h.ldg, h.batch, gbs))
    return 1;
  const int nM = (int)ceil_div(m, 128);
  g = NsChainGroup{};
  g.m = m;
  g.n = n;
  g.batch = h.batch;
  g.nG = (int)ceil_div(m, kChainBN);
  g.nX = (int)ceil_div(n, kChainBN);
  g.TG = nM * g.nG;
  g.TX = nM * g.nX;
  g.TS = 0;
  for (int mt = 0; mt < nM; mt++) g.TS += g.nG - (mt >> 1);
  g.kbG = (int)ceil_div(n, 64);
  g.kbM = (int)ceil_div(m, 64);
  g.final_kind = h.out_f32 ? 2 : (h.final_bf16 ? 1 : 0);
  g.scale0 = h.scale0;
  g.fold_eps = h.fold_eps;
  g.G = h.G;
  g.ldg = h.ldg;
  g.gbs = gbs;
  g.out_f32 = h.out_f32;
  g.ld_out = h.ld_out;
  g.obs = h.obs;
  g.cnt = h.cnt;
  (void)iters;
  return PL_OK;
}

int ns_chain_launch(int ngroups, const NsChainGroupHost* hs, const double* coeffs, int iters, unsigned* abort_word,
                    unsigned* err, cudaStream_t st, bool* used) {
  *used = false;
  if (!g_ns_chain || ngroups < 1 || ngroups > kChainMaxGroups || iters > kChainMaxIters || iters < 1) return PL_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  PL_CUDA(cudaStreamIsCapturing(st, &cap));
  if (cap != cudaStreamCaptureStatusNone && !g_ns_chain_capture) return PL_OK;  // the per-step launches instead
  using S = GemmSmem<kChainBN, EPI_BF16>;
  NsChainMapSet mset;
  NsChainArgs a{};
  a.ngroups = ngroups;
  a.iters = iters;
  for (int k = 0; k < ngroups; k++) {
    const int rc = chain_group(hs[k], iters, mset.g[k], a.g[k]);
    if (rc == 1) return PL_OK;
    if (rc) return rc;
    a.pjobs[0] += (long)a.g[k].batch * a.g[k].TS;
    a.pjobs[1] += (long)a.g[k].batch * a.g[k].TS;
    a.pjobs[2] += (long)a.g[k].batch * a.g[k].TX;
  }
  a.step_jobs = a.pjobs[0] + a.pjobs[1] + a.pjobs[2];
  a.abort_word = abort_word;
  a.err = err ? err : device_error_word();
  for (int i = 0; i < 3 * iters; i++) a.coef[i] = (float)coeffs[i];

  static int num_sms[64] = {0};
  int dev = 0;
  PL_CUDA(cudaGetDevice(&dev));
  PL_REQUIRE(dev >= 0 && dev < 64, PL_ERR_UNSUPPORTED, "device index %d out of range", dev);
  if (!num_sms[dev]) {
    PL_CUDA(cudaFuncSetAttribute((const void*)ns_chain_kernel<kChainBN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)S::TOTAL));
    PL_CUDA(cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev));
  }
  const long total = (long)iters * a.step_jobs;
  const int grid = (int)(total < num_sms[dev] ? total : num_sms[dev]);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(320, 1, 1);
  cfg.dynamicSmemBytes = S::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PL_CUDA(cudaLaunchKernelEx(&cfg, ns_chain_kernel<kChainBN>, mset, a));
  count_launch();
  PL_LAUNCH("ns_chain_kernel");
  *used = true;
  return PL_OK;
}

int ns_chain_try(int m, int n, int batch, const double* coeffs, int iters, NsWork& w, __nv_bfloat16* X, long ldx,
                 long xbs, __nv_bfloat16* const xbuf[2], float* out_f32, long ld_out, long obs,
                 __nv_bfloat16* final_bf16, float* scale0, cudaStream_t st, __nv_bfloat16** result, bool* used,
                 double fold_eps) {
  *used = false;
  if (!w.cnt) return PL_OK;  // (short matrices reach here only when the fused one-CTA kernel cannot take them)
  NsChainGroupHost h{};
  h.m = m;
  h.n = n;
  h.batch = batch;
  h.X = X;
  h.xbuf[0] = xbuf[0];
  h.xbuf[1] = xbuf[1];
  h.ldx = ldx;
  h.xbs = xbs;
  h.G = w.G;
  h.B = w.B;
  h.ldg = w.ldg;
  h.out_f32 = out_f32;
  h.ld_out = ld_out;
  h.obs = obs;
  h.final_bf16 = final_bf16;
  h.scale0 = scale0;
  h.fold_eps = scale0 ? fold_eps : -1.0;
  h.cnt = w.cnt;
  PL_CUDA(cudaMemsetAsync(w.cnt, 0, sizeof(unsigned) * (size_t)ns_chain_counter_words(batch), st));
  const int rc = ns_chain_launch(1, &h, coeffs, iters, w.cnt + 3L * batch, w.err, st, used);
  if (rc || !*used) return rc;
  if (result) *result = out_f32 ? nullptr : (final_bf16 ? final_bf16 : xbuf[iters & 1]);
  return PL_OK;
}

}  // namespace pl
