// Host side of the tcgen05 GEMM: TMA tensor maps, kernel-instance dispatch, launch.
#include <cudaTypedefs.h>

#include <string.h>

#include <mutex>

#include "pl_gemm.cuh"
#include "pl_runtime.h"

namespace pl {

using GemmKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, int, int,
                           int, EpiArgs);

// Instance tables live in pl_gemm_inst.cu (single CTAs) and pl_gemm_pair_inst.cu (CTA pairs).
GemmKernel gemm_instance(int bn, int epi, bool a_mn, bool b_mn, uint32_t* smem_bytes);
GemmKernel gemm_instance_at(int bn, int epi, bool a_mn, bool b_mn, uint32_t* smem_bytes);
GemmKernel gemm_pair_instance(int bn, int epi, bool a_mn, bool b_mn, uint32_t* smem_bytes);

// 0: single CTAs only; 1: CTA pairs for every 256-wide tile of at least 256 rows; 2 (the default): CTA
// pairs for the weight gradients only (both operands MN-major). Measured on the C5 update (262,144-row
// minibatches): pairs run the weight gradient at 1,152 against 1,052 TFLOP/s, the forward (1,026 vs
// 1,053) and the data gradient (850 vs 916) slower; with pairs for the weight gradients alone the
// update took 1,852-1,857 against 1,868-1,871 ms in alternating runs on one box (weight gradients
// 566 against 588 ms per update).
static int g_pair_mode = 2;
int gemm_set_pair_mode(int mode) {
  const int prev = g_pair_mode;
  if (mode >= 0) g_pair_mode = mode <= 2 ? mode : 0;
  return prev;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

// 3-D bf16 tensor map over {cols (contiguous), rows, batch} with a {64, box_rows, 1} box and the
// 128-byte swizzle the UMMA descriptors expect. Out-of-range elements read as zero.
int gemm_operand_map(CUtensorMap* map, const Operand& op, uint32_t box_rows) {
  auto enc = encode_fn();
  PL_REQUIRE(enc != nullptr, PL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  PL_REQUIRE(((uintptr_t)op.ptr & 15) == 0, PL_ERR_INVALID, "GEMM operand base not 16-byte aligned");
  PL_REQUIRE(op.ld % 8 == 0 && op.ld >= op.cols, PL_ERR_INVALID, "GEMM operand ld=%ld must be >= cols and a multiple of 8",
             op.ld);
  long bstride = op.batch > 1 ? op.bstride : op.ld * op.rows;
  PL_REQUIRE(bstride % 8 == 0, PL_ERR_INVALID, "GEMM operand batch stride must be a multiple of 8 elements");
  cuuint64_t dims[3] = {(cuuint64_t)op.cols, (cuuint64_t)op.rows, (cuuint64_t)(op.batch > 0 ? op.batch : 1)};
  cuuint64_t strides[2] = {(cuuint64_t)op.ld * 2, (cuuint64_t)bstride * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(op.ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PL_REQUIRE(r == CUDA_SUCCESS, PL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%ld cols=%ld ld=%ld", (int)r,
             op.rows, op.cols, op.ld);
  return PL_OK;
}

// Store map of a bf16 output for the staged epilogue: {cols, rows, batch} with a {32, 32, 1} box and
// the 64-byte swizzle the staging tiles are written in. Returns false when the output cannot take TMA
// stores (alignment), in which case the epilogue writes directly.
bool gemm_store_map(CUtensorMap* map, const void* ptr, long rows, long cols, long ld, long batch, long bstride) {
  auto enc = encode_fn();
  if (!enc || !ptr || ((uintptr_t)ptr & 15) || (ld * 2) % 16 || ld < cols) return false;
  if (batch > 1 && (bstride * 2) % 16) return false;
  const long bs = batch > 1 ? bstride : ld * rows;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)(batch > 0 ? batch : 1)};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)((bs * 2 + 15) / 16 * 16)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int gemm_launch(int bn, int epi, bool a_mn, bool b_mn, const Operand& A, const Operand& B, int M, int N, int K,
                int batch, const EpiArgs& ep_in, cudaStream_t st) {
  const int bn_in = bn;
  PL_REQUIRE(M > 0 && N > 0 && K > 0, PL_ERR_INVALID, "GEMM with empty extent M=%d N=%d K=%d", M, N, K);
  // Operand storage must cover the logical extents the tiles index.
  PL_REQUIRE(a_mn ? (A.rows >= K && A.cols >= M) : (A.rows >= M && A.cols >= K), PL_ERR_INVALID,
             "GEMM A storage %ldx%ld too small for M=%d K=%d", A.rows, A.cols, M, K);
  PL_REQUIRE(b_mn ? (B.rows >= K && B.cols >= N) : (B.rows >= N && B.cols >= K), PL_ERR_INVALID,
             "GEMM B storage %ldx%ld too small for N=%d K=%d", B.rows, B.cols, N, K);
  uint32_t smem = 0;
  GemmKernel k = nullptr;
  const bool pair = (g_pair_mode == 1 || (g_pair_mode == 2 && a_mn && b_mn)) && bn == 256 && epi != EPI_PPO && M > 128 &&
                    (k = gemm_pair_instance(bn, epi, a_mn, b_mn, &smem)) != nullptr;
  // the data gradient of a short-K product (the head's, K <= 128) is a memory-bound epilogue: 128-wide
  // tiles whose aux comes through TMA into shared memory (needs the staged stores, checked below)
  bool at = false;
  if (!pair && epi == EPI_DGRAD && K <= 128 && ep_in.aux && batch == 1 && ep_in.k_splits <= 1) {
    uint32_t smem_at = 0;
    GemmKernel ka = gemm_instance_at(128, epi, a_mn, b_mn, &smem_at);
    if (ka) {
      at = true;
      k = ka;
      smem = smem_at;
      bn = 128;
    }
  }
  if (!pair && !at) k = gemm_instance(bn, epi, a_mn, b_mn, &smem);
  PL_REQUIRE(k != nullptr, PL_ERR_UNSUPPORTED, "no GEMM instance bn=%d epi=%d a_mn=%d b_mn=%d", bn, epi, (int)a_mn,
             (int)b_mn);
  if (epi == EPI_PPO) PL_REQUIRE(N <= bn, PL_ERR_INVALID, "PPO head needs all %d outputs in one tile (bn=%d)", N, bn);
  CUtensorMap ma, mb;
  int rc = gemm_operand_map(&ma, A, a_mn ? 64 : 128);
  if (rc) return rc;
  rc = gemm_operand_map(&mb, B, b_mn ? 64 : (uint32_t)(pair ? bn / 2 : bn));  // a pair CTA loads half of B's rows
  if (rc) return rc;
  EpiArgs ep = ep_in;
  if (!ep.err) ep.err = device_error_word();
  CUtensorMap mc, mc2;
  memset(&mc, 0, sizeof(mc));
  memset(&mc2, 0, sizeof(mc2));
  ep.tma_out = 0;
  if (epi == EPI_FWD || epi == EPI_DGRAD || epi == EPI_BF16) {
    bool ok = gemm_store_map(&mc, ep.out, ep.out_rows, ep.out_cols, ep.ldo, batch, ep.out_bstride);
    if (ok && epi == EPI_FWD && ep.out2) ok = gemm_store_map(&mc2, ep.out2, ep.out_rows, ep.out_cols, ep.ldo2, 1, 0);
    // the staged epilogue reads its aux tile with aligned 16-byte loads
    if (ok && ep.aux && (((uintptr_t)ep.aux & 15) || (ep.ld_aux % 8) || (batch > 1 && (ep.aux_bstride % 8))))
      ok = false;
    ep.tma_out = ok ? 1 : 0;
  }
  if (at) {
    // the aux operand map ({64, 128} boxes, 128-byte swizzle) rides in the second store map's slot
    Operand aux{ep.aux, ep.out_rows, ep.out_cols, ep.ld_aux, 1, 0};
    if (!ep.tma_out || gemm_operand_map(&mc2, aux, 128) != PL_OK) {
      clear_error();
      at = false;
      bn = bn_in;
      k = gemm_instance(bn, epi, a_mn, b_mn, &smem);
      PL_REQUIRE(k != nullptr, PL_ERR_UNSUPPORTED, "no GEMM instance bn=%d epi=%d", bn, epi);
    }
  }
  int splits = ep.k_splits > 1 ? ep.k_splits : 1;
  PL_REQUIRE(splits == 1 || batch == 1, PL_ERR_INVALID, "split-K and batching are exclusive");
  ep.nbatch = batch;
  static int num_sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && num_sms[dev] == 0) cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int sms = (dev >= 0 && dev < 64 && num_sms[dev] > 0) ? num_sms[dev] : 148;
  dim3 grid;
  if (pair) {
    // one cluster of two CTAs per pair tile of 256 rows, at most one CTA per SM
    const long ptiles = ceil_div(N, bn) * ceil_div(M, 256) * (long)(splits > 1 ? splits : batch);
    const long pairs = ptiles < sms / 2 ? ptiles : sms / 2;
    grid = dim3((unsigned)(2 * pairs), 1, 1);
  } else {
    const long tiles = ceil_div(N, bn) * ceil_div(M, 128) * (long)(splits > 1 ? splits : batch);
    grid = dim3((unsigned)(tiles < sms ? tiles : sms), 1, 1);
  }
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> g(mu);
    static void* configured[256];
    static int nconf = 0;
    bool found = false;
    for (int i = 0; i < nconf; i++)
      if (configured[i] == (void*)k) found = true;
    if (!found) {
      PL_CUDA(cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      if (nconf < 256) configured[nconf++] = (void*)k;
    }
  }
  k<<<grid, 320, smem, st>>>(ma, mb, mc, mc2, M, N, K, ep);
  count_launch();
  PL_LAUNCH("tc_gemm_kernel");
  return PL_OK;
}

}  // namespace pl
