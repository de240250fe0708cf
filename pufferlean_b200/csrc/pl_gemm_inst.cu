// Kernel instances of the tcgen05 GEMM used by the update path, and their lookup table.
#include "pl_gemm.cuh"

namespace pl {

using GemmKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, int, int,
                           int, EpiArgs);

template <int BN, bool AM, bool BM_, int EPI, bool AT = false>
static GemmKernel inst(uint32_t* smem) {
  *smem = GemmSmem<BN, EPI, AT>::TOTAL;
  return &tc_gemm_kernel<BN, AM, BM_, EPI, AT>;
}

// The data gradient with its aux tiles through TMA (short-K products: the head's, K <= 128).
GemmKernel gemm_instance_at(int bn, int epi, bool a_mn, bool b_mn, uint32_t* smem) {
  if (bn == 128 && !a_mn && b_mn && epi == EPI_DGRAD) return inst<128, false, true, EPI_DGRAD, true>(smem);
  return nullptr;
}

#define PL_INST(BN, AM, BMN, EPI) \
  if (bn == BN && a_mn == AM && b_mn == BMN && epi == EPI) return inst<BN, AM, BMN, EPI>(smem);

GemmKernel gemm_instance(int bn, int epi, bool a_mn, bool b_mn, uint32_t* smem) {
  // plain fp32 output: every operand-major combination (weight gradients, tests)
  PL_INST(128, false, false, EPI_F32)
  PL_INST(128, false, true, EPI_F32)
  PL_INST(128, true, false, EPI_F32)
  PL_INST(128, true, true, EPI_F32)
  PL_INST(256, false, false, EPI_F32)
  PL_INST(256, false, true, EPI_F32)
  PL_INST(256, true, true, EPI_F32)
  // bf16 output with optional fused axpby (Newton-Schulz chain)
  PL_INST(128, false, false, EPI_BF16)
  PL_INST(128, false, true, EPI_BF16)
  PL_INST(256, false, false, EPI_BF16)
  PL_INST(256, false, true, EPI_BF16)
  // MLP forward / data-gradient / PPO head
  PL_INST(64, false, false, EPI_FWD)
  PL_INST(128, false, false, EPI_FWD)
  PL_INST(256, false, false, EPI_FWD)
  PL_INST(64, false, true, EPI_DGRAD)
  PL_INST(128, false, true, EPI_DGRAD)
  PL_INST(256, false, true, EPI_DGRAD)
  PL_INST(64, false, false, EPI_PPO)
  PL_INST(128, false, false, EPI_PPO)
  return nullptr;
}

}  // namespace pl
