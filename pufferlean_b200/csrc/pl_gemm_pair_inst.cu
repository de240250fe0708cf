// Kernel instances of the CTA-pair (cta_group::2) GEMM and their lookup table.
#include "pl_gemm.cuh"

namespace pl {

using GemmKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, int, int,
                           int, EpiArgs);

template <int BN, bool AM, bool BM_, int EPI>
static GemmKernel inst_pair(uint32_t* smem) {
  *smem = GemmPairSmem<BN, EPI>::TOTAL;
  return &tc_gemm_pair_kernel<BN, AM, BM_, EPI>;
}

#define PL_INST_PAIR(BN, AM, BMN, EPI) \
  if (bn == BN && a_mn == AM && b_mn == BMN && epi == EPI) return inst_pair<BN, AM, BMN, EPI>(smem);

GemmKernel gemm_pair_instance(int bn, int epi, bool a_mn, bool b_mn, uint32_t* smem) {
  PL_INST_PAIR(256, false, false, EPI_F32)
  PL_INST_PAIR(256, false, true, EPI_F32)
  PL_INST_PAIR(256, true, true, EPI_F32)
  PL_INST_PAIR(256, false, false, EPI_BF16)
  PL_INST_PAIR(256, false, true, EPI_BF16)
  PL_INST_PAIR(256, false, false, EPI_FWD)
  PL_INST_PAIR(256, false, true, EPI_DGRAD)
  return nullptr;
}

}  // namespace pl
