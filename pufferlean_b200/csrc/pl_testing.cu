// Test hooks (include/pufferlean_b200_testing.h): the GEMM and its epilogues on raw device pointers.
#include "../../include/pufferlean_b200_testing.h"
#include "pl_gemm.cuh"
#include "pl_mlp.cuh"

extern "C" int pl_test_gemm(const pl_test_gemm_args* g, void* stream) {
  PL_REQUIRE(g != nullptr, PL_ERR_INVALID, "pl_test_gemm: NULL args");
  pl::Operand A{g->a, g->a_rows, g->a_cols, g->a_ld, g->batch > 1 ? g->batch : 1, g->a_bstride};
  pl::Operand B{g->b, g->b_rows, g->b_cols, g->b_ld, g->batch > 1 ? g->batch : 1, g->b_bstride};
  pl::EpiArgs ep{};
  ep.out = g->out;
  ep.ldo = g->ldo;
  ep.out_bstride = g->out_bstride;
  ep.out_rows = g->out_rows;
  ep.out_cols = g->out_cols;
  ep.alpha = g->alpha;
  ep.beta = g->beta;
  ep.aux = (const __nv_bfloat16*)g->aux;
  ep.ld_aux = g->ld_aux;
  ep.aux_bstride = g->aux_bstride;
  ep.bias = g->bias;
  ep.out2 = g->out2;
  ep.ldo2 = g->ldo2;
  ep.colsum = g->colsum;
  ep.ld_colsum = g->ld_colsum;
  ep.act = g->act;
  ep.act_idx = g->act_idx;
  ep.adv = g->adv;
  ep.ret = g->ret;
  ep.olp = g->olp;
  ep.ov = g->ov;
  ep.A = g->A;
  ep.vf = g->vf;
  ep.ent = g->ent;
  ep.clip = g->clip;
  ep.vfclip = g->vfclip;
  ep.newlp = g->newlp;
  ep.newval = g->newval;
  ep.loss_part = g->loss_part;
  ep.k_splits = g->k_splits;
  return pl::gemm_launch(g->bn, g->epi, g->a_mn != 0, g->b_mn != 0, A, B, g->M, g->N, g->K,
                         g->batch > 1 ? g->batch : 1, ep, (cudaStream_t)stream);
}

extern "C" int pl_test_gemm_pair_mode(int mode) { return pl::gemm_set_pair_mode(mode); }
extern "C" int pl_test_ns_small_mode(int mode) { return pl::ns_set_small_mode(mode); }
extern "C" int pl_test_ns_chain_mode(int mode) { return pl::ns_set_chain_mode(mode); }
extern "C" int pl_test_ns_chain_capture(int mode) { return pl::ns_set_chain_capture(mode); }

extern "C" int pl_test_device_error(unsigned* code) {
  unsigned* w = pl::device_error_word();
  unsigned v = 0;
  if (w) {
    PL_CUDA(cudaMemcpy(&v, w, sizeof(unsigned), cudaMemcpyDeviceToHost));
    PL_CUDA(cudaMemset(w, 0, sizeof(unsigned)));
  }
  if (code) *code = v;
  return PL_OK;
}
