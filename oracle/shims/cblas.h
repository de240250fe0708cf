/* CBLAS name map used only to compile the reference's CPU BLAS path (oracle/_ref).
 * The reference includes <cblas.h>; this header routes its two GEMM entry points to the
 * ILP64 OpenBLAS that numpy bundles (exported as scipy_cblas_[ds]gemm64_, 64-bit extents). */
#ifndef PL_ORACLE_CBLAS_SHIM_H
#define PL_ORACLE_CBLAS_SHIM_H
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void scipy_cblas_dgemm64_(enum CBLAS_ORDER, enum CBLAS_TRANSPOSE, enum CBLAS_TRANSPOSE,
                          long long, long long, long long, double, const double*, long long,
                          const double*, long long, double, double*, long long);
void scipy_cblas_sgemm64_(enum CBLAS_ORDER, enum CBLAS_TRANSPOSE, enum CBLAS_TRANSPOSE,
                          long long, long long, long long, float, const float*, long long,
                          const float*, long long, float, float*, long long);
#define cblas_dgemm(o, ta, tb, m, n, k, al, A, lda, B, ldb, be, C, ldc)                          \
  scipy_cblas_dgemm64_((o), (ta), (tb), (long long)(m), (long long)(n), (long long)(k), (al), (A), \
                       (long long)(lda), (B), (long long)(ldb), (be), (C), (long long)(ldc))
#define cblas_sgemm(o, ta, tb, m, n, k, al, A, lda, B, ldb, be, C, ldc)                          \
  scipy_cblas_sgemm64_((o), (ta), (tb), (long long)(m), (long long)(n), (long long)(k), (al), (A), \
                       (long long)(lda), (B), (long long)(ldb), (be), (C), (long long)(ldc))
#ifdef __cplusplus
}
#endif
#endif
