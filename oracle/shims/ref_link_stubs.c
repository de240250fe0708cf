/* Link-time companions for compiling the reference's CPU C files on their own (oracle/_ref).
 * pufferblas.c refers to three symbols that live in the reference's CUDA translation unit and to
 * OpenBLAS's thread setter; the CPU functions the oracle harness calls never reach the first
 * three, and the fourth forwards to numpy's bundled OpenBLAS. */
#include <stddef.h>
int g_mgLossOn = 0;
double g_mgLoss[7] = {0, 0, 0, 0, 0, 0, 0};
int cuda_lstm_ppo_grad_batch(const double* pp, const double* obsB, const double* actA, const double* advA,
                             const double* retA, const double* oldA, const double* termA, const double* h0s,
                             const double* c0s, size_t B, size_t T, size_t H, size_t D, size_t A, double vfCoef,
                             double entCoef, double clipEps, double* gOut, double* outHostOrNull, int tier) {
  (void)pp; (void)obsB; (void)actA; (void)advA; (void)retA; (void)oldA; (void)termA; (void)h0s; (void)c0s;
  (void)B; (void)T; (void)H; (void)D; (void)A; (void)vfCoef; (void)entCoef; (void)clipEps; (void)gOut;
  (void)outHostOrNull; (void)tier;
  return 0; /* "no device path": the reference then runs its CPU code */
}
void scipy_openblas_set_num_threads64_(int);
void openblas_set_num_threads(int n) { scipy_openblas_set_num_threads64_(n); }
