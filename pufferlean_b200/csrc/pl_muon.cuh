// Muon building blocks shared by the update driver.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

namespace pl {
extern const double kMuonCoeffs[5][3];
// Loads an iters x 3 Newton-Schulz table into constant memory (used by the f64 tier).
int set_ns_coeffs(const double* coeffs, int iters, cudaStream_t st);
// f64 workspace (in doubles) muon_mat_exact needs for one rows x cols matrix.
size_t exact_ws_doubles(int rows, int cols);
// Tight-tier Muon step of one matrix, in place on W and M (bit-exact with the reference oracle). The
// gradient scale is gs, or the device value *gsp when gsp is not NULL (no host round trip).
int muon_mat_exact(int rows, int cols, double* W, double* M, const double* G, double gs, double lr, double wd,
                   double mu, double eps, int iters, double* ws, cudaStream_t st, const double* gsp = nullptr);
// stepVec on n bias entries, in place on b and m (scale gs, or *gsp on the device).
int stepvec_launch(double* b, double* m, const double* g, double lr, double wd, double mu, double gs, long n,
                   cudaStream_t st, const double* gsp = nullptr);
// One layer of the tight tier's group step: W at pm + oW (rows x cols), bias at pm + ob (rows), their
// momenta P doubles further on; Wf and bf receive the f32 copies of the new values.
struct ExactLayer {
  int rows, cols;
  long oW, ob;
  float* Wf;
  float* bf;
};
// True when every matrix fits one CTA's shared memory (then muon_group_exact runs the whole step).
bool muon_group_fits(const ExactLayer* ls, int n, int iters);
// Every layer's exact Muon step (matrices and biases) from the f32 gradient g (same offsets as pm), with
// the gradient scale read on the device from gsp, in one launch; bit-identical to muon_mat_exact and
// stepvec_launch on the widened gradient.
int muon_group_exact(const ExactLayer* ls, int n, double* pm, long P, const float* g, double lr, double wd, double mu,
                     double eps, int iters, const double* gsp, cudaStream_t st);
}  // namespace pl
