// Host-side bookkeeping twins of the reference's C helpers: per-epoch shuffle and truncated GAE.
// These stay on the host in the reference's update path as well (ffi/pufferffi.c:946-1041); they
// are restated here so the library is a drop-in for the whole call sequence of one update.
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/pufferlean_b200.h"

extern "C" {

// Fisher-Yates per epoch, splitmix64 state chained across epochs (Puffer/RL/VecTrain.lean:240-252).
int pl_shuffle_perm(size_t NT, size_t epochs, uint64_t rng, double* out) {
  if (!out && NT * epochs) return PL_ERR_INVALID;
  uint32_t* a = (uint32_t*)malloc(sizeof(uint32_t) * (NT ? NT : 1));
  if (!a) return PL_ERR_NOMEM;
  uint64_t s = rng;
  for (size_t e = 0; e < epochs; e++) {
    for (size_t i = 0; i < NT; i++) a[i] = (uint32_t)i;
    for (size_t i = 0; i < NT; i++) {
      const size_t j = NT - 1 - i;
      s += 0x9E3779B97F4A7C15ULL;
      uint64_t z = s;
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
      z ^= z >> 31;
      const size_t k = (size_t)(z % (uint64_t)(j + 1));
      const uint32_t t = a[j];
      a[j] = a[k];
      a[k] = t;
    }
    double* dst = out + e * NT;
    for (size_t i = 0; i < NT; i++) dst[i] = (double)a[i];
  }
  free(a);
  return PL_OK;
}

// Truncated GAE, rho = c = 1, reward clamp, adv[T-1] = 0, ret = adv + val (row e*T + t).
int pl_gae_soa(const double* vals, const double* rews, const double* terms, size_t N, size_t T, double gamma,
               double lam, double* out) {
  if ((!vals || !rews || !terms || !out) && N * T) return PL_ERR_INVALID;
  const size_t NT = N * T;
  double* adv = out;
  double* ret = out + NT;
  const volatile double gl = gamma * lam;
  for (size_t e = 0; e < N; e++) {
    const size_t base = e * T;
    if (T >= 1) adv[base + T - 1] = 0.0;
    double last = 0.0;
    for (size_t i = 0; i + 1 < T; i++) {
      const size_t t = base + (T - 2 - i);
      const double nnt = (terms[t] != 0.0) ? 0.0 : 1.0;
      const double rr = rews[t];
      const double r = rr > 1.0 ? 1.0 : (rr < -1.0 ? -1.0 : rr);
      volatile double gv = gamma * vals[t + 1];
      volatile double gvn = gv * nnt;
      volatile double s1 = r + gvn;
      const double delta = s1 - vals[t];
      volatile double k = gl * last;
      volatile double kn = k * nnt;
      last = delta + kn;
      adv[t] = last;
    }
  }
  for (size_t t = 0; t < NT; t++) ret[t] = adv[t] + vals[t];
  return PL_OK;
}

}  // extern "C"
