// Host-side bookkeeping twins of the reference's C helpers: column slice, per-epoch shuffle, truncated
// GAE, the feed-forward minibatch row gather, prioritised segment sampling and the MinGRU minibatch
// scalar gather. These stay on the host in the reference's update path as well (ffi/pufferffi.c:13-20,
// 946-1081, 1094-1176); they are restated here so the library is a drop-in for the whole call sequence
// of one update.
#include <math.h>
#include <stdio.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "../../include/pufferlean_b200.h"
#include "pl_host_stage.h"
#include "pl_runtime.h"

extern "C" {

// out = arr[off, off + len): one contiguous copy (ffi/pufferffi.c:13-20). The range must lie inside the
// n-element array (the reference leaves that to the caller; here it fails with PL_ERR_INVALID).
int pl_slice(const double* arr, size_t n, size_t off, size_t len, double* out) {
  if (len == 0) return PL_OK;
  if (!arr || !out || off > n || len > n - off)
    return pl::set_error(PL_ERR_INVALID, "pl_slice: range [%zu, %zu + %zu) outside an array of %zu", off, off, len, n);
  memcpy(out, arr + off, len * sizeof(double));
  return PL_OK;
}

// Minibatch row gather (ffi/pufferffi.c:1046-1081): row k of the minibatch is column row
// (size_t)idxs[k] (truncation of the f64-encoded index, as the reference's cast): its D observation
// values and its action, advantage, return and old log-prob. Plain copies, so bit-exact. Every index
// is checked against the NT rows first (NaN, negative or >= NT fails with PL_ERR_INVALID and nothing
// is written); large minibatches split their rows over the host threads.
int pl_gather_minibatch(const double* obsCol, const double* actions, const double* advs, const double* rets,
                        const double* olps, size_t NT, const double* idxs, size_t Nmb, size_t D, double* mbObs,
                        double* mbAct, double* mbAdv, double* mbRet, double* mbOlp) {
  if (Nmb == 0) return PL_OK;
  if (!actions || !advs || !rets || !olps || !idxs || !mbAct || !mbAdv || !mbRet || !mbOlp || (D && (!obsCol || !mbObs)))
    return pl::set_error(PL_ERR_INVALID, "pl_gather_minibatch: NULL column");
  for (size_t k = 0; k < Nmb; k++)
    if (!(idxs[k] >= 0.0 && idxs[k] < (double)NT))
      return pl::set_error(PL_ERR_INVALID, "pl_gather_minibatch: index %zu (%g) is not a row in [0, %zu)", k, idxs[k],
                           NT);
  auto rows = [&](size_t k0, size_t k1) {
    for (size_t k = k0; k < k1; k++) {
      const size_t i = (size_t)idxs[k];
      if (D) memcpy(mbObs + k * D, obsCol + i * D, D * sizeof(double));
      mbAct[k] = actions[i];
      mbAdv[k] = advs[i];
      mbRet[k] = rets[i];
      mbOlp[k] = olps[i];
    }
  };
  const size_t work = Nmb * (D + 4);
  if (work < ((size_t)1 << 20) || pl::host_threads() < 2) {
    rows(0, Nmb);
    return PL_OK;
  }
  pl::host_parallel([&](int t, int T) {
    const size_t per = (Nmb + (size_t)T - 1) / (size_t)T;
    const size_t k0 = (size_t)t * per, k1 = k0 + per < Nmb ? k0 + per : Nmb;
    if (k0 < k1) rows(k0, k1);
  });
  return PL_OK;
}

// Fisher-Yates per epoch, splitmix64 state chained across epochs (Puffer/RL/VecTrain.lean:240-252).
// The generator is counter-based (step i of the whole sequence draws splitmix64(seed + (i + 1) * gamma)),
// so for large inputs the draws of every epoch are computed on all host threads at once and each
// epoch's swap pass, the only sequential part, runs on its own thread; the output is the same.
static inline uint64_t sm64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
static const uint64_t kGolden = 0x9E3779B97F4A7C15ULL;

int pl_shuffle_perm(size_t NT, size_t epochs, uint64_t rng, double* out) {
  if (!out && NT * epochs) return PL_ERR_INVALID;
  if (NT * epochs >= ((size_t)1 << 16) && NT < ((size_t)1 << 32)) {
    uint32_t* k = (uint32_t*)malloc(sizeof(uint32_t) * NT * epochs);
    uint32_t* a = (uint32_t*)malloc(sizeof(uint32_t) * NT * epochs);
    if (!k || !a) {
      free(k);
      free(a);
      return PL_ERR_NOMEM;
    }
    const size_t total = NT * epochs;
    pl::host_parallel([&](int t, int T) {  // the draws: step i of epoch e is step e NT + i of the stream
      const size_t lo = total * t / T, hi = total * (t + 1) / T;
      for (size_t q = lo; q < hi; q++) {
        const size_t i = q % NT, j = NT - 1 - i;
        k[q] = (uint32_t)(sm64(rng + (uint64_t)(q + 1) * kGolden) % (uint64_t)(j + 1));
      }
    });
    pl::host_parallel([&](int t, int T) {  // the swaps, one epoch per thread
      for (size_t e = (size_t)t; e < epochs; e += (size_t)T) {
        uint32_t* ae = a + e * NT;
        const uint32_t* ke = k + e * NT;
        for (size_t i = 0; i < NT; i++) ae[i] = (uint32_t)i;
        for (size_t i = 0; i < NT; i++) {
          if (i + 32 < NT) __builtin_prefetch(ae + ke[i + 32], 1);  // the draws are known ahead
          const size_t j = NT - 1 - i, kk = ke[i];
          const uint32_t tmp = ae[j];
          ae[j] = ae[kk];
          ae[kk] = tmp;
        }
      }
    });
    pl::host_parallel([&](int t, int T) {
      const size_t lo = total * t / T, hi = total * (t + 1) / T;
      for (size_t q = lo; q < hi; q++) out[q] = (double)a[q];
    });
    free(k);
    free(a);
    return PL_OK;
  }
  uint32_t* a = (uint32_t*)malloc(sizeof(uint32_t) * (NT ? NT : 1));
  if (!a) return PL_ERR_NOMEM;
  uint64_t s = rng;
  for (size_t e = 0; e < epochs; e++) {
    for (size_t i = 0; i < NT; i++) a[i] = (uint32_t)i;
    for (size_t i = 0; i < NT; i++) {
      const size_t j = NT - 1 - i;
      s += kGolden;
      const size_t k = (size_t)(sm64(s) % (uint64_t)(j + 1));
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

// Truncated GAE, rho = c = 1, reward clamp, adv[T-1] = 0, ret = adv + val (row e*T + t). Every
// environment's backward scan is independent: large inputs split the environments over the host
// threads (each scan keeps its own operation order, so the output is the same).
static void gae_envs(const double* vals, const double* rews, const double* terms, size_t e0, size_t e1, size_t T,
                     double gamma, double lam, double* adv, double* ret) {
  const volatile double gl = gamma * lam;
  for (size_t e = e0; e < e1; e++) {
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
    for (size_t t = base; t < base + T; t++) ret[t] = adv[t] + vals[t];
  }
}

int pl_gae_soa(const double* vals, const double* rews, const double* terms, size_t N, size_t T, double gamma,
               double lam, double* out) {
  if ((!vals || !rews || !terms || !out) && N * T) return PL_ERR_INVALID;
  const size_t NT = N * T;
  double* adv = out;
  double* ret = out + NT;
  if (NT >= ((size_t)1 << 15) && N >= 64) {
    pl::host_parallel([&](int t, int Tn) {
      gae_envs(vals, rews, terms, N * t / Tn, N * (t + 1) / Tn, T, gamma, lam, adv, ret);
    });
    return PL_OK;
  }
  gae_envs(vals, rews, terms, 0, N, T, gamma, lam, adv, ret);
  return PL_OK;
}

// Prioritised segment sampling: priorities |adv|^alpha summed in segment order, probabilities with
// the 1e-6 floor, a sequential prefix sum, splitmix64 draws (state rng + (i+1)*GOLD), a lower-bound
// search and the importance weight (N p)^-beta. Same operations in the same order as the reference
// host sampler, so the result is bit-identical.
int pl_prio_sample(const double* advL1, size_t N, size_t mbSegs, double prioAlpha, double annealBeta, uint64_t rng,
                   double* segIdx, double* mbPrio) {
  if (mbSegs == 0) return PL_OK;
  if (!advL1 || !segIdx || !mbPrio || N == 0) return PL_ERR_INVALID;
  double* w = (double*)malloc(sizeof(double) * N);
  double* p = (double*)malloc(sizeof(double) * N);
  double* cum = (double*)malloc(sizeof(double) * N);
  if (!w || !p || !cum) {
    free(w);
    free(p);
    free(cum);
    return PL_ERR_NOMEM;
  }
  double sumW = 0.0;
  for (size_t e = 0; e < N; e++) {
    w[e] = exp(prioAlpha * log(advL1[e] + 1e-12));
    sumW += w[e];
  }
  const double denom = sumW + 1e-6;
  double acc = 0.0;
  for (size_t e = 0; e < N; e++) {
    p[e] = (w[e] + 1e-6) / denom;
    acc += p[e];
    cum[e] = acc;
  }
  const double total = acc;
  for (size_t i = 0; i < mbSegs; i++) {
    uint64_t z = rng + (uint64_t)(i + 1) * 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    z ^= z >> 31;
    const double u = (double)(z >> 11) / 9007199254740992.0 * total;
    size_t lo = 0, hi = N;
    while (lo < hi) {
      const size_t mid = (lo + hi) >> 1;
      if (cum[mid] >= u)
        hi = mid;
      else
        lo = mid + 1;
    }
    const size_t idx = lo < N ? lo : N - 1;
    segIdx[i] = (double)idx;
    mbPrio[i] = exp((-annealBeta) * log((double)N * p[idx] + 1e-12));
  }
  free(w);
  free(p);
  free(cum);
  return PL_OK;
}

// MinGRU minibatch scalars, time-major (os = t*Bmb + b, si = seg[b]*T + t): the advantage mean and
// population std over the sampled rows (b outer, t inner), then act, mbPrio-weighted normalised adv,
// ret = adv + value, old log-prob, terminal flag, old value.
int pl_gather_seq_minibatch(const double* actCol, const double* logpCol, const double* termCol,
                            const double* advFlat, const double* valueBuf, const double* segIdx, const double* mbPrio,
                            size_t T, size_t Bmb, double* out) {
  const size_t nb = T * Bmb;
  if (nb == 0) return PL_OK;
  if (!actCol || !logpCol || !termCol || !advFlat || !valueBuf || !segIdx || !mbPrio || !out) return PL_ERR_INVALID;
  const double navd = (double)nb;
  double sum = 0.0;
  for (size_t b = 0; b < Bmb; b++) {
    const double* ab = advFlat + (size_t)segIdx[b] * T;
    for (size_t t = 0; t < T; t++) sum += ab[t];
  }
  const double mean = sum / navd;
  double sq = 0.0;
  for (size_t b = 0; b < Bmb; b++) {
    const double* ab = advFlat + (size_t)segIdx[b] * T;
    for (size_t t = 0; t < T; t++) {
      const double d = ab[t] - mean;
      sq += d * d;
    }
  }
  const double stde = sqrt(sq / navd) + 1e-8;
  double *pact = out, *padv = out + nb, *pret = out + 2 * nb, *pold = out + 3 * nb, *pterm = out + 4 * nb,
         *pov = out + 5 * nb;
  for (size_t b = 0; b < Bmb; b++) {
    const size_t e = (size_t)segIdx[b];
    const double mp = mbPrio[b];
    for (size_t t = 0; t < T; t++) {
      const size_t si = e * T + t, os = t * Bmb + b;
      const double a = advFlat[si], v = valueBuf[si];
      pact[os] = (double)(unsigned long long)actCol[si];
      padv[os] = mp * (a - mean) / stde;
      pret[os] = a + v;
      pold[os] = logpCol[si];
      pov[os] = v;
      pterm[os] = termCol[si] > 0.5 ? 1.0 : 0.0;
    }
  }
  return PL_OK;
}

// Checkpoint file: u64 P (little-endian) then P f64 bit patterns (little-endian); written byte by
// byte so the layout does not depend on the host's endianness.
static void put_u64le(unsigned char* b, uint64_t v) {
  for (int i = 0; i < 8; i++) b[i] = (unsigned char)(v >> (8 * i));
}
static uint64_t get_u64le(const unsigned char* b) {
  uint64_t v = 0;
  for (int i = 0; i < 8; i++) v |= (uint64_t)b[i] << (8 * i);
  return v;
}

int pl_ckpt_write(const char* path, const double* w, size_t P) {
  if (!path || (!w && P)) return PL_ERR_INVALID;
  FILE* f = fopen(path, "wb");
  if (!f) return PL_ERR_INVALID;
  unsigned char b[8];
  put_u64le(b, (uint64_t)P);
  int ok = fwrite(b, 1, 8, f) == 8;
  for (size_t i = 0; ok && i < P; i++) {
    uint64_t bits;
    memcpy(&bits, &w[i], 8);
    put_u64le(b, bits);
    ok = fwrite(b, 1, 8, f) == 8;
  }
  ok = (fclose(f) == 0) && ok;
  return ok ? PL_OK : PL_ERR_INVALID;
}

int pl_ckpt_read(const char* path, double* w, size_t cap, size_t* P) {
  if (!path || !P) return PL_ERR_INVALID;
  FILE* f = fopen(path, "rb");
  if (!f) return PL_ERR_INVALID;
  fseek(f, 0, SEEK_END);
  const long size = ftell(f);
  fseek(f, 0, SEEK_SET);
  unsigned char b[8];
  if (size < 8 || fread(b, 1, 8, f) != 8) {
    fclose(f);
    *P = 0;
    return size < 8 ? PL_OK : PL_ERR_INVALID;
  }
  const uint64_t hdr = get_u64le(b);
  const uint64_t avail = (uint64_t)(size - 8) / 8;
  const size_t n = (size_t)(hdr < avail ? hdr : avail);
  *P = n;
  if (!w) {
    fclose(f);
    return PL_OK;  // size query
  }
  if (n > cap) {
    fclose(f);
    return PL_ERR_INVALID;
  }
  int ok = 1;
  for (size_t i = 0; ok && i < n; i++) {
    ok = fread(b, 1, 8, f) == 8;
    const uint64_t bits = get_u64le(b);
    memcpy(&w[i], &bits, 8);
  }
  fclose(f);
  return ok ? PL_OK : PL_ERR_INVALID;
}

int pl_policy_save(size_t handle, size_t P, const char* path) {
  if (!handle || !path) return PL_ERR_INVALID;
  double* w = (double*)malloc(sizeof(double) * 2 * (P ? P : 1));
  if (!w) return PL_ERR_NOMEM;
  int rc = pl_policy_download(handle, P, w);  // [params; mom]
  if (!rc) rc = pl_ckpt_write(path, w, P);
  free(w);
  return rc;
}

int pl_policy_restore(const char* path, size_t* P, size_t* handle) {
  if (!path || !P || !handle) return PL_ERR_INVALID;
  size_t n = 0;
  int rc = pl_ckpt_read(path, nullptr, 0, &n);
  if (rc) return rc;
  double* pm = (double*)calloc(2 * (n ? n : 1), sizeof(double));
  if (!pm) return PL_ERR_NOMEM;
  rc = pl_ckpt_read(path, pm, n, &n);
  if (!rc) rc = pl_policy_load(pm, n, handle);
  free(pm);
  if (!rc) *P = n;
  return rc;
}

}  // extern "C"

// Per-segment GAE with bootstrap, then the advantages normalised over all N*T: the host C of the LSTM
// trainer (ffi/pufferffi.c:975-1010, lean_ffi_lstm_gae_boot_norm), same recurrence and fold order.
// Time-major columns [t*N + n]; out = [adv(N*T); ret(N*T)].
extern "C" int pl_lstm_gae_boot_norm(const double* vals, const double* rews, const double* terms,
                                     const double* bootV, size_t N, size_t T, double gamma, double lam,
                                     double* out) {
  if (!vals || !rews || !terms || !bootV || !out) return PL_ERR_INVALID;
  const size_t NT = N * T;
  double* adv = out;
  double* ret = out + NT;
  for (size_t n = 0; n < N; n++) {
    double lastA = 0.0;
    for (size_t i = 0; i < T; i++) {
      const size_t t = T - 1 - i, idx = t * N + n;
      const double nnt = (terms[idx] > 0.5) ? 0.0 : 1.0;
      const double vNext = (t + 1 < T) ? vals[(t + 1) * N + n] : bootV[n];
      const double delta = rews[idx] + gamma * vNext * nnt - vals[idx];
      lastA = delta + gamma * lam * nnt * lastA;
      adv[idx] = lastA;
      ret[idx] = lastA + vals[idx];
    }
  }
  const size_t den = NT > 0 ? NT : 1;
  double sum = 0.0;
  for (size_t i = 0; i < NT; i++) sum += adv[i];
  const double mean = sum / (double)den;
  double vsum = 0.0;
  for (size_t i = 0; i < NT; i++) {
    const double d = adv[i] - mean;
    vsum += d * d;
  }
  const double inv = 1.0 / (sqrt(vsum / (double)den) + 1e-8);
  for (size_t i = 0; i < NT; i++) adv[i] = (adv[i] - mean) * inv;
  return PL_OK;
}
