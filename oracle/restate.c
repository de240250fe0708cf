/* oracle/restate.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A CPU restatement, in plain f64 C, of the reference algorithms on the PPO+Muon update path.
 * Each function cites the reference file:line it follows (paths are relative to the reference
 * project root). Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm call into this library, and only as the checker or the timed CPU baseline; the product
 * library never links or loads it.
 *
 * Pinning: the f64 functions here are checked bit-for-bit against the reference's own C code
 * compiled from its sources (oracle/_ref, see oracle/Makefile) on the seeded known-answer inputs
 * of the reference's verify-* modes; the resulting vectors are committed under tests/golden/.
 *
 * Build with -O2 -ffp-contract=off (no fused multiply-add), which is what makes the f64 folds
 * reproduce the reference's IEEE op order exactly (lakefile.lean:69-71, 101-103). */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_GOLD 0x9E3779B97F4A7C15ULL

/* ---------------------------------------------------------------- PRNG -------------------- */
/* rngNext: one splitmix64 step (Puffer/RL/Train.lean:18-24). Returns the word; *s advances by GOLD. */
uint64_t orc_rng_next(uint64_t* s) {
  uint64_t sp = *s + ORC_GOLD;
  *s = sp;
  uint64_t z = sp;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
/* uniform01: top 53 bits over 2^53 (Puffer/RL/Train.lean:27-28). */
double orc_uniform01(uint64_t w) { return (double)(w >> 11) / 9007199254740992.0; }
/* randF lo hi: lo + (hi-lo)*uniform01 (Exe/Puffer.lean:65-67). */
double orc_randF(double lo, double hi, uint64_t* s) {
  uint64_t w = orc_rng_next(s);
  return lo + (hi - lo) * orc_uniform01(w);
}

/* ---------------------------------------------------------------- advantage scans ---------- */
/* computePuffAdvantageV applied to each of B rows of a B x T row-major batch
 * (Puffer/RL/VecTrain.lean:98-114): adv[T-1]=0; t=T-2..0; terminal = term != 0. */
void orc_vtrace(const double* rew, const double* val, const double* term, const double* imp, size_t B, size_t T,
                double gamma, double lam, double rhoClip, double cClip, double* adv) {
  for (size_t b = 0; b < B; b++) {
    const double* rw = rew + b * T;
    const double* vv = val + b * T;
    const double* tm = term + b * T;
    const double* im = imp + b * T;
    double* ad = adv + b * T;
    for (size_t t = 0; t < T; t++) ad[t] = 0.0;
    double lastA = 0.0;
    for (size_t i = 0; i + 1 < T; i++) {
      size_t t = T - 2 - i;
      double nnt = (tm[t] != 0.0) ? 0.0 : 1.0;
      double iv = im[t];
      double rho = iv < rhoClip ? iv : rhoClip;
      double c = iv < cClip ? iv : cClip;
      double rr = rw[t];
      double r = rr > 1.0 ? 1.0 : (rr < -1.0 ? -1.0 : rr);
      double delta = rho * (r + gamma * vv[t + 1] * nnt - vv[t]);
      lastA = delta + gamma * lam * c * lastA * nnt;
      ad[t] = lastA;
    }
  }
}

/* vtraceMinGRUFlat (Puffer/RL/VecTrain.lean:122-139): scalar delta rho*r + gamma*V'*nnt - V, the last
 * step bootstrapped from bootv[row], terminal = term > 0.5, t = T-1..0. `min` is Lean's Float min
 * (a <= b ? a : b), identical to the `<` ternary on finite inputs. */
void orc_vtrace_mingru(const double* rew, const double* val, const double* term, const double* imp,
                       const double* bootv, size_t B, size_t T, double gamma, double lam, double rhoClip,
                       double cClip, double* adv) {
  for (size_t e = 0; e < B; e++) {
    double lastA = 0.0;
    for (size_t i = 0; i < T; i++) {
      size_t t = T - 1 - i, idx = e * T + t;
      double nnt = term[idx] > 0.5 ? 0.0 : 1.0;
      double vNext = (t + 1 < T) ? val[e * T + t + 1] : bootv[e];
      double rho = imp[idx] <= rhoClip ? imp[idx] : rhoClip;
      double c = imp[idx] <= cClip ? imp[idx] : cClip;
      double rr = rew[idx];
      double r = rr > 1.0 ? 1.0 : (rr < -1.0 ? -1.0 : rr);
      double delta = rho * r + gamma * vNext * nnt - val[idx];
      lastA = delta + gamma * lam * c * lastA * nnt;
      adv[idx] = lastA;
    }
  }
}

/* Sigma_t |adv[e,t]| per segment, sequential in t (the host prioSample's inner sum,
 * ffi/pufferffi.c:1094-1106 consumes it; device twin ffi/puffercuda.cu:311-312). */
void orc_adv_l1(const double* adv, size_t N, size_t T, double* out) {
  for (size_t e = 0; e < N; e++) {
    double s = 0.0;
    for (size_t t = 0; t < T; t++) s += fabs(adv[e * T + t]);
    out[e] = s;
  }
}

/* Truncated GAE over env segments with returns (the MLP trainer's buildBatchSoA; the reference's C twin is
 * ffi/pufferffi.c:946-971). It is computePuffAdvantageV with rho = c = 1, so it is restated through
 * orc_vtrace's recurrence with the importance factors fixed at one. out = [adv(NT); ret(NT)]. */
void orc_gae_soa(const double* vals, const double* rews, const double* terms, size_t N, size_t T, double gamma,
                 double lam, double* out) {
  size_t NT = N * T;
  double* adv = out;
  double* ret = out + NT;
  for (size_t e = 0; e < N; e++) {
    size_t base = e * T;
    for (size_t t = 0; t < T; t++) adv[base + t] = 0.0;
    double lastA = 0.0;
    for (size_t i = 0; i + 1 < T; i++) {
      size_t t = base + (T - 2 - i);
      double nnt = (terms[t] != 0.0) ? 0.0 : 1.0;
      double rr = rews[t];
      double r = rr > 1.0 ? 1.0 : (rr < -1.0 ? -1.0 : rr);
      double delta = r + gamma * vals[t + 1] * nnt - vals[t];
      lastA = delta + gamma * lam * lastA * nnt;
      adv[t] = lastA;
    }
  }
  for (size_t t = 0; t < NT; t++) ret[t] = adv[t] + vals[t];
}

/* ---------------------------------------------------------------- bookkeeping -------------- */
/* shuffleIdx (Puffer/RL/VecTrain.lean:240-252) once per epoch, states chained, f64-encoded into
 * perm[epochs*NT] (the flat layout ffi/pufferffi.c:1017-1041 returns). */
void orc_shuffle_perm(size_t NT, size_t epochs, uint64_t rng, double* out) {
  size_t* a = (size_t*)malloc(sizeof(size_t) * (NT ? NT : 1));
  uint64_t s = rng;
  for (size_t e = 0; e < epochs; e++) {
    for (size_t i = 0; i < NT; i++) a[i] = i;
    for (size_t i = 0; i < NT; i++) {
      size_t j = NT - 1 - i;
      uint64_t w = orc_rng_next(&s);
      size_t k = (size_t)(w % (uint64_t)(j + 1));
      size_t tmp = a[j];
      a[j] = a[k];
      a[k] = tmp;
    }
    for (size_t i = 0; i < NT; i++) out[e * NT + i] = (double)a[i];
  }
  free(a);
}

/* mkBatchArrays-style row gather: dst rows = src rows at idx (ffi/pufferffi.c:1046-1081 semantics). */
void orc_gather_minibatch(const double* obs, const double* act, const double* adv, const double* ret,
                          const double* olp, const double* idx, size_t Nmb, size_t D, double* mbObs, double* mbAct,
                          double* mbAdv, double* mbRet, double* mbOlp) {
  for (size_t k = 0; k < Nmb; k++) {
    size_t r = (size_t)idx[k];
    memcpy(mbObs + k * D, obs + r * D, sizeof(double) * D);
    mbAct[k] = act[r];
    mbAdv[k] = adv[r];
    mbRet[k] = ret[r];
    mbOlp[k] = olp[r];
  }
}

/* normalizeAdv (Puffer/RL/NNTrain.lean:274-279): sequential folds, population std, +1e-8. */
void orc_normalize_adv(const double* adv, size_t n, double* out) {
  double dn = (double)n;
  double s = 0.0;
  for (size_t i = 0; i < n; i++) s = s + adv[i];
  double mean = s / dn;
  double v = 0.0;
  for (size_t i = 0; i < n; i++) v = v + (adv[i] - mean) * (adv[i] - mean);
  double std = sqrt(v / dn);
  for (size_t i = 0; i < n; i++) out[i] = (adv[i] - mean) / (std + 1e-8);
}

/* ---------------------------------------------------------------- Muon --------------------- */
/* PufferLib's tuned 5-row quintic schedule (Puffer/Float/Muon.lean:64-67). */
const double ORC_MUON_COEFFS[5][3] = {{4.0848, -6.8946, 2.9270}, {3.9505, -6.3029, 2.6377},
                                      {3.7418, -5.5913, 2.3037}, {2.8769, -3.1427, 1.2046},
                                      {2.8366, -3.0525, 1.2012}};

/* matmul (Puffer/Float/Muon.lean:19-31): C[i][j] = fold_l s + A[i][l]*B[l][j] from 0.0. */
static void orc_matmul(const double* A, const double* B, int m, int k, int n, double* C) {
  for (int i = 0; i < m; i++)
    for (int j = 0; j < n; j++) {
      double s = 0.0;
      for (int l = 0; l < k; l++) s = s + A[(long)i * k + l] * B[(long)l * n + j];
      C[(long)i * n + j] = s;
    }
}
static void orc_transpose(const double* X, int rows, int cols, double* Xt) {
  for (int i = 0; i < rows; i++)
    for (int j = 0; j < cols; j++) Xt[(long)j * rows + i] = X[(long)i * cols + j];
}
/* frobNorm (Puffer/Float/Muon.lean:45-46): two-level fold (per-row sum of squares, then rows). */
double orc_frob_norm(const double* X, int rows, int cols) {
  double s = 0.0;
  for (int i = 0; i < rows; i++) {
    double rs = 0.0;
    for (int j = 0; j < cols; j++) {
      double x = X[(long)i * cols + j];
      rs = rs + x * x;
    }
    s = s + rs;
  }
  return sqrt(s);
}

/* newtonSchulzWith (Puffer/Float/Muon.lean:74-90) over an arbitrary `iters` x 3 coefficient table:
 * X = X0 / (frob + eps); per row (a,b,c): rows<=cols: A=X X^T, AX, A(AX); else A=X^T X, XA, (XA)A;
 * X = a X + b (AX|XA) + c (AAX|XAA). */
void orc_newton_schulz(const double* X0, int rows, int cols, double eps, const double* coeffs, int iters,
                       double* Xout) {
  long n = (long)rows * cols;
  int mn = rows < cols ? rows : cols;
  double* Xt = (double*)malloc(sizeof(double) * n);
  double* A = (double*)malloc(sizeof(double) * (long)mn * mn);
  double* P = (double*)malloc(sizeof(double) * n);
  double* Q = (double*)malloc(sizeof(double) * n);
  double inv = 1.0 / (orc_frob_norm(X0, rows, cols) + eps);
  for (long i = 0; i < n; i++) Xout[i] = inv * X0[i];
  for (int it = 0; it < iters; it++) {
    double a = coeffs[3 * it + 0], b = coeffs[3 * it + 1], c = coeffs[3 * it + 2];
    orc_transpose(Xout, rows, cols, Xt);
    if (rows <= cols) {
      orc_matmul(Xout, Xt, rows, cols, rows, A);
      orc_matmul(A, Xout, rows, rows, cols, P);
      orc_matmul(A, P, rows, rows, cols, Q);
    } else {
      orc_matmul(Xt, Xout, cols, rows, cols, A);
      orc_matmul(Xout, A, rows, cols, cols, P);
      orc_matmul(P, A, rows, cols, cols, Q);
    }
    for (long i = 0; i < n; i++) Xout[i] = a * Xout[i] + b * P[i] + c * Q[i];
  }
  free(Xt);
  free(A);
  free(P);
  free(Q);
}

/* stepMat (Puffer/Float/Muon.lean:94-102): newMom = mu*mom + 1*g; upd = 1*g + mu*newMom;
 * W' = (1 - lr*wd) W + (lr*sqrt(max(1, rows/cols))) NS(upd)   (ascent form). */
void orc_muon_stepmat(const double* W, const double* G, const double* M, int rows, int cols, double lr, double wd,
                      double mu, double eps, const double* coeffs, int iters, double* nW, double* nM) {
  long n = (long)rows * cols;
  double* u = (double*)malloc(sizeof(double) * n);
  double* X = (double*)malloc(sizeof(double) * n);
  for (long i = 0; i < n; i++) {
    nM[i] = mu * M[i] + 1.0 * G[i];
    u[i] = 1.0 * G[i] + mu * nM[i];
  }
  orc_newton_schulz(u, rows, cols, eps, coeffs, iters, X);
  double r = (double)rows / (double)cols;
  double scale = sqrt(1.0 <= r ? r : 1.0);
  double c1 = 1.0 - lr * wd, c2 = lr * scale;
  for (long i = 0; i < n; i++) nW[i] = c1 * W[i] + c2 * X[i];
  free(u);
  free(X);
}

/* stepVec (Puffer/Float/Muon.lean:105-108). */
void orc_muon_stepvec(const double* b, const double* g, const double* m, int n, double lr, double wd, double mu,
                      double* nb, double* nm) {
  for (int i = 0; i < n; i++) {
    double newm = mu * m[i] + g[i];
    double upd = g[i] + mu * newm;
    nb[i] = b[i] * (1.0 - lr * wd) + lr * upd;
    nm[i] = newm;
  }
}

/* ---------------------------------------------------------------- MLP PPO gradient --------- */
/* Activation of the hidden layers: 0 = ReLU (every reference MLP kernel, ffi/pufferblas.c:721),
 * 1 = GELU tanh form 0.5 x (1 + tanh(0.7978845608028654 (x + 0.044715 x^3))) (Puffer/Net/Forward.lean:271-273). */
static double orc_act(double z, int act) {
  if (act == 0) return z > 0.0 ? z : 0.0;
  double u = 0.7978845608028654 * (z + 0.044715 * z * z * z);
  return 0.5 * z * (1.0 + tanh(u));
}
static double orc_act_grad(double z, int act) {
  if (act == 0) return z > 0.0 ? 1.0 : 0.0;
  double u = 0.7978845608028654 * (z + 0.044715 * z * z * z);
  double t = tanh(u);
  return 0.5 * (1.0 + t) + 0.5 * z * (1.0 - t * t) * 0.7978845608028654 * (1.0 + 3.0 * 0.044715 * z * z);
}

/* Parameter count of the flat layout [W1(H*D)|b1(H)|{W_l(H*H)|b_l(H)} for l=2..L|Wo(O*H)|bo(O)];
 * L = 1 is the reference's [W1|b1|W2|b2] (ffi/puffercuda.cu:746, Puffer/RL/FFITrain.lean:136). */
size_t orc_mlp_param_count(size_t D, size_t H, size_t A, size_t L) {
  size_t O = A + 1;
  return H * D + H + (L - 1) * (H * H + H) + O * H + O;
}

/* Summed PPO-objective gradient over N rows (gradient ASCENT convention), generalised to L hidden
 * layers. Per row it is the reference's scalar backward: forward, log-softmax WITHOUT max subtraction,
 * ratio = exp(logp_a - old), clipped surrogate branch choice, entropy term, value term with optional
 * PufferLib value clip (ffi/pufferffi.c:87-140 and :142-208; ffi/pufferblas.c:699-747).
 * ov == NULL or vfClip <= 0 selects the unclipped value gradient. newlp/newval may be NULL. */
void orc_mlp_ppo_grad(const double* params, const double* obs, const double* acts, const double* advs,
                      const double* rets, const double* olps, const double* ov, size_t N, size_t D, size_t H,
                      size_t A, size_t L, int act, double vfCoef, double entCoef, double clipEps, double vfClip,
                      double* g, double* newlp, double* newval) {
  size_t O = A + 1;
  size_t P = orc_mlp_param_count(D, H, A, L);
  for (size_t i = 0; i < P; i++) g[i] = 0.0;
  /* layer offsets */
  size_t* oW = (size_t*)malloc(sizeof(size_t) * (L + 1));
  size_t* ob = (size_t*)malloc(sizeof(size_t) * (L + 1));
  size_t off = 0;
  for (size_t l = 0; l <= L; l++) {
    size_t in = (l == 0) ? D : H, outd = (l == L) ? O : H;
    oW[l] = off;
    off += outd * in;
    ob[l] = off;
    off += outd;
  }
  double* z = (double*)malloc(sizeof(double) * L * H);
  double* h = (double*)malloc(sizeof(double) * L * H);
  double* out = (double*)malloc(sizeof(double) * O);
  double* dout = (double*)malloc(sizeof(double) * O);
  double* dh = (double*)malloc(sizeof(double) * H);
  double* dz = (double*)malloc(sizeof(double) * H);
  double* pk = (double*)malloc(sizeof(double) * (A ? A : 1));
  for (size_t n = 0; n < N; n++) {
    const double* x = obs + n * D;
    /* forward */
    for (size_t l = 0; l < L; l++) {
      const double* in = (l == 0) ? x : h + (l - 1) * H;
      size_t nin = (l == 0) ? D : H;
      for (size_t j = 0; j < H; j++) {
        const double* w = params + oW[l] + j * nin;
        double acc = 0.0;
        for (size_t k = 0; k < nin; k++) acc += w[k] * in[k];
        double zz = params[ob[l] + j] + acc;
        z[l * H + j] = zz;
        h[l * H + j] = orc_act(zz, act);
      }
    }
    const double* hl = h + (L - 1) * H;
    for (size_t k = 0; k < O; k++) {
      const double* w = params + oW[L] + k * H;
      double acc = 0.0;
      for (size_t j = 0; j < H; j++) acc += w[j] * hl[j];
      out[k] = params[ob[L] + k] + acc;
    }
    /* PPO objective backward */
    size_t a = (size_t)acts[n];
    double adv = advs[n], ret = rets[n], oldLogp = olps[n];
    double sumexp = 0.0;
    for (size_t k = 0; k < A; k++) sumexp += exp(out[k]);
    double lse = log(sumexp);
    double pout = 0.0;
    for (size_t k = 0; k < A; k++) {
      pk[k] = exp(out[k] - lse);
      pout += pk[k] * out[k];
    }
    double logpA = out[a] - lse;
    double ratio = exp(logpA - oldLogp);
    double lo = 1.0 - clipEps, hi = 1.0 + clipEps;
    double ratioC = ratio < lo ? lo : (ratio > hi ? hi : ratio);
    double surr1 = adv * ratio, surr2 = adv * ratioC;
    double dPol;
    if (surr1 <= surr2)
      dPol = adv * ratio;
    else {
      double cg = (lo < ratio && ratio < hi) ? 1.0 : 0.0;
      dPol = adv * cg * ratio;
    }
    for (size_t k = 0; k < A; k++) {
      double dp = dPol * (((k == a) ? 1.0 : 0.0) - pk[k]);
      double de = entCoef * pk[k] * (pout - out[k]);
      dout[k] = dp + de;
    }
    double vnew = out[A], dv;
    if (ov && vfClip > 0.0) {
      double vold = ov[n], d = vnew - vold;
      double vclip = vold + (d < -vfClip ? -vfClip : (d > vfClip ? vfClip : d));
      double du = (vnew - ret) * (vnew - ret), dc = (vclip - ret) * (vclip - ret);
      if (du >= dc)
        dv = vnew - ret;
      else if (d > -vfClip && d < vfClip)
        dv = vnew - ret;
      else
        dv = 0.0;
    } else
      dv = vnew - ret;
    dout[A] = -vfCoef * dv;
    if (newlp) newlp[n] = logpA;
    if (newval) newval[n] = vnew;
    /* backward: head */
    for (size_t j = 0; j < H; j++) dh[j] = 0.0;
    for (size_t k = 0; k < O; k++) {
      double dk = dout[k];
      double* gw = g + oW[L] + k * H;
      const double* w = params + oW[L] + k * H;
      for (size_t j = 0; j < H; j++) {
        gw[j] += dk * hl[j];
        dh[j] += dk * w[j];
      }
      g[ob[L] + k] += dk;
    }
    /* hidden layers, top to bottom */
    for (size_t l = L; l-- > 0;) {
      const double* in = (l == 0) ? x : h + (l - 1) * H;
      size_t nin = (l == 0) ? D : H;
      for (size_t j = 0; j < H; j++) dz[j] = dh[j] * orc_act_grad(z[l * H + j], act);
      if (act == 0)
        for (size_t j = 0; j < H; j++) dz[j] = (z[l * H + j] > 0.0) ? dh[j] : 0.0;
      for (size_t j = 0; j < nin && l > 0; j++) dh[j] = 0.0;
      for (size_t j = 0; j < H; j++) {
        double* gw = g + oW[l] + j * nin;
        const double* w = params + oW[l] + j * nin;
        for (size_t k = 0; k < nin; k++) {
          gw[k] += dz[j] * in[k];
          if (l > 0) dh[k] += dz[j] * w[k];
        }
        g[ob[l] + j] += dz[j];
      }
    }
  }
  free(oW);
  free(ob);
  free(z);
  free(h);
  free(out);
  free(dout);
  free(dh);
  free(dz);
  free(pk);
}

/* Global-norm clip of a summed gradient to the clipped MEAN gradient (the resident drivers' formula,
 * ffi/puffercuda.cu:5122-5131 / Puffer/RL/MinGRUTrain.lean:640-648): gnorm = sqrt(sum (g*sc)^2),
 * cc = (maxNorm > 0 && gnorm > maxNorm ? maxNorm/gnorm : 1) * sc, g *= cc. maxNorm <= 0 is the bare
 * mean scale g *= sc. Sequential fold. */
void orc_grad_clip(double* g, size_t P, double maxNorm, double sc) {
  if (maxNorm > 0.0) {
    double ss = 0.0;
    for (size_t i = 0; i < P; i++) {
      double x = g[i] * sc;
      ss = ss + x * x;
    }
    double gnorm = sqrt(ss);
    double cc = ((maxNorm > 0.0 && gnorm > maxNorm) ? maxNorm / gnorm : 1.0) * sc;
    for (size_t i = 0; i < P; i++) g[i] = g[i] * cc;
  } else {
    for (size_t i = 0; i < P; i++) g[i] = sc * g[i];
  }
}

/* Muon over the whole flat MLP: every weight matrix via stepMat, every bias via stepVec, in layer order
 * (applyMuon, Puffer/RL/NNTrain.lean:379-388, generalised to L hidden layers). pm = [params(P); mom(P)]
 * updated in place; g is the already-scaled gradient. */
void orc_apply_muon(double* pm, const double* g, size_t D, size_t H, size_t A, size_t L, double lr, double wd,
                    double mu, double eps, const double* coeffs, int iters) {
  size_t O = A + 1;
  size_t P = orc_mlp_param_count(D, H, A, L);
  double* par = pm;
  double* mom = pm + P;
  size_t off = 0;
  for (size_t l = 0; l <= L; l++) {
    size_t in = (l == 0) ? D : H, outd = (l == L) ? O : H;
    size_t n = outd * in;
    double* nW = (double*)malloc(sizeof(double) * n);
    double* nM = (double*)malloc(sizeof(double) * n);
    orc_muon_stepmat(par + off, g + off, mom + off, (int)outd, (int)in, lr, wd, mu, eps, coeffs, iters, nW, nM);
    memcpy(par + off, nW, sizeof(double) * n);
    memcpy(mom + off, nM, sizeof(double) * n);
    free(nW);
    free(nM);
    off += n;
    orc_muon_stepvec(par + off, g + off, mom + off, (int)outd, lr, wd, mu, par + off, mom + off);
    off += outd;
  }
}

/* One whole update over resident columns (the semantics of lean_cuda_train_update_resident,
 * ffi/puffercuda.cu:1187-1294, generalised to L hidden layers): for each epoch e and minibatch m,
 * rows perm[e*NT + lo .. hi) with mbSize = NT/numMB and the last minibatch taking the remainder;
 * gather, normalizeAdv over the minibatch, summed gradient, clip to the mean, Muon in place.
 * ov may be NULL (unclipped value loss). pm = [params; mom] updated in place. */
void orc_train_update(double* pm, const double* obs, const double* acts, const double* adv, const double* ret,
                      const double* olp, const double* ov, const double* perm, size_t NT, size_t D, size_t H,
                      size_t A, size_t L, int act, size_t epochs, size_t numMB, double lr, double wd, double mu,
                      double eps, double vfCoef, double entCoef, double clipEps, double vfClip, double maxGradNorm,
                      const double* coeffs, int iters) {
  size_t P = orc_mlp_param_count(D, H, A, L);
  size_t mbSize = NT / numMB;
  if (mbSize < 1) mbSize = 1;
  double* mbObs = (double*)malloc(sizeof(double) * NT * D);
  double* mbAct = (double*)malloc(sizeof(double) * NT);
  double* mbAdv = (double*)malloc(sizeof(double) * NT);
  double* mbAdvN = (double*)malloc(sizeof(double) * NT);
  double* mbRet = (double*)malloc(sizeof(double) * NT);
  double* mbOlp = (double*)malloc(sizeof(double) * NT);
  double* mbOv = (double*)malloc(sizeof(double) * NT);
  double* g = (double*)malloc(sizeof(double) * P);
  int useVClip = (ov != NULL && vfClip > 0.0);
  for (size_t e = 0; e < epochs; e++)
    for (size_t m = 0; m < numMB; m++) {
      size_t lo = m * mbSize;
      size_t hi = (m + 1 == numMB) ? NT : (m + 1) * mbSize;
      if (hi > NT) hi = NT;
      if (hi <= lo) continue;
      size_t Nmb = hi - lo;
      const double* idx = perm + e * NT + lo;
      orc_gather_minibatch(obs, acts, adv, ret, olp, idx, Nmb, D, mbObs, mbAct, mbAdv, mbRet, mbOlp);
      if (useVClip)
        for (size_t k = 0; k < Nmb; k++) mbOv[k] = ov[(size_t)idx[k]];
      orc_normalize_adv(mbAdv, Nmb, mbAdvN);
      orc_mlp_ppo_grad(pm, mbObs, mbAct, mbAdvN, mbRet, mbOlp, useVClip ? mbOv : NULL, Nmb, D, H, A, L, act, vfCoef,
                       entCoef, clipEps, vfClip, g, NULL, NULL);
      orc_grad_clip(g, P, maxGradNorm, 1.0 / (double)Nmb);
      orc_apply_muon(pm, g, D, H, A, L, lr, wd, mu, eps, coeffs, iters);
    }
  free(mbObs);
  free(mbAct);
  free(mbAdv);
  free(mbAdvN);
  free(mbRet);
  free(mbOlp);
  free(mbOv);
  free(g);
}

/* ---------------------------------------------------------------- init --------------------- */
/* randMat (Puffer/RL/NNTrain.lean:392-403): entries uniform01*(2 scale) - scale, row-major. */
void orc_rand_mat(size_t rows, size_t cols, double scale, uint64_t* s, double* out) {
  for (size_t i = 0; i < rows * cols; i++) {
    uint64_t w = orc_rng_next(s);
    out[i] = orc_uniform01(w) * (2.0 * scale) - scale;
  }
}
/* initMLP (Puffer/RL/NNTrain.lean:418-422) flattened (flattenMLP, FFITrain.lean:136): Kaiming-uniform,
 * bound sqrt(2)/sqrt(din) for W1 and 1/sqrt(H) for W2, biases zero. Returns the advanced state. */
uint64_t orc_init_mlp(size_t din, size_t H, size_t dout, uint64_t rng, double* flat) {
  uint64_t s = rng;
  double* W1 = flat;
  double* b1 = W1 + H * din;
  double* W2 = b1 + H;
  double* b2 = W2 + dout * H;
  orc_rand_mat(H, din, sqrt(2.0) * (1.0 / sqrt((double)din)), &s, W1);
  orc_rand_mat(dout, H, 1.0 / sqrt((double)H), &s, W2);
  for (size_t j = 0; j < H; j++) b1[j] = 0.0;
  for (size_t k = 0; k < dout; k++) b2[k] = 0.0;
  return s;
}

/* cosineLr (Puffer/RL/FFITrain.lean:115-120). */
double orc_cosine_lr(double lr, double minLrRatio, size_t u, size_t updates) {
  if (u == 0) return lr;
  double lrMin = lr * minLrRatio;
  double ratio = (double)u / (double)(updates > 1 ? updates : 1);
  return lrMin + 0.5 * (lr - lrMin) * (1.0 + cos(3.14159265358979323846 * ratio));
}

/* ---------------------------------------------------------------- MinGRU -------------------- */
/* Parameter count of the flattenMG layout (Puffer/RL/MinGRUTrain.lean:282-292):
 * [wEnc(H*D) | bEnc(H) | L x layer(K*H x H) | wDec(A*H) | bDec(A) | wVal(H) | bVal(1)].
 * K = 3 is the reference's [hid | gate | proj] layer (Puffer/Net/MinGRU.lean:9-17); K = 2 drops the
 * highway projection ([hid | gate], output = the scan state). */
size_t orc_mg_param_count(size_t D, size_t H, size_t L, size_t A, size_t K) {
  return H * D + H + L * K * H * H + A * H + A + H + 1;
}

static double orc_sig(double x) { return 1.0 / (1.0 + exp(-x)); }

/* One sequence of the MinGRU PPO gradient with truncated BPTT: the reference's scalar C
 * (ffi/pufferffi.c:763-876, lean_ffi_mingru_ppo_grad_seq) op for op for K = 3 and encAct = 0,
 * generalised to K = 2 (no highway) and a GELU encoder (encAct = 1, Puffer/Net/Forward.lean:271-273).
 * Zero initial state; the state resets to zero after a terminal step and no gradient flows back across
 * it. g[P] is zeroed and receives this sequence's summed ascent gradient; newlp/newval (T each, may be
 * NULL) receive the taken action's log-prob and the value at every step. */
/* W > 1: W multi-discrete heads of sizes hs (sum A) in place of the one categorical head, actA then
 * holds W actions per step ([t*W + h]); the head follows k_mg_ppo_b_md (ffi/puffercuda.cu:4940-4980)
 * restated in f64: per head the max-subtracted softmax, the joint log-prob sum_h log(exp(x_a - m)/se),
 * one clipped ratio, per-logit gradient dPol (1[k = a_h] - p) + ent p (sum_j p_j x_j - x_k). */
void orc_mingru_grad_seq_md(const double* params, const double* obsAll, const double* actA, const double* advA,
                            const double* retA, const double* oldA, const double* termA, const double* ovA, size_t T,
                            size_t H, size_t D, size_t L, size_t A, size_t K, int encAct, double vfCoef,
                            double entCoef, double clipEps, double vfClip, size_t W, const int* hs, double* g,
                            double* newlp, double* newval) {
  const size_t wEncSz = H * D, layerSz = K * H * H;
  const size_t P = orc_mg_param_count(D, H, L, A, K);
  const double* wEnc = params;
  const double* bEnc = params + wEncSz;
  const double* layersBase = params + wEncSz + H;
  const double* wDec = layersBase + L * layerSz;
  const double* bDec = wDec + A * H;
  const double* wVal = bDec + A;
  const double* bVal = wVal + H;
  for (size_t i = 0; i < P; i++) g[i] = 0.0;
  double* gWEnc = g;
  double* gBEnc = g + wEncSz;
  double* gLayers = g + wEncSz + H;
  double* gWDec = gLayers + L * layerSz;
  double* gBDec = gWDec + A * H;
  double* gWVal = gBDec + A;
  double* gBVal = gWVal + H;
  const size_t TLH = T * L * H;
  double* hin = (double*)malloc(sizeof(double) * TLH);
  double* prevS = (double*)malloc(sizeof(double) * TLH);
  double* hidA = (double*)malloc(sizeof(double) * TLH);
  double* gateA = (double*)malloc(sizeof(double) * TLH);
  double* projA = (double*)malloc(sizeof(double) * TLH);
  double* oA = (double*)malloc(sizeof(double) * TLH);
  double* zEnc = (double*)malloc(sizeof(double) * T * H);
  double* hfin = (double*)malloc(sizeof(double) * T * H);
  double* lg = (double*)malloc(sizeof(double) * T * A);
  double* val = (double*)malloc(sizeof(double) * T);
  double* st = (double*)calloc(L * H, sizeof(double));
  double* hb = (double*)malloc(sizeof(double) * H);
  double* yb = (double*)malloc(sizeof(double) * K * H);
  double* hnew = (double*)malloc(sizeof(double) * H);
  for (size_t t = 0; t < T; t++) {
    const double* obs = obsAll + t * D;
    for (size_t i = 0; i < H; i++) {
      double acc = 0.0;
      const double* w = wEnc + i * D;
      for (size_t k = 0; k < D; k++) acc += w[k] * obs[k];
      double z = bEnc[i] + acc;
      zEnc[t * H + i] = z;
      hb[i] = encAct ? orc_act(z, 1) : z;
    }
    for (size_t l = 0; l < L; l++) {
      const double* Wl = layersBase + l * layerSz;
      size_t base = (t * L + l) * H;
      for (size_t j = 0; j < H; j++) {
        hin[base + j] = hb[j];
        prevS[base + j] = st[l * H + j];
      }
      for (size_t r = 0; r < K * H; r++) {
        double acc = 0.0;
        const double* w = Wl + r * H;
        for (size_t j = 0; j < H; j++) acc += w[j] * hb[j];
        yb[r] = acc;
      }
      for (size_t j = 0; j < H; j++) {
        double hidj = yb[j], gatej = yb[H + j], projj = K == 3 ? yb[2 * H + j] : 0.0;
        double zj = orc_sig(gatej);
        double gj = (hidj >= 0.0) ? (hidj + 0.5) : orc_sig(hidj);
        double prevj = st[l * H + j];
        double oj = (1.0 - zj) * prevj + zj * gj;
        if (K == 3) {
          double hgj = orc_sig(projj);
          hnew[j] = hgj * oj + (1.0 - hgj) * hb[j];
        } else {
          hnew[j] = oj;
        }
        hidA[base + j] = hidj;
        gateA[base + j] = gatej;
        projA[base + j] = projj;
        oA[base + j] = oj;
        st[l * H + j] = oj;
      }
      for (size_t j = 0; j < H; j++) hb[j] = hnew[j];
    }
    for (size_t j = 0; j < H; j++) hfin[t * H + j] = hb[j];
    for (size_t k = 0; k < A; k++) {
      double acc = 0.0;
      const double* w = wDec + k * H;
      for (size_t j = 0; j < H; j++) acc += w[j] * hb[j];
      lg[t * A + k] = bDec[k] + acc;
    }
    {
      double acc = 0.0;
      for (size_t j = 0; j < H; j++) acc += wVal[j] * hb[j];
      val[t] = bVal[0] + acc;
    }
    if (termA[t] != 0.0)
      for (size_t x = 0; x < L * H; x++) st[x] = 0.0;
  }
  double* dOnext = (double*)calloc(L * H, sizeof(double));
  double* dprev = (double*)malloc(sizeof(double) * L * H);
  double* dhn = (double*)malloc(sizeof(double) * H);
  double* dhin = (double*)malloc(sizeof(double) * H);
  double* dhf = (double*)malloc(sizeof(double) * H);
  double* dyh = (double*)malloc(sizeof(double) * H);
  double* dyg = (double*)malloc(sizeof(double) * H);
  double* dyp = (double*)malloc(sizeof(double) * H);
  double* pk = (double*)malloc(sizeof(double) * A);
  for (size_t tt = T; tt-- > 0;) {
    size_t t = tt;
    const double* obs = obsAll + t * D;
    const double* logits = lg + t * A;
    double adv = advA[t], ret = retA[t], oldLogp = oldA[t], vold = ovA[t];
    double logpA = 0.0, lse = 0.0, pout = 0.0;
    size_t a = 0;
    if (W <= 1) {
      double sumexp = 0.0;
      for (size_t k = 0; k < A; k++) sumexp += exp(logits[k]);
      lse = log(sumexp);
      for (size_t k = 0; k < A; k++) {
        pk[k] = exp(logits[k] - lse);
        pout += pk[k] * logits[k];
      }
      a = (size_t)actA[t];
      logpA = logits[a] - lse;
    } else {
      size_t off = 0;
      for (size_t h = 0; h < W; h++) {
        const size_t sz = (size_t)hs[h], ah = (size_t)actA[t * W + h];
        double m = logits[off];
        for (size_t k = 1; k < sz; k++)
          if (logits[off + k] > m) m = logits[off + k];
        double se = 0.0;
        for (size_t k = 0; k < sz; k++) se += exp(logits[off + k] - m);
        logpA += log(exp(logits[off + ah] - m) / se);
        off += sz;
      }
    }
    double ratio = exp(logpA - oldLogp);
    double lo = 1.0 - clipEps, hi = 1.0 + clipEps;
    double ratioC = ratio < lo ? lo : (ratio > hi ? hi : ratio);
    double surr1 = adv * ratio, surr2 = adv * ratioC;
    double dPol;
    if (surr1 <= surr2)
      dPol = adv * ratio;
    else {
      double cg = (lo < ratio && ratio < hi) ? 1.0 : 0.0;
      dPol = adv * cg * ratio;
    }
    double vnew = val[t], dvloss_dv;
    if (vfClip > 0.0) {
      double dd = vnew - vold;
      double vclip = vold + (dd < -vfClip ? -vfClip : (dd > vfClip ? vfClip : dd));
      double du = (vnew - ret) * (vnew - ret), cc = (vclip - ret) * (vclip - ret);
      if (du >= cc)
        dvloss_dv = (vnew - ret);
      else if (dd > -vfClip && dd < vfClip)
        dvloss_dv = (vnew - ret);
      else
        dvloss_dv = 0.0;
    } else {
      dvloss_dv = (vnew - ret);
    }
    double dvalue = -vfCoef * dvloss_dv;
    if (newlp) newlp[t] = logpA;
    if (newval) newval[t] = vnew;
    const double* hf = hfin + t * H;
    for (size_t j = 0; j < H; j++) dhf[j] = 0.0;
    if (W > 1) {
      /* per head: p_k and sum_j p_j x_j of that head; pk then holds the logit gradient */
      size_t off = 0;
      for (size_t h = 0; h < W; h++) {
        const size_t sz = (size_t)hs[h], ah = (size_t)actA[t * W + h];
        double m = logits[off];
        for (size_t k = 1; k < sz; k++)
          if (logits[off + k] > m) m = logits[off + k];
        double se = 0.0;
        for (size_t k = 0; k < sz; k++) se += exp(logits[off + k] - m);
        const double lh = m + log(se);
        double po = 0.0;
        for (size_t k = 0; k < sz; k++) po += exp(logits[off + k] - lh) * logits[off + k];
        for (size_t k = 0; k < sz; k++) {
          const double p = exp(logits[off + k] - lh);
          pk[off + k] = dPol * (((k == ah) ? 1.0 : 0.0) - p) + entCoef * p * (po - logits[off + k]);
        }
        off += sz;
      }
    }
    for (size_t k = 0; k < A; k++) {
      double dl = W > 1 ? pk[k] : dPol * (((k == a) ? 1.0 : 0.0) - pk[k]) + entCoef * pk[k] * (pout - logits[k]);
      double* gw = gWDec + k * H;
      const double* w = wDec + k * H;
      for (size_t j = 0; j < H; j++) {
        gw[j] += dl * hf[j];
        dhf[j] += dl * w[j];
      }
      gBDec[k] += dl;
    }
    for (size_t j = 0; j < H; j++) {
      gWVal[j] += dvalue * hf[j];
      dhf[j] += dvalue * wVal[j];
    }
    gBVal[0] += dvalue;
    for (size_t j = 0; j < H; j++) dhn[j] = dhf[j];
    for (size_t ll = L; ll-- > 0;) {
      size_t l = ll;
      size_t base = (t * L + l) * H;
      const double* Wl = layersBase + l * layerSz;
      double* Wg = gLayers + l * layerSz;
      for (size_t j = 0; j < H; j++) dhin[j] = 0.0;
      for (size_t j = 0; j < H; j++) {
        double hidj = hidA[base + j], gatej = gateA[base + j], projj = projA[base + j], oj = oA[base + j],
               prevj = prevS[base + j], hinj = hin[base + j];
        double zj = orc_sig(gatej);
        double gj = (hidj >= 0.0) ? (hidj + 0.5) : orc_sig(hidj);
        double dhnj = dhn[j];
        double do_;
        if (K == 3) {
          double hgj = orc_sig(projj);
          double dhg = dhnj * (oj - hinj);
          do_ = dhnj * hgj + dOnext[l * H + j];
          dhin[j] += dhnj * (1.0 - hgj);
          dyp[j] = dhg * hgj * (1.0 - hgj);
        } else {
          do_ = dhnj + dOnext[l * H + j];
          dyp[j] = 0.0;
        }
        double dz = do_ * (gj - prevj);
        dprev[l * H + j] = do_ * (1.0 - zj);
        double dg = do_ * zj;
        double dgate = dz * zj * (1.0 - zj);
        double sg;
        if (hidj >= 0.0)
          sg = 1.0;
        else {
          double s = orc_sig(hidj);
          sg = s * (1.0 - s);
        }
        dyh[j] = dg * sg;
        dyg[j] = dgate;
      }
      for (size_t j = 0; j < H; j++) {
        double dh_ = dyh[j];
        double* gw = Wg + j * H;
        const double* w = Wl + j * H;
        for (size_t k = 0; k < H; k++) {
          gw[k] += dh_ * hin[base + k];
          dhin[k] += dh_ * w[k];
        }
        double dga = dyg[j];
        double* gw2 = Wg + (H + j) * H;
        const double* w2 = Wl + (H + j) * H;
        for (size_t k = 0; k < H; k++) {
          gw2[k] += dga * hin[base + k];
          dhin[k] += dga * w2[k];
        }
        if (K == 3) {
          double dpr = dyp[j];
          double* gw3 = Wg + (2 * H + j) * H;
          const double* w3 = Wl + (2 * H + j) * H;
          for (size_t k = 0; k < H; k++) {
            gw3[k] += dpr * hin[base + k];
            dhin[k] += dpr * w3[k];
          }
        }
      }
      for (size_t j = 0; j < H; j++) dhn[j] = dhin[j];
    }
    for (size_t i = 0; i < H; i++) {
      double de = encAct ? dhn[i] * orc_act_grad(zEnc[t * H + i], 1) : dhn[i];
      gBEnc[i] += de;
      double* gw = gWEnc + i * D;
      for (size_t k = 0; k < D; k++) gw[k] += de * obs[k];
    }
    if (t > 0) {
      double gate_ = (termA[t - 1] == 0.0) ? 1.0 : 0.0;
      for (size_t x = 0; x < L * H; x++) dOnext[x] = dprev[x] * gate_;
    }
  }
  free(hin); free(prevS); free(hidA); free(gateA); free(projA); free(oA); free(zEnc); free(hfin); free(lg);
  free(val); free(st); free(hb); free(yb); free(hnew); free(dOnext); free(dprev); free(dhn); free(dhin);
  free(dhf); free(dyh); free(dyg); free(dyp); free(pk);
}

void orc_mingru_grad_seq(const double* params, const double* obsAll, const double* actA, const double* advA,
                         const double* retA, const double* oldA, const double* termA, const double* ovA, size_t T,
                         size_t H, size_t D, size_t L, size_t A, size_t K, int encAct, double vfCoef,
                         double entCoef, double clipEps, double vfClip, double* g, double* newlp, double* newval) {
  orc_mingru_grad_seq_md(params, obsAll, actA, advA, retA, oldA, termA, ovA, T, H, D, L, A, K, encAct, vfCoef, entCoef,
                         clipEps, vfClip, 1, NULL, g, newlp, newval);
}

/* The batched form the device kernel computes: B sequences packed time-major ([t*B + b] for the
 * scalars, [(t*B + b)*D + j] for obs; the layout of lean_cuda_mingru_ppo_grad, ffi/puffercuda.cu:5206),
 * summed over b in order 0..B-1 of the per-sequence gradients (the verify-mingru-grad-gpu check,
 * Exe/Puffer.lean:2398-2440). out = [g(P); newlp(T*B); newval(T*B)], the last two time-major. */
/* W > 1: scal = [act (W per row, [(t*B + b)*W + h]) | adv | ret | old | term | ov], (W + 5)*T*B values
 * (the packed layout of ffi/puffercuda.cu:5216-5221). */
void orc_mingru_grad_batch_md(const double* params, const double* obsTB, const double* scal, size_t B, size_t T,
                              size_t H, size_t D, size_t L, size_t A, size_t K, int encAct, double vfCoef,
                              double entCoef, double clipEps, double vfClip, size_t W, const int* hs, double* out) {
  const size_t P = orc_mg_param_count(D, H, L, A, K), nb = T * B, Wa = W < 1 ? 1 : W;
  double* gb = (double*)malloc(sizeof(double) * P);
  double* so = (double*)malloc(sizeof(double) * T * D);
  double* sc = (double*)malloc(sizeof(double) * (Wa + 5) * T);
  double* nl = (double*)malloc(sizeof(double) * T);
  double* nv = (double*)malloc(sizeof(double) * T);
  for (size_t i = 0; i < P; i++) out[i] = 0.0;
  for (size_t b = 0; b < B; b++) {
    for (size_t t = 0; t < T; t++) {
      for (size_t j = 0; j < D; j++) so[t * D + j] = obsTB[(t * B + b) * D + j];
      for (size_t h = 0; h < Wa; h++) sc[t * Wa + h] = scal[(t * B + b) * Wa + h];
      for (size_t q = 1; q < 6; q++) sc[(Wa + q - 1) * T + t] = scal[(Wa + q - 1) * nb + t * B + b];
    }
    const double* s1 = sc + Wa * T;
    orc_mingru_grad_seq_md(params, so, sc, s1, s1 + T, s1 + 2 * T, s1 + 3 * T, s1 + 4 * T, T, H, D, L, A, K, encAct,
                           vfCoef, entCoef, clipEps, vfClip, Wa, hs, gb, nl, nv);
    for (size_t i = 0; i < P; i++) out[i] = out[i] + gb[i];
    for (size_t t = 0; t < T; t++) {
      out[P + t * B + b] = nl[t];
      out[P + nb + t * B + b] = nv[t];
    }
  }
  free(gb); free(so); free(sc); free(nl); free(nv);
}
void orc_mingru_grad_batch(const double* params, const double* obsTB, const double* scal, size_t B, size_t T,
                           size_t H, size_t D, size_t L, size_t A, size_t K, int encAct, double vfCoef,
                           double entCoef, double clipEps, double vfClip, double* out) {
  orc_mingru_grad_batch_md(params, obsTB, scal, B, T, H, D, L, A, K, encAct, vfCoef, entCoef, clipEps, vfClip, 1, NULL,
                           out);
}

/* Prioritised segment sampling (ffi/pufferffi.c:1094-1125, lean_ffi_prio_sample):
 * w_e = exp(alpha log(L1_e + 1e-12)), p_e = (w_e + 1e-6)/(sum w + 1e-6), cum = prefix sum (sequential),
 * draw i: u = uniform01(splitmix64(rng + (i+1) GOLD)) * total, idx = first e with cum_e >= u,
 * mbPrio_i = exp(-beta log(N p_idx + 1e-12)). segIdx is written as doubles. */
void orc_prio_sample(const double* advL1, size_t N, size_t mbSegs, double prioAlpha, double annealBeta,
                     uint64_t rng, double* idxArr, double* mpArr) {
  double* prioW = (double*)malloc(N * sizeof(double));
  double* prioProbs = (double*)malloc(N * sizeof(double));
  double* cum = (double*)malloc(N * sizeof(double));
  double sumW = 0.0;
  for (size_t e = 0; e < N; e++) {
    double w = exp(prioAlpha * log(advL1[e] + 1e-12));
    prioW[e] = w;
    sumW += w;
  }
  double denom = sumW + 1e-6, acc = 0.0;
  for (size_t e = 0; e < N; e++) {
    double p = (prioW[e] + 1e-6) / denom;
    prioProbs[e] = p;
    acc += p;
    cum[e] = acc;
  }
  double total = acc;
  for (size_t i = 0; i < mbSegs; i++) {
    uint64_t z = rng + (uint64_t)(i + 1) * ORC_GOLD;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    z = z ^ (z >> 31);
    double u = (double)(z >> 11) / 9007199254740992.0 * total;
    size_t lo = 0, hi = N;
    while (lo < hi) {
      size_t mid = (lo + hi) >> 1;
      if (cum[mid] >= u)
        hi = mid;
      else
        lo = mid + 1;
    }
    size_t idx = (lo < N) ? lo : (N - 1);
    idxArr[i] = (double)idx;
    mpArr[i] = exp((-annealBeta) * log((double)N * prioProbs[idx] + 1e-12));
  }
  free(prioW);
  free(prioProbs);
  free(cum);
}

/* MinGRU minibatch scalar gather (ffi/pufferffi.c:1137-1176, lean_ffi_gather_seq_minibatch):
 * advMean / advStd over the Bmb*T sampled advantages (bi outer, t inner, population std), then for
 * os = t*Bmb + bi, si = seg[bi]*T + t: act = (double)(u64)act[si], adv = mbPrio[bi]*(a - mean)/(std + 1e-8),
 * ret = a + v, old = logp[si], term = term[si] > 0.5, ov = v. out = [act|adv|ret|old|term|ov] (6 * T * Bmb). */
/* W > 1: actCol holds W actions per row ([(e*T + t)*W + h]) and the act block of out is W wide
 * ([os*W + h]); out = (W + 5)*T*Bmb values. */
void orc_gather_seq_minibatch_md(const double* actCol, const double* logpCol, const double* termCol,
                                 const double* advFlat, const double* valueBuf, const double* segIdx,
                                 const double* mbPrio, size_t T, size_t Bmb, size_t W, double* out) {
  size_t nb = T * Bmb, Wa = W < 1 ? 1 : W;
  double navd = (double)(nb > 0 ? nb : 1), sum = 0.0;
  for (size_t bi = 0; bi < Bmb; bi++) {
    size_t e = (size_t)segIdx[bi];
    const double* ab = advFlat + e * T;
    for (size_t t = 0; t < T; t++) sum += ab[t];
  }
  double advMean = sum / navd, sq = 0.0;
  for (size_t bi = 0; bi < Bmb; bi++) {
    size_t e = (size_t)segIdx[bi];
    const double* ab = advFlat + e * T;
    for (size_t t = 0; t < T; t++) {
      double d = ab[t] - advMean;
      sq += d * d;
    }
  }
  double advStd = sqrt(sq / navd);
  double* pact = out;
  double* padv = out + Wa * nb;
  double* pret = out + (Wa + 1) * nb;
  double* pold = out + (Wa + 2) * nb;
  double* pterm = out + (Wa + 3) * nb;
  double* pov = out + (Wa + 4) * nb;
  double stde = advStd + 1e-8;
  for (size_t bi = 0; bi < Bmb; bi++) {
    size_t e = (size_t)segIdx[bi];
    double mp = mbPrio[bi];
    for (size_t t = 0; t < T; t++) {
      size_t si = e * T + t, os = t * Bmb + bi;
      double a = advFlat[si], v = valueBuf[si];
      for (size_t h = 0; h < Wa; h++) pact[os * Wa + h] = (double)(unsigned long long)actCol[si * Wa + h];
      padv[os] = mp * (a - advMean) / stde;
      pret[os] = a + v;
      pold[os] = logpCol[si];
      pov[os] = v;
      pterm[os] = termCol[si] > 0.5 ? 1.0 : 0.0;
    }
  }
}
void orc_gather_seq_minibatch(const double* actCol, const double* logpCol, const double* termCol,
                              const double* advFlat, const double* valueBuf, const double* segIdx,
                              const double* mbPrio, size_t T, size_t Bmb, double* out) {
  orc_gather_seq_minibatch_md(actCol, logpCol, termCol, advFlat, valueBuf, segIdx, mbPrio, T, Bmb, 1, out);
}

/* applyMuonMG (Puffer/RL/MinGRUTrain.lean:265-279): stepMat on wEnc, every layer, wDec and wVal; stepVec
 * on bEnc, bDec, bVal. pm = [params(P); mom(P)] in the flattenMG layout, updated in place; g is the
 * already-clipped gradient. */
void orc_apply_muon_mg(double* pm, const double* g, size_t D, size_t H, size_t L, size_t A, size_t K, double lr,
                       double wd, double mu, double eps, const double* coeffs, int iters) {
  size_t P = orc_mg_param_count(D, H, L, A, K);
  double* par = pm;
  double* mom = pm + P;
  size_t off = 0;
  size_t nmat = L + 3;
  for (size_t q = 0; q <= nmat; q++) {
    size_t rows, cols, bias;
    if (q == 0) { rows = H; cols = D; bias = H; }
    else if (q <= L) { rows = K * H; cols = H; bias = 0; }
    else if (q == L + 1) { rows = A; cols = H; bias = A; }
    else if (q == L + 2) { rows = 1; cols = H; bias = 1; }
    else break;
    size_t n = rows * cols;
    double* nW = (double*)malloc(sizeof(double) * n);
    double* nM = (double*)malloc(sizeof(double) * n);
    orc_muon_stepmat(par + off, g + off, mom + off, (int)rows, (int)cols, lr, wd, mu, eps, coeffs, iters, nW, nM);
    memcpy(par + off, nW, sizeof(double) * n);
    memcpy(mom + off, nM, sizeof(double) * n);
    free(nW);
    free(nM);
    off += n;
    if (bias) {
      orc_muon_stepvec(par + off, g + off, mom + off, (int)bias, lr, wd, mu, par + off, mom + off);
      off += bias;
    }
  }
}

/* One MinGRU update over the rollout columns (the per-minibatch chain of Puffer/RL/MinGRUTrain.lean:800-850
 * with the device-resident prep of ffi/puffercuda.cu:316-507): value := val0, ratio := 1; then per
 * minibatch: V-trace (MinGRU form, bootstrap boot) with the live ratio/value buffers -> adv, sum |adv| per
 * segment -> prioritised sampling (rng advances by mbSegs*GOLD) -> scalar gather + obs sequences ->
 * summed BPTT gradient over the sampled segments -> value/ratio iterate (the last sampler of a segment
 * writes) -> gradClipMG with sc = 1/(Bmb*T) -> applyMuonMG. Columns are rows e*T + t; obs is
 * [(e*T + t)*D + j]. pm = [params; mom] updated in place. Returns the advanced rng. */
/* W > 1: act holds W actions per row and the heads are the multi-discrete ones of sizes hs. */
uint64_t orc_mingru_update_md(double* pm, const double* obs, const double* rew, const double* term, const double* act,
                              const double* logp, const double* val0, const double* boot, size_t N, size_t T,
                              size_t D, size_t H, size_t L, size_t A, size_t K, int encAct, size_t numMB,
                              size_t mbSegs, double gamma, double lam, double rhoClip, double cClip, double prioAlpha,
                              double annealBeta, uint64_t rng, double lr, double wd, double mu, double eps,
                              double vfCoef, double entCoef, double clipEps, double vfClip, double maxGradNorm,
                              const double* coeffs, int iters, size_t W, const int* hs) {
  const size_t NT = N * T, P = orc_mg_param_count(D, H, L, A, K), Wa = W < 1 ? 1 : W;
  double* value = (double*)malloc(sizeof(double) * NT);
  double* ratio = (double*)malloc(sizeof(double) * NT);
  double* adv = (double*)malloc(sizeof(double) * NT);
  double* l1 = (double*)malloc(sizeof(double) * N);
  double* seg = (double*)malloc(sizeof(double) * mbSegs);
  double* mp = (double*)malloc(sizeof(double) * mbSegs);
  double* sc = (double*)malloc(sizeof(double) * (Wa + 5) * T * mbSegs);
  double* obsTB = (double*)malloc(sizeof(double) * T * mbSegs * D);
  double* gout = (double*)malloc(sizeof(double) * (P + 2 * T * mbSegs));
  memcpy(value, val0, sizeof(double) * NT);
  for (size_t i = 0; i < NT; i++) ratio[i] = 1.0;
  for (size_t mb = 0; mb < numMB; mb++) {
    orc_vtrace_mingru(rew, value, term, ratio, boot, N, T, gamma, lam, rhoClip, cClip, adv);
    orc_adv_l1(adv, N, T, l1);
    orc_prio_sample(l1, N, mbSegs, prioAlpha, annealBeta, rng, seg, mp);
    rng += (uint64_t)mbSegs * ORC_GOLD;
    orc_gather_seq_minibatch_md(act, logp, term, adv, value, seg, mp, T, mbSegs, Wa, sc);
    for (size_t t = 0; t < T; t++)
      for (size_t b = 0; b < mbSegs; b++) {
        size_t e = (size_t)seg[b];
        memcpy(obsTB + (t * mbSegs + b) * D, obs + (e * T + t) * D, sizeof(double) * D);
      }
    orc_mingru_grad_batch_md(pm, obsTB, sc, mbSegs, T, H, D, L, A, K, encAct, vfCoef, entCoef, clipEps, vfClip, Wa, hs,
                             gout);
    for (size_t b = 0; b < mbSegs; b++) {
      size_t e = (size_t)seg[b];
      for (size_t t = 0; t < T; t++) {
        size_t si = e * T + t, os = t * mbSegs + b;
        ratio[si] = exp(gout[P + os] - logp[si]);
        value[si] = gout[P + T * mbSegs + os];
      }
    }
    orc_grad_clip(gout, P, maxGradNorm, 1.0 / (double)(mbSegs * T));
    orc_apply_muon_mg(pm, gout, D, H, L, A, K, lr, wd, mu, eps, coeffs, iters);
  }
  free(value); free(ratio); free(adv); free(l1); free(seg); free(mp); free(sc); free(obsTB); free(gout);
  return rng;
}
uint64_t orc_mingru_update(double* pm, const double* obs, const double* rew, const double* term, const double* act,
                           const double* logp, const double* val0, const double* boot, size_t N, size_t T,
                           size_t D, size_t H, size_t L, size_t A, size_t K, int encAct, size_t numMB,
                           size_t mbSegs, double gamma, double lam, double rhoClip, double cClip, double prioAlpha,
                           double annealBeta, uint64_t rng, double lr, double wd, double mu, double eps,
                           double vfCoef, double entCoef, double clipEps, double vfClip, double maxGradNorm,
                           const double* coeffs, int iters) {
  return orc_mingru_update_md(pm, obs, rew, term, act, logp, val0, boot, N, T, D, H, L, A, K, encAct, numMB, mbSegs,
                              gamma, lam, rhoClip, cClip, prioAlpha, annealBeta, rng, lr, wd, mu, eps, vfCoef, entCoef,
                              clipEps, vfClip, maxGradNorm, coeffs, iters, 1, NULL);
}

/* initMinGRU (Puffer/RL/MinGRUTrain.lean:311-344) flattened: wEnc bound sqrt(2)/sqrt(D), layers
 * (K*H x H each) 1/sqrt(H), wDec and wVal 1/sqrt(H), biases zero. Returns the advanced state. */
uint64_t orc_init_mingru(size_t D, size_t H, size_t L, size_t A, size_t K, uint64_t rng, double* flat) {
  uint64_t s = rng;
  double* p = flat;
  orc_rand_mat(H, D, sqrt(2.0) * (1.0 / sqrt((double)D)), &s, p);
  p += H * D;
  for (size_t j = 0; j < H; j++) p[j] = 0.0;
  p += H;
  for (size_t l = 0; l < L; l++) {
    orc_rand_mat(K * H, H, 1.0 / sqrt((double)H), &s, p);
    p += K * H * H;
  }
  double* wDec = p;
  p += A * H;
  double* bDec = p;
  p += A;
  double* wVal = p;
  p += H;
  orc_rand_mat(A, H, 1.0 / sqrt((double)H), &s, wDec);
  orc_rand_mat(1, H, 1.0 / sqrt((double)H), &s, wVal);
  for (size_t k = 0; k < A; k++) bDec[k] = 0.0;
  p[0] = 0.0;
  return s;
}

/* ---------------------------------------------------------------- wide action heads --------- */
/* Summed PPO-objective gradient of the one-hidden-layer ReLU MLP with a wide head (ascent convention):
 * mode 1 = W categorical heads of sizes hs[0..W) (joint log-prob of log-softmax WITHOUT max subtraction,
 * one clip on the joint ratio; ffi/puffercuda.cu:706-727, restated in f64), mode 2 = W Gaussian dims
 * (out = [means | raw log-stds clamped to [lsLo, 2] | value]; ffi/pufferffi.c:311-360 op for op, whose
 * forward accumulates the dot products from the last index down, gauss_forward :233-237). acts is
 * N x W. ov == NULL or vfClip <= 0: unclipped value gradient. g[P] is zeroed; newlp/newval may be NULL. */
void orc_mlp_ppo_grad_wide(const double* params, const double* obs, const double* acts, const double* advs,
                           const double* rets, const double* olps, const double* ov, size_t N, size_t D, size_t H,
                           size_t O, size_t W, int mode, const int* hs, double vfCoef, double entCoef, double clipEps,
                           double vfClip, double lsLo, double* g, double* newlp, double* newval) {
  const double lsHi = 2.0;
  const size_t P = H * D + H + O * H + O;
  const double* W1 = params;
  const double* b1 = params + H * D;
  const double* W2 = params + H * D + H;
  const double* b2 = params + H * D + H + O * H;
  for (size_t i = 0; i < P; i++) g[i] = 0.0;
  double* gW1 = g;
  double* gb1 = g + H * D;
  double* gW2 = g + H * D + H;
  double* gb2 = g + H * D + H + O * H;
  double* z1 = (double*)malloc(sizeof(double) * H);
  double* h = (double*)malloc(sizeof(double) * H);
  double* out = (double*)malloc(sizeof(double) * O);
  double* dout = (double*)malloc(sizeof(double) * O);
  double* dh = (double*)malloc(sizeof(double) * H);
  const double halfLog2pi = 0.5 * log(2.0 * 3.14159265358979323846);
  for (size_t n = 0; n < N; n++) {
    const double* x = obs + n * D;
    const double* act = acts + n * W;
    for (size_t j = 0; j < H; j++) {
      const double* w = W1 + j * D;
      double acc = 0.0;
      for (size_t k = D; k-- > 0;) acc = w[k] * x[k] + acc;
      double z = b1[j] + acc;
      z1[j] = z;
      h[j] = z > 0.0 ? z : 0.0;
    }
    for (size_t k = 0; k < O; k++) {
      const double* w = W2 + k * H;
      double acc = 0.0;
      for (size_t j = H; j-- > 0;) acc = w[j] * h[j] + acc;
      out[k] = b2[k] + acc;
    }
    double adv = advs[n], ret = rets[n], oldLogp = olps[n];
    double logp = 0.0;
    if (mode == 1) {
      size_t off = 0;
      for (size_t hh = 0; hh < W; hh++) {
        double se = 0.0;
        for (int k = 0; k < hs[hh]; k++) se += exp(out[off + k]);
        logp += out[off + (size_t)act[hh]] - log(se);
        off += hs[hh];
      }
    } else {
      for (size_t i = 0; i < W; i++) {
        double ls = out[W + i];
        ls = ls < lsLo ? lsLo : (ls > lsHi ? lsHi : ls);
        double invStd = exp(-ls);
        double z = (act[i] - out[i]) * invStd;
        logp += -0.5 * z * z - ls - halfLog2pi;
      }
    }
    double ratio = exp(logp - oldLogp);
    double lo = 1.0 - clipEps, hi = 1.0 + clipEps;
    double ratioC = ratio < lo ? lo : (ratio > hi ? hi : ratio);
    double surr1 = adv * ratio, surr2 = adv * ratioC;
    double dPol;
    if (surr1 <= surr2)
      dPol = adv * ratio;
    else {
      double cg = (lo < ratio && ratio < hi) ? 1.0 : 0.0;
      dPol = adv * cg * ratio;
    }
    if (mode == 1) {
      size_t off = 0;
      for (size_t hh = 0; hh < W; hh++) {
        double se = 0.0;
        for (int k = 0; k < hs[hh]; k++) se += exp(out[off + k]);
        double lse = log(se), pout = 0.0;
        for (int k = 0; k < hs[hh]; k++) pout += exp(out[off + k] - lse) * out[off + k];
        for (int k = 0; k < hs[hh]; k++) {
          double p = exp(out[off + k] - lse);
          dout[off + k] = dPol * (((size_t)k == (size_t)act[hh] ? 1.0 : 0.0) - p) + entCoef * p * (pout - out[off + k]);
        }
        off += hs[hh];
      }
    } else {
      for (size_t i = 0; i < W; i++) {
        double lsr = out[W + i];
        double ls = lsr < lsLo ? lsLo : (lsr > lsHi ? lsHi : lsr);
        double lsGrad = (lsLo < lsr && lsr < lsHi) ? 1.0 : 0.0;
        double invStd = exp(-ls);
        double z = (act[i] - out[i]) * invStd;
        dout[i] = dPol * (z * invStd);
        dout[W + i] = lsGrad * (dPol * (z * z - 1.0) + entCoef);
      }
    }
    double vnew = out[O - 1], dvloss_dv;
    if (ov && vfClip > 0.0) {
      double vold = ov[n], dd = vnew - vold;
      double vclip = vold + (dd < -vfClip ? -vfClip : (dd > vfClip ? vfClip : dd));
      double du = (vnew - ret) * (vnew - ret), dc = (vclip - ret) * (vclip - ret);
      if (du >= dc)
        dvloss_dv = (vnew - ret);
      else if (dd > -vfClip && dd < vfClip)
        dvloss_dv = (vnew - ret);
      else
        dvloss_dv = 0.0;
    } else {
      dvloss_dv = (vnew - ret);
    }
    dout[O - 1] = -vfCoef * dvloss_dv;
    if (newlp) newlp[n] = logp;
    if (newval) newval[n] = vnew;
    for (size_t j = 0; j < H; j++) dh[j] = 0.0;
    for (size_t k = 0; k < O; k++) {
      double dk = dout[k];
      double* gw = gW2 + k * H;
      const double* w = W2 + k * H;
      for (size_t j = 0; j < H; j++) {
        gw[j] += dk * h[j];
        dh[j] += dk * w[j];
      }
      gb2[k] += dk;
    }
    for (size_t j = 0; j < H; j++) {
      double dz = (z1[j] > 0.0) ? dh[j] : 0.0;
      double* gw = gW1 + j * D;
      for (size_t d = 0; d < D; d++) gw[d] += dz * x[d];
      gb1[j] += dz;
    }
  }
  free(z1); free(h); free(out); free(dout); free(dh);
}

/* One wide resident update (lean_cuda_train_update_wide_resident, ffi/puffercuda.cu:1307-1409): per
 * epoch and minibatch (mbSize = NT/numMB, the last takes the remainder) gather the rows, normalizeAdv,
 * the summed gradient, mean + global-norm clip (gradClip with maxGradNorm), then stepMat on W1 and W2
 * and stepVec on the biases. pm = [params; mom] updated in place. */
void orc_train_update_wide(double* pm, const double* obs, const double* acts, const double* adv, const double* ret,
                           const double* olp, const double* ov, const double* perm, const int* hs, size_t NT,
                           size_t D, size_t H, size_t O, size_t W, int mode, size_t epochs, size_t numMB, double lr,
                           double wd, double mu, double eps, double vfCoef, double entCoef, double clipEps,
                           double vfClip, double maxGradNorm, double lsLo, const double* coeffs, int iters) {
  const size_t P = H * D + H + O * H + O;
  size_t mbSize = NT / numMB;
  if (mbSize < 1) mbSize = 1;
  double* mObs = (double*)malloc(sizeof(double) * NT * D);
  double* mAct = (double*)malloc(sizeof(double) * NT * W);
  double* mAdv = (double*)malloc(sizeof(double) * NT);
  double* mAdvN = (double*)malloc(sizeof(double) * NT);
  double* mRet = (double*)malloc(sizeof(double) * NT);
  double* mOlp = (double*)malloc(sizeof(double) * NT);
  double* mOv = (double*)malloc(sizeof(double) * NT);
  double* g = (double*)malloc(sizeof(double) * P);
  for (size_t e = 0; e < epochs; e++)
    for (size_t m = 0; m < numMB; m++) {
      size_t lo = m * mbSize, hi = (m + 1 == numMB) ? NT : (m + 1) * mbSize;
      if (hi > NT) hi = NT;
      if (hi <= lo) continue;
      size_t Nmb = hi - lo;
      const double* idx = perm + e * NT + lo;
      for (size_t k = 0; k < Nmb; k++) {
        size_t r = (size_t)idx[k];
        memcpy(mObs + k * D, obs + r * D, sizeof(double) * D);
        memcpy(mAct + k * W, acts + r * W, sizeof(double) * W);
        mAdv[k] = adv[r];
        mRet[k] = ret[r];
        mOlp[k] = olp[r];
        mOv[k] = ov ? ov[r] : 0.0;
      }
      orc_normalize_adv(mAdv, Nmb, mAdvN);
      orc_mlp_ppo_grad_wide(pm, mObs, mAct, mAdvN, mRet, mOlp, ov ? mOv : NULL, Nmb, D, H, O, W, mode, hs, vfCoef,
                            entCoef, clipEps, vfClip, lsLo, g, NULL, NULL);
      orc_grad_clip(g, P, maxGradNorm, 1.0 / (double)Nmb);
      orc_apply_muon(pm, g, D, H, O - 1, 1, lr, wd, mu, eps, coeffs, iters);
    }
  free(mObs); free(mAct); free(mAdv); free(mAdvN); free(mRet); free(mOlp); free(mOv); free(g);
}

/* ---------------------------------------------------------------- LSTM (the third recurrent core) */
/* One LSTM + categorical/value head sequence, truncated BPTT (ffi/pufferffi.c:556-630,
 * lean_ffi_lstm_ppo_grad_seq): params [Wx(4H x D) | Wh(4H x H) | bih(4H) | Wo(O x H) | bo(O)], O = A + 1,
 * gate rows i, f, g, o; h0/c0 the detached initial state; a terminal at step t zeroes the state before
 * step t + 1 and stops the gradient there. Left-folded dots in the reference's order; the head's
 * log-softmax without the max subtracted; no value clip. g[P] is overwritten. */
static double orc_lstm_sig(double x) { return 1.0 / (1.0 + exp(-x)); }
size_t orc_lstm_param_count(size_t D, size_t H, size_t A) {
  return 4 * H * D + 4 * H * H + 4 * H + (A + 1) * H + (A + 1);
}
void orc_lstm_grad_seq(const double* params, const double* obs, const double* actA, const double* advA,
                       const double* retA, const double* oldA, const double* termA, const double* h0,
                       const double* c0, size_t T, size_t H, size_t D, size_t A, double vfCoef, double entCoef,
                       double clipEps, double* g, double* newlp, double* newval) {
  const size_t dout = A + 1, H4 = 4 * H, P = orc_lstm_param_count(D, H, A);
  const double* Wx = params;
  const double* Wh = Wx + H4 * D;
  const double* bih = Wh + H4 * H;
  const double* Wo = bih + H4;
  const double* bo = Wo + dout * H;
  for (size_t i = 0; i < P; i++) g[i] = 0.0;
  double* gWx = g;
  double* gWh = gWx + H4 * D;
  double* gbih = gWh + H4 * H;
  double* gWo = gbih + H4;
  double* gbo = gWo + dout * H;
  double* ii = (double*)malloc(sizeof(double) * T * H);
  double* ff = (double*)malloc(sizeof(double) * T * H);
  double* gga = (double*)malloc(sizeof(double) * T * H);
  double* oo = (double*)malloc(sizeof(double) * T * H);
  double* tc = (double*)malloc(sizeof(double) * T * H);
  double* hp = (double*)malloc(sizeof(double) * T * H);
  double* cp = (double*)malloc(sizeof(double) * T * H);
  double* ht = (double*)malloc(sizeof(double) * T * H);
  double* outs = (double*)malloc(sizeof(double) * T * dout);
  double* h = (double*)malloc(sizeof(double) * H);
  double* c = (double*)malloc(sizeof(double) * H);
  double* gate = (double*)malloc(sizeof(double) * H4);
  for (size_t j = 0; j < H; j++) {
    h[j] = h0[j];
    c[j] = c0[j];
  }
  for (size_t t = 0; t < T; t++) {
    if (t > 0 && termA[t - 1] != 0.0)
      for (size_t j = 0; j < H; j++) h[j] = c[j] = 0.0;
    for (size_t j = 0; j < H; j++) {
      hp[t * H + j] = h[j];
      cp[t * H + j] = c[j];
    }
    const double* x = obs + t * D;
    for (size_t k = 0; k < H4; k++) {
      double gx = 0.0, gh = 0.0;
      const double* wx = Wx + k * D;
      const double* wh = Wh + k * H;
      for (size_t d = 0; d < D; d++) gx += wx[d] * x[d];
      for (size_t d = 0; d < H; d++) gh += wh[d] * h[d];
      gate[k] = bih[k] + gx + gh;
    }
    for (size_t j = 0; j < H; j++) {
      double ig = orc_lstm_sig(gate[j]), fg = orc_lstm_sig(gate[H + j]), gg = tanh(gate[2 * H + j]),
             og = orc_lstm_sig(gate[3 * H + j]);
      double cj = fg * c[j] + ig * gg, tcj = tanh(cj);
      ii[t * H + j] = ig;
      ff[t * H + j] = fg;
      gga[t * H + j] = gg;
      oo[t * H + j] = og;
      tc[t * H + j] = tcj;
      c[j] = cj;
      h[j] = og * tcj;
      ht[t * H + j] = h[j];
    }
    for (size_t m = 0; m < dout; m++) {
      double acc = 0.0;
      const double* w = Wo + m * H;
      for (size_t j = 0; j < H; j++) acc += w[j] * h[j];
      outs[t * dout + m] = bo[m] + acc;
    }
  }
  double* dh_next = (double*)calloc(H, sizeof(double));
  double* dc_next = (double*)calloc(H, sizeof(double));
  double* dh = (double*)malloc(sizeof(double) * H);
  double* dhprev = (double*)malloc(sizeof(double) * H);
  double* dcprev = (double*)malloc(sizeof(double) * H);
  double* dgate = (double*)malloc(sizeof(double) * H4);
  double* dout_ = (double*)malloc(sizeof(double) * dout);
  double* pk = (double*)malloc(sizeof(double) * (A ? A : 1));
  for (size_t tt = T; tt-- > 0;) {
    const size_t t = tt;
    const double* out = outs + t * dout;
    const size_t a = (size_t)actA[t];
    const double adv = advA[t], ret = retA[t], oldLogp = oldA[t];
    double sumexp = 0.0;
    for (size_t k = 0; k < A; k++) sumexp += exp(out[k]);
    const double lse = log(sumexp);
    double pout = 0.0;
    for (size_t k = 0; k < A; k++) {
      pk[k] = exp(out[k] - lse);
      pout += pk[k] * out[k];
    }
    const double logpA = out[a] - lse, ratio = exp(logpA - oldLogp), lo = 1.0 - clipEps, hi = 1.0 + clipEps;
    const double ratioC = ratio < lo ? lo : (ratio > hi ? hi : ratio), surr1 = adv * ratio, surr2 = adv * ratioC;
    double dPol;
    if (surr1 <= surr2)
      dPol = adv * ratio;
    else
      dPol = adv * ((lo < ratio && ratio < hi) ? 1.0 : 0.0) * ratio;
    for (size_t k = 0; k < A; k++) {
      double dp = dPol * (((k == a) ? 1.0 : 0.0) - pk[k]);
      double de = entCoef * pk[k] * (pout - out[k]);
      dout_[k] = dp + de;
    }
    dout_[A] = -vfCoef * (out[A] - ret);
    if (newlp) newlp[t] = logpA;
    if (newval) newval[t] = out[A];
    for (size_t j = 0; j < H; j++) dh[j] = dh_next[j];
    for (size_t m = 0; m < dout; m++) {
      const double dm = dout_[m];
      double* gw = gWo + m * H;
      const double* w = Wo + m * H;
      gbo[m] += dm;
      for (size_t j = 0; j < H; j++) {
        gw[j] += dm * ht[t * H + j];
        dh[j] += dm * w[j];
      }
    }
    for (size_t j = 0; j < H; j++) {
      const double tcj = tc[t * H + j], og = oo[t * H + j];
      const double dcj = dc_next[j] + dh[j] * og * (1.0 - tcj * tcj);
      const double do_ = dh[j] * tcj, ig = ii[t * H + j], fg = ff[t * H + j], gg = gga[t * H + j],
                   cprev = cp[t * H + j];
      const double df_ = dcj * cprev, di_ = dcj * gg, dg_ = dcj * ig;
      dcprev[j] = dcj * fg;
      dgate[j] = di_ * ig * (1.0 - ig);
      dgate[H + j] = df_ * fg * (1.0 - fg);
      dgate[2 * H + j] = dg_ * (1.0 - gg * gg);
      dgate[3 * H + j] = do_ * og * (1.0 - og);
    }
    for (size_t d = 0; d < H; d++) dhprev[d] = 0.0;
    const double* x = obs + t * D;
    const double* hprevk = hp + t * H;
    for (size_t k = 0; k < H4; k++) {
      const double da = dgate[k];
      gbih[k] += da;
      double* gwx = gWx + k * D;
      for (size_t d = 0; d < D; d++) gwx[d] += da * x[d];
      double* gwh = gWh + k * H;
      const double* wh = Wh + k * H;
      for (size_t d = 0; d < H; d++) {
        gwh[d] += da * hprevk[d];
        dhprev[d] += da * wh[d];
      }
    }
    const int flow = (t > 0 && termA[t - 1] == 0.0);
    for (size_t j = 0; j < H; j++) {
      dh_next[j] = flow ? dhprev[j] : 0.0;
      dc_next[j] = flow ? dcprev[j] : 0.0;
    }
  }
  free(ii); free(ff); free(gga); free(oo); free(tc); free(hp); free(cp); free(ht); free(outs);
  free(h); free(c); free(gate); free(dh_next); free(dc_next); free(dh); free(dhprev); free(dcprev); free(dgate);
  free(dout_); free(pk);
}

/* The batched form (lean_ffi_lstm_ppo_grad_batch_blas, ffi/pufferblas.c:897-1018): B sequences packed
 * time-major (obs [(t*B + b)*D + d], scalars [t*B + b], h0s/c0s [b*H + j]); the summed gradient over b in
 * order 0..B-1 of the per-sequence ones. out = [g(P); newlp(T*B); newval(T*B)], the last two time-major. */
void orc_lstm_grad_batch(const double* params, const double* obsB, const double* acts, const double* advs,
                         const double* rets, const double* olps, const double* terms, const double* h0s,
                         const double* c0s, size_t B, size_t T, size_t H, size_t D, size_t A, double vfCoef,
                         double entCoef, double clipEps, double* out) {
  const size_t P = orc_lstm_param_count(D, H, A), nb = T * B;
  double* gb = (double*)malloc(sizeof(double) * P);
  double* so = (double*)malloc(sizeof(double) * T * D);
  double* sc = (double*)malloc(sizeof(double) * 5 * T);
  double* nl = (double*)malloc(sizeof(double) * T);
  double* nv = (double*)malloc(sizeof(double) * T);
  for (size_t i = 0; i < P; i++) out[i] = 0.0;
  for (size_t b = 0; b < B; b++) {
    for (size_t t = 0; t < T; t++) {
      for (size_t d = 0; d < D; d++) so[t * D + d] = obsB[(t * B + b) * D + d];
      sc[t] = acts[t * B + b];
      sc[T + t] = advs[t * B + b];
      sc[2 * T + t] = rets[t * B + b];
      sc[3 * T + t] = olps[t * B + b];
      sc[4 * T + t] = terms[t * B + b];
    }
    orc_lstm_grad_seq(params, so, sc, sc + T, sc + 2 * T, sc + 3 * T, sc + 4 * T, h0s + b * H, c0s + b * H, T, H, D, A,
                      vfCoef, entCoef, clipEps, gb, nl, nv);
    for (size_t i = 0; i < P; i++) out[i] = out[i] + gb[i];
    for (size_t t = 0; t < T; t++) {
      out[P + t * B + b] = nl[t];
      out[P + nb + t * B + b] = nv[t];
    }
  }
  free(gb); free(so); free(sc); free(nl); free(nv);
}

/* Per-segment GAE with bootstrap, then the advantages normalised over all N*T (ffi/pufferffi.c:975-1010,
 * lean_ffi_lstm_gae_boot_norm): time-major columns [t*N + n]; out = [adv(N*T); ret(N*T)]. */
void orc_lstm_gae_boot_norm(const double* vals, const double* rews, const double* terms, const double* bootV,
                            size_t N, size_t T, double gamma, double lam, double* out) {
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
}
