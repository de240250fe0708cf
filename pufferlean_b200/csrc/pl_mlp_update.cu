// The PPO+Muon update of the feed-forward policy: one session per (policy handle, shapes), every
// buffer resident, epochs x minibatches run back to back on one stream.
//
// Per minibatch (bf16 tier):
//   gather rows of the resident columns through the epoch's shuffle (+ advantage mean/std)
//   forward   H_l = act(H_{l-1} W_l^T + b_l)             tcgen05 GEMM, bias+act epilogue
//   head      logits/value = H_L W_o^T + b_o -> dOut     tcgen05 GEMM, PPO-objective-gradient epilogue
//   backward  dW_l = dZ_l^T H_{l-1} (MN-major operands, split-K, fixed-order slice sum)
//             dZ_{l-1} = (dZ_l W_l) * act'(Z_{l-1})      tcgen05 GEMM, act' epilogue + bias column sums
//   clip      global grad norm of the mean gradient (fixed-order f64 reduction)
//   Muon      f64 Nesterov -> Frobenius normalise -> Newton-Schulz on the tensor cores ->
//             f64 decoupled-decay ascent step on the master weights + their bf16 shadow
// The tight tier (bf16 = 0) runs the same sequence with fp32 SIMT GEMMs and the f64 Newton-Schulz
// of the reference oracle. Semantics follow lean_cuda_train_update_resident
// (ffi/puffercuda.cu:1187-1294): mbSize = NT/numMB with the last minibatch taking the remainder,
// gradients summed over rows then scaled to the mean (and clipped when maxGradNorm > 0), value
// clip when old values are supplied and vfClip > 0.
#include <math.h>
#include <string.h>

#include <atomic>
#include <functional>
#include <mutex>
#include <vector>

#include "pl_comm.h"
#include "pl_gemm.cuh"
#include "pl_mlp.cuh"
#include "pl_muon.cuh"
#include "pl_runtime.h"
#include "pl_host_stage.h"

using namespace pl;

struct pl_update {
  pl_update_desc d;
  int dev = 0;
  double* pm = nullptr;  // [params(P); mom(P)] f64 (policy handle)
  size_t P = 0;
  int L = 1, O = 0, Op = 64, Dp = 64, Hp = 64;
  long mbSize = 0, mbMax = 0;
  bool fast = true;
  std::vector<Layer> layers;
  std::vector<double> coeffs;
  int iters = 5;
  std::vector<void*> allocs;
  // columns
  void* obs = nullptr;  // fast: bf16 [NT x Dp]; tight: f32 [NT x D]
  int* act_c = nullptr;
  double* adv_c = nullptr;
  float *ret_c = nullptr, *olp_c = nullptr, *ov_c = nullptr;
  int* perm = nullptr;
  double* stage = nullptr;
  size_t stage_elems = 0;
  // minibatch
  void* X = nullptr;
  std::vector<void*> Hs, Zs;
  void* dZ[2] = {nullptr, nullptr};
  void* dOut = nullptr;
  float* Out = nullptr;  // tight tier logits
  int* mb_act = nullptr;
  float *mb_adv = nullptr, *mb_ret = nullptr, *mb_olp = nullptr, *mb_ov = nullptr;
  double* adv_part = nullptr;
  double* ms = nullptr;
  float* colpart = nullptr;
  float* splitk = nullptr;
  size_t splitk_elems = 0;
  float* grad = nullptr;
  double* gn_part = nullptr;
  double* cc = nullptr;
  float* loss_part = nullptr;
  // parameters in compute precision
  std::vector<__nv_bfloat16*> Wb;  // fast tier shadows (out_p x in_p)
  std::vector<float*> Wf;          // tight tier fp32 weights (out x in)
  std::vector<float*> bf;          // fp32 biases (out_p)
  NsWork ns;
  double* exact_ws = nullptr;
  uint64_t launches = 0;
  bool grad_only = false;  // pl_mlp_ppo_grad: no normalisation, no optimizer step
  bool alloc_failed = false;
  float* adv_f = nullptr;  // fp32 scan output of pl_update_set_advantages_dev
  // data parallelism
  bool dp = false;             // world > 1 with a communicator
  // strong-scaling split (pl_update_split_minibatch): every rank holds the same columns and takes rows
  // [lo + n*r/R, lo + n*(r+1)/R) of each minibatch [lo, lo + n)
  bool split = false;
  long nglob = 0;  // rows of the current minibatch over all ranks: the gradient mean's divisor
  // the gradient all-reduce in per-layer buckets on a second stream, each started as soon as that
  // layer's gradient block is complete, so it runs under the rest of the backward pass
  bool overlap = true;
  cudaStream_t ast = nullptr;
  std::vector<cudaEvent_t> aev;  // [layers] block complete, [layers] all-reduces done
  double comm_ms = 0, comm_bytes = 0, comm_launches = 0;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> comm_ev;
  std::vector<double> comm_ev_bytes;
  size_t comm_ev_used = 0;
  double* adv_sums = nullptr;  // [sum, sum of squares, count] of the minibatch's raw advantages
  std::vector<int> owner;      // Newton-Schulz owner rank of each layer
  std::vector<std::vector<int>> ns_groups;  // layers of equal shape, orthogonalised as one batch
  std::vector<ExactLayer> exact_group;      // tight tier: every layer when each fits one CTA's step
  long ns_batch = 1;                        // workspace slots: every layer's (one at a time under data parallelism)
  std::vector<long> ns_slot0;               // first slot of each group (its matrices' X, G, Pm and result)
  long ns_slotx = 0, ns_slotg = 0, ns_slotf = 0;  // elements per slot of X0 / X1, of G / B and of Xf
  float* ns_scale = nullptr;                // first-step Newton-Schulz factors of a group: [group] s, [group] s^2
  std::vector<float*> xres;    // per-layer orthogonalised update (m x n wide layout, fp32)
  // profiling: CUDA events around each launch group, per class
  bool prof = false;
  std::vector<cudaEvent_t> ev;
  size_t ev_used = 0;
  std::vector<int> ev_cls;
  double prof_flops[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  double prof_launch[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  double prof_ms[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  bool loss_on = false;
  double losses[7] = {0, 0, 0, 0, 0, 0, 0};
  HostStage hstage;  // pinned staging of host observations rounded to bf16 on the host
  // Observations kept in the first epoch's shuffle order (reference-shaped call, bf16 tier): the host
  // rounds and copies the rows of each first-epoch minibatch on a copy stream just ahead of it, so the
  // upload runs under the compute; later epochs read rows through perm translated into those positions.
  const double* pend_obs = nullptr;   // host rows not yet uploaded (until the first epoch has run)
  const double* pend_perm = nullptr;  // the host shuffle whose first epoch orders them
  bool obs_epoch0 = false;            // obs holds rows in the first epoch's order
  int* pos0 = nullptr;                // NT ints, scratch of the translation
  int* operm = nullptr;               // epochs x NT first-epoch positions
  cudaStream_t cst = nullptr;
  cudaEvent_t cev = nullptr, sev = nullptr;
  // wide action heads (pl_update_set_head): 0 categorical, 1 multi-discrete, 2 Gaussian
  int head_mode = 0;
  int W = 1;
  int* hs_dev = nullptr;      // head sizes (mode 1)
  float* actw_c = nullptr;    // action column [NT x W]
  float* mb_actw = nullptr;   // its minibatch rows [mbMax x W]
  float* Outw = nullptr;      // fast tier: fp32 head GEMM output [mbMax x Op]
};

namespace {

// Log-std clamp of the Gaussian head (the resident device path's bounds, ffi/puffercuda.cu:1647-1648).
constexpr float kContLogStdLo = -20.f, kContLogStdHi = 2.f;

static std::mutex g_mu;
static bool g_loss_on = false;
static bool g_host_bf16 = true;
static bool g_dp_overlap = true;  // sessions created afterwards overlap the gradient all-reduce
static bool g_exact_group = true;  // tight-tier sessions created afterwards may use the one-launch Muon step
static bool g_ns_one_launch = true;  // bf16 tier: the groups' Newton-Schulz chains share one launch
static std::atomic<uint64_t> g_upload_bytes{0};  // host-to-device bytes of the last set_columns call  // bf16 tier: host observations rounded to bf16 on the host threads
static double g_losses[7] = {0, 0, 0, 0, 0, 0, 0};

template <typename T>
static T* dalloc(pl_update* u, size_t n) {
  void* p = nullptr;
  if (n == 0) n = 1;
  if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) {
    cudaGetLastError();
    u->alloc_failed = true;
    set_error(PL_ERR_NOMEM, "cudaMalloc of %zu bytes failed", n * sizeof(T));
    return nullptr;
  }
  u->allocs.push_back(p);
  return (T*)p;
}

static void free_all(pl_update* u) {
  for (void* p : u->allocs) cudaFree(p);
  u->allocs.clear();
}

// Profiling spans: an event before and after each launch group, recorded on the launch stream.
struct Span {
  pl_update* u;
  int cls;
  cudaStream_t st;
  double flops;
  Span(pl_update* u_, int c, cudaStream_t s, double f) : u(u_), cls(c), st(s), flops(f) {
    if (!u->prof) return;
    while (u->ev.size() < u->ev_used + 2) {
      cudaEvent_t e;
      cudaEventCreate(&e);
      u->ev.push_back(e);
    }
    cudaEventRecord(u->ev[u->ev_used], st);
  }
  ~Span() {
    if (!u->prof) return;
    cudaEventRecord(u->ev[u->ev_used + 1], st);
    u->ev_cls.push_back(cls);
    u->ev_used += 2;
    u->prof_flops[cls] += flops;
    u->prof_launch[cls] += 1;
  }
};

static void prof_collect(pl_update* u) {
  if (u->comm_ev_used) {
    cudaDeviceSynchronize();
    for (size_t i = 0; i < u->comm_ev_used; i++) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, u->comm_ev[i].first, u->comm_ev[i].second);
      u->comm_ms += ms;
      u->comm_bytes += u->comm_ev_bytes[i];
      u->comm_launches += 1;
    }
    u->comm_ev_used = 0;
  }
  if (u->ev_used == 0) return;
  cudaDeviceSynchronize();
  for (size_t i = 0; i < u->ev_cls.size(); i++) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, u->ev[2 * i], u->ev[2 * i + 1]);
    u->prof_ms[u->ev_cls[i]] += ms;
  }
  u->ev_cls.clear();
  u->ev_used = 0;
}

static inline double gf(long M, long N, long K) { return 2.0 * (double)M * (double)N * (double)K; }

static int build_layout(pl_update* u) {
  const pl_update_desc& d = u->d;
  u->L = (int)(d.arch.L ? d.arch.L : 1);
  u->O = (int)d.A + 1;
  u->Op = u->O <= 64 ? 64 : 128;
  u->Dp = (int)round_up((long)d.D, 64);
  u->Hp = (int)round_up((long)d.H, 64);
  u->layers.clear();
  size_t off = 0;
  for (int l = 0; l <= u->L; l++) {
    Layer ly;
    ly.in = l == 0 ? (int)d.D : (int)d.H;
    ly.out = l == u->L ? u->O : (int)d.H;
    ly.in_p = l == 0 ? u->Dp : u->Hp;
    ly.out_p = l == u->L ? u->Op : u->Hp;
    ly.oW = off;
    off += (size_t)ly.out * ly.in;
    ly.ob = off;
    off += (size_t)ly.out;
    u->layers.push_back(ly);
  }
  u->P = off;
  u->mbSize = (long)(d.NT / d.numMB);
  if (u->mbSize < 1) u->mbSize = 1;
  u->mbMax = (long)d.NT - (long)(d.numMB - 1) * u->mbSize;
  if (u->mbMax < u->mbSize) u->mbMax = u->mbSize;
  if (u->mbMax > (long)d.NT) u->mbMax = (long)d.NT;
  return PL_OK;
}

static int alloc_session(pl_update* u) {
  const pl_update_desc& d = u->d;
  const long NT = (long)d.NT, M = u->mbMax;
  const int L = u->L;
  const bool fast = u->fast;
  const size_t es = fast ? 2 : 4;  // activation element size
  (void)es;
  // columns
  if (fast)
    u->obs = dalloc<__nv_bfloat16>(u, (size_t)NT * u->Dp);
  else
    u->obs = dalloc<float>(u, (size_t)NT * d.D);
  u->act_c = dalloc<int>(u, NT);
  u->adv_c = dalloc<double>(u, NT);
  u->ret_c = dalloc<float>(u, NT);
  u->olp_c = dalloc<float>(u, NT);
  u->ov_c = d.use_old_values ? dalloc<float>(u, NT) : nullptr;
  u->perm = dalloc<int>(u, (size_t)d.epochs * NT);
  u->stage_elems = (size_t)std::min<long>(std::max<long>(NT * 8, (long)d.epochs * NT), 1L << 25);
  if (u->stage_elems < (size_t)NT) u->stage_elems = NT;
  if (u->stage_elems < u->P) u->stage_elems = u->P;  // the tight tier widens the gradient here
  u->stage = dalloc<double>(u, u->stage_elems);
  // minibatch
  const int mt = (int)ceil_div(M, 128);
  if (fast) {
    u->X = dalloc<__nv_bfloat16>(u, (size_t)M * u->Dp);
    for (int l = 0; l < L; l++) {
      u->Hs.push_back(dalloc<__nv_bfloat16>(u, (size_t)M * u->Hp));
      u->Zs.push_back(d.arch.act == 1 ? (void*)dalloc<__nv_bfloat16>(u, (size_t)M * u->Hp) : nullptr);
    }
    u->dZ[0] = dalloc<__nv_bfloat16>(u, (size_t)M * u->Hp);
    u->dZ[1] = dalloc<__nv_bfloat16>(u, (size_t)M * u->Hp);
    u->dOut = dalloc<__nv_bfloat16>(u, (size_t)M * u->Op);
  } else {
    u->X = dalloc<float>(u, (size_t)M * d.D);
    for (int l = 0; l < L; l++) {
      u->Hs.push_back(dalloc<float>(u, (size_t)M * d.H));
      u->Zs.push_back(dalloc<float>(u, (size_t)M * d.H));
    }
    u->dZ[0] = dalloc<float>(u, (size_t)M * d.H);
    u->dZ[1] = dalloc<float>(u, (size_t)M * d.H);
    u->dOut = dalloc<float>(u, (size_t)M * u->O);
    u->Out = dalloc<float>(u, (size_t)M * u->O);
  }
  u->mb_act = dalloc<int>(u, M);
  u->mb_adv = dalloc<float>(u, M);
  u->mb_ret = dalloc<float>(u, M);
  u->mb_olp = dalloc<float>(u, M);
  u->mb_ov = d.use_old_values ? dalloc<float>(u, M) : nullptr;
  u->adv_part = dalloc<double>(u, 2 * 4096);
  u->ms = dalloc<double>(u, 4);
  u->colpart = dalloc<float>(u, (size_t)colsum_scratch_elems(mt, std::max(u->Hp, u->Op)));
  u->grad = dalloc<float>(u, u->P);
  u->gn_part = dalloc<double>(u, 4096);
  u->cc = dalloc<double>(u, 4);
  u->loss_part = dalloc<float>(u, (size_t)mt * 8);
  // split-K slices for the largest weight gradient
  size_t maxw = 0;
  for (auto& ly : u->layers) maxw = std::max(maxw, (size_t)ly.out * ly.in);
  u->splitk_elems = maxw * 8;
  // the tight tier's SIMT weight gradients (with the bias column) split K, the minibatch rows, into
  // slices of 64 (at most 16 MB of workspace)
  if (!fast)
    for (auto& ly : u->layers)
      u->splitk_elems = std::max(u->splitk_elems,
                                 (size_t)std::min<long>(splitk_wb_elems((int)u->mbMax, ly.out, ly.in), 1L << 22));
  u->splitk = dalloc<float>(u, u->splitk_elems);  // tight tier: the split-K weight gradients
  // parameters in compute precision
  for (auto& ly : u->layers) {
    if (fast) {
      u->Wb.push_back(dalloc<__nv_bfloat16>(u, (size_t)ly.out_p * ly.in_p));
      u->Wf.push_back(nullptr);
    } else {
      u->Wb.push_back(nullptr);
      u->Wf.push_back(dalloc<float>(u, (size_t)ly.out * ly.in));
    }
    u->bf.push_back(dalloc<float>(u, ly.out_p));
  }
  // Muon workspace
  long mmax = 0, nmax = 0;
  for (auto& ly : u->layers) {
    long m = std::min(ly.out, ly.in), n = std::max(ly.out, ly.in);
    mmax = std::max(mmax, m);
    nmax = std::max(nmax, n);
  }
  const long ldx = round_up(nmax, 64), ldg = round_up(mmax, 64);
  // equal-shaped layers (the hidden 2048 x 2048 matrices of configs[4]) share one batched
  // Newton-Schulz: one launch per GEMM of the chain covers all of them, filling the GPU's SMs
  u->ns_groups.clear();
  for (size_t l = 0; l < u->layers.size(); l++) {
    bool placed = false;
    for (auto& g : u->ns_groups) {
      const Layer& f = u->layers[g[0]];
      if (f.out == u->layers[l].out && f.in == u->layers[l].in) {
        g.push_back((int)l);
        placed = true;
        break;
      }
    }
    if (!placed) u->ns_groups.push_back({(int)l});
  }
  // each group has slots of its own (under data parallelism each layer: layer l in slot l), so that
  // all the Newton-Schulz chains of a Muon step can run in one launch
  u->ns_slot0.clear();
  long next = 0;
  for (auto& g : u->ns_groups) {
    u->ns_slot0.push_back(next);
    next += (long)g.size();
  }
  u->ns_batch = std::max<long>(1, u->dp ? (long)u->layers.size() : next);
  if (fast) {
    // one batch slot holds the largest matrix; a group's batch uses slots of its own (smaller) size
    const long slotx = round_up(mmax, 128) * ldx, slotg = round_up(mmax, 128) * ldg;
    u->ns_slotx = slotx;
    u->ns_slotg = slotg;
    u->ns_slotf = mmax * ldx;
    u->ns.ldx = ldx;
    u->ns.ldg = ldg;
    u->ns.X0 = dalloc<__nv_bfloat16>(u, (size_t)(slotx * u->ns_batch));
    u->ns.X1 = dalloc<__nv_bfloat16>(u, (size_t)(slotx * u->ns_batch));
    u->ns.G = dalloc<__nv_bfloat16>(u, (size_t)(slotg * u->ns_batch));
    u->ns.B = dalloc<__nv_bfloat16>(u, (size_t)(slotg * u->ns_batch));
    u->ns.Xf = dalloc<float>(u, (size_t)(mmax * ldx * u->ns_batch));
    // per-block sums of u^2 of one group: at most kMuonBlocksMax in all (muon_group_blocks), or one
    // block per layer of a larger group
    u->ns.part = dalloc<double>(u, std::max<size_t>(4096, kMuonBlocksMax + u->layers.size()));
    u->ns_scale = dalloc<float>(u, 2 * u->layers.size());
    // per group 3 x batch chain counters at 3 x its first slot; the last word is the shared abort word
    u->ns.cnt = dalloc<unsigned>(u, (size_t)ns_chain_counter_words(u->ns_batch));
    for (void* p : {(void*)u->ns.X0, (void*)u->ns.X1, (void*)u->ns.G, (void*)u->ns.B})
      if (p) cudaMemset(p, 0, 1);  // touch
  } else {
    size_t ws = 0;
    for (auto& ly : u->layers) ws = std::max(ws, exact_ws_doubles(ly.out, ly.in));
    u->exact_ws = dalloc<double>(u, ws);
    // layers small enough for one CTA each take the one-launch group step
    u->exact_group.clear();
    for (size_t l = 0; l < u->layers.size(); l++) {
      const Layer& ly = u->layers[l];
      u->exact_group.push_back(ExactLayer{ly.out, ly.in, (long)ly.oW, (long)ly.ob, u->Wf[l], u->bf[l]});
    }
    if (!g_exact_group || !muon_group_fits(u->exact_group.data(), (int)u->exact_group.size(), u->iters))
      u->exact_group.clear();
  }
  if (u->dp) {
    u->adv_sums = dalloc<double>(u, 4);
    if (fast)
      for (auto& ly : u->layers) u->xres.push_back(dalloc<float>(u, (size_t)ly.out * ly.in));
  }
  if (u->alloc_failed) return PL_ERR_NOMEM;
  // zero the padded shadow weights/biases once; their pads stay zero for the session
  for (size_t l = 0; l < u->layers.size(); l++) {
    if (u->Wb[l]) PL_CUDA(cudaMemset(u->Wb[l], 0, sizeof(__nv_bfloat16) * u->layers[l].out_p * u->layers[l].in_p));
    PL_CUDA(cudaMemset(u->bf[l], 0, sizeof(float) * u->layers[l].out_p));
  }
  if (fast) {
    PL_CUDA(cudaMemset(u->X, 0, sizeof(__nv_bfloat16) * M * u->Dp));
    PL_CUDA(cudaMemset(u->ns.X0, 0, sizeof(__nv_bfloat16) * u->ns_slotx * u->ns_batch));
    PL_CUDA(cudaMemset(u->ns.X1, 0, sizeof(__nv_bfloat16) * u->ns_slotx * u->ns_batch));
  }
  return PL_OK;
}

// f64 master -> compute-precision copies of every layer (after load and after each Muon step).
static int refresh_shadows(pl_update* u, cudaStream_t st) {
  for (size_t l = 0; l < u->layers.size(); l++) {
    const Layer& ly = u->layers[l];
    int rc;
    if (u->fast)
      rc = launch_w_to_bf16(u->pm + ly.oW, ly.out, ly.in, u->Wb[l], ly.in_p, st);
    else
      rc = launch_f64_to_f32(u->pm + ly.oW, (long)ly.out * ly.in, u->Wf[l], st);
    if (rc) return rc;
    rc = launch_f64_to_f32(u->pm + ly.ob, ly.out, u->bf[l], st);
    if (rc) return rc;
  }
  return PL_OK;
}

static int pick_bn(int N) { return N <= 64 ? 64 : (N <= 128 ? 128 : 256); }

// Weight gradient dW[out x in] = sum_rows dZ[row, out] * Hin[row, in] into grad (f32, row-major)
static int wgrad_fast(pl_update* u, const void* dZ, long ldz, int out, const void* Hin, long ldh, int in, int Nmb,
                      float* dst, cudaStream_t st) {
  Operand A{dZ, Nmb, out, ldz, 1, 0};
  Operand B{Hin, Nmb, in, ldh, 1, 0};
  const int bn = in <= 128 ? 128 : 256;
  const long tiles = ceil_div(out, 128) * ceil_div(in, bn);
  const long kb = ceil_div(Nmb, 64);
  // Split count: the persistent kernel deals tiles x S jobs round-robin to the SMs, so the step takes
  // ceil(tiles S / SMs) jobs of ceil(kb / S) k-blocks on the busiest SM; take the S that minimises
  // that product (the fewest slices on a tie), with at least 4 k-blocks per slice and the fp32 slices
  // within the workspace. 128 tiles of a 2048 x 2048 weight over 262,144 rows: S = 8 (7 waves, 98.8 %
  // of the SMs busy) instead of 3 (3 waves, 86.5 %); the 2048 x 1024 layer: 16 instead of 5.
  int nsm = 148;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, u->dev);
  int S = 1;
  long best = -1;
  for (int c = 1; c <= 16; c++) {
    if (c > 1 && (kb / c < 4 || (size_t)c * out * in > u->splitk_elems)) break;
    const long cost = ceil_div(tiles * c, nsm) * ceil_div(kb, c);
    if (best < 0 || cost < best) {
      best = cost;
      S = c;
    }
  }
  EpiArgs e{};
  e.ldo = in;
  e.out_rows = out;
  e.out_cols = in;
  e.alpha = 1.f;
  if (S == 1) {
    e.out = dst;
    return gemm_launch(bn, EPI_F32, true, true, A, B, out, in, Nmb, 1, e, st);
  }
  e.out = u->splitk;
  e.out_bstride = (long)out * in;
  e.k_splits = S;
  int rc = gemm_launch(bn, EPI_F32, true, true, A, B, out, in, Nmb, 1, e, st);
  if (rc) return rc;
  return launch_splitk_reduce(u->splitk, S, (long)out * in, dst, st);
}

// Launch arguments of layers grp[q0, q0 + kMuonGroupMax) for the Muon group kernels: xin(q) is layer
// grp[q]'s Newton-Schulz input (NULL where this rank does not orthogonalise it), xres(q) its result,
// both in the wide layout with leading dimension ldx.
template <class FX, class FR>
static MuonGroupArgs muon_args(const pl_update* u, const std::vector<int>& grp, int q0, long ldx, FX xin, FR xres) {
  MuonGroupArgs a{};
  const Layer& f = u->layers[grp[0]];
  a.nb = std::min<int>(kMuonGroupMax, (int)grp.size() - q0);
  a.rows = f.out;
  a.cols = f.in;
  a.ldx = ldx;
  a.ldw = f.in_p;
  for (int j = 0; j < a.nb; j++) {
    const int l = grp[q0 + j];
    const Layer& ly = u->layers[l];
    a.gW[j] = u->grad + ly.oW;
    a.mW[j] = u->pm + u->P + ly.oW;
    a.X[j] = xin(q0 + j);
    a.Xf[j] = xres(q0 + j);
    a.W[j] = u->pm + ly.oW;
    a.Wb[j] = u->Wb[l];
    a.gb[j] = u->grad + ly.ob;
    a.b[j] = u->pm + ly.ob;
    a.mb[j] = u->pm + u->P + ly.ob;
    a.bf[j] = u->bf[l];
  }
  return a;
}

// The Muon update's factor for a rows x cols weight: sqrt(max(1, rows / cols)).
static double muon_shape_scale(const Layer& ly) {
  const double r = (double)ly.out / (double)ly.in;
  return sqrt(r > 1.0 ? r : 1.0);
}

// One batch of equal-shape matrices for ns_run_groups: its workspace slots, the wide input (w.X0,
// leading dimension ldx, xbs between matrices), the fp32 result and the first step's factors.
struct NsGroupRun {
  NsWork w;
  int m = 0, n = 0, batch = 0;
  long ldx = 0, xbs = 0;
  float* out = nullptr;
  long ld_out = 0, obs = 0;
  bool small = false;     // the fused one-CTA kernel, which normalises the raw input itself
  float* scale = nullptr;  // otherwise [batch] 1 / (||u|| + eps), [batch] its square
};

// Newton-Schulz of several batches: those the persistent chain takes share launches
// (kNsChainMaxGroups each), so that short dependent chains run beside a large batch's tiles; the
// short-matrix batches, and any the chain declines, run through ns_run_batched on their own slots.
static int ns_run_groups(pl_update* u, const std::vector<NsGroupRun>& gs, cudaStream_t st) {
  int rc = PL_OK;
  std::vector<NsChainGroupHost> hs;
  std::vector<size_t> hg;
  for (size_t k = 0; k < gs.size(); k++) {
    const NsGroupRun& g = gs[k];
    if (g.small) continue;
    NsChainGroupHost h{};
    h.m = g.m;
    h.n = g.n;
    h.batch = g.batch;
    h.X = g.w.X0;
    h.xbuf[0] = g.w.X0;
    h.xbuf[1] = g.w.X1;
    h.ldx = g.ldx;
    h.xbs = g.xbs;
    h.G = g.w.G;
    h.B = g.w.B;
    h.ldg = g.w.ldg;
    h.out_f32 = g.out;
    h.ld_out = g.ld_out;
    h.obs = g.obs;
    h.scale0 = g.scale;
    h.fold_eps = -1.0;
    h.cnt = g.w.cnt;
    hs.push_back(h);
    hg.push_back(k);
  }
  std::vector<char> done(gs.size(), 0);
  for (size_t k0 = 0; g_ns_one_launch && k0 < hs.size() && !rc; k0 += kNsChainMaxGroups) {
    const int k = (int)std::min(hs.size() - k0, (size_t)kNsChainMaxGroups);
    // every group's counters and the abort word (the last word) start at zero
    PL_CUDA(cudaMemsetAsync(u->ns.cnt, 0, sizeof(unsigned) * (size_t)ns_chain_counter_words(u->ns_batch), st));
    bool used = false;
    rc = ns_chain_launch(k, hs.data() + k0, u->coeffs.data(), u->iters, u->ns.cnt + 3 * u->ns_batch, u->ns.err, st,
                         &used);
    if (used)
      for (int j = 0; j < k; j++) done[hg[k0 + j]] = 1;
  }
  for (size_t k = 0; k < gs.size() && !rc; k++) {
    if (done[k]) continue;
    NsWork w = gs[k].w;
    const NsGroupRun& g = gs[k];
    rc = ns_run_batched(g.m, g.n, g.batch, u->coeffs.data(), u->iters, w, g.w.X0, g.ldx, g.xbs, g.out, g.ld_out,
                        g.obs, st, nullptr, nullptr, g.small ? nullptr : g.scale, g.small ? u->d.eps : -1.0);
  }
  return rc;
}

// The workspace view whose first slot is s0.
static NsWork ns_slots(const pl_update* u, long s0) {
  NsWork w = u->ns;
  w.X0 += s0 * u->ns_slotx;
  w.X1 += s0 * u->ns_slotx;
  w.G += s0 * u->ns_slotg;
  w.B += s0 * u->ns_slotg;
  w.Xf += s0 * u->ns_slotf;
  w.cnt += 3 * s0;
  return w;
}

// Data-parallel Muon: every rank advances the momentum of every layer; each layer's Newton-Schulz
// runs on its owner rank only (pl_muon_shard_plan), which also writes its unscaled input (in the
// layer's own slot) and the factor, all the rank's layers in one chain launch; one grouped broadcast
// hands every rank every orthogonalised update; every rank then applies the identical f64 step, so
// the weights stay bit-identical across ranks.
static int muon_sharded(pl_update* u, double lr, cudaStream_t st) {
  const pl_update_desc& d = u->d;
  int rc = PL_OK;
  std::vector<NsGroupRun> runs;
  double ns_flops = 0.0;
  for (size_t l = 0; l < u->layers.size(); l++) {
    const Layer& ly = u->layers[l];
    const int m = std::min(ly.out, ly.in), nn = std::max(ly.out, ly.in);
    const bool own = u->owner[l] == d.rank;
    const bool small = ns_small_eligible(m, nn, 1, u->iters);
    const int blocks = muon_group_blocks(ly.out, ly.in, 1);
    const std::vector<int> one{(int)l};
    NsGroupRun r;
    r.w = ns_slots(u, (long)l);
    {
      Span sp(u, 6, st, 0);
      rc = launch_muon_x0(
          muon_args(u, one, 0, u->ns.ldx, [&](int) { return own ? r.w.X0 : (__nv_bfloat16*)nullptr; },
                    [&](int) { return (const float*)u->xres[l]; }),
          blocks, u->cc, d.mu, own && !small ? u->ns.part : nullptr, st);
      if (!rc && own && !small) rc = launch_muon_scale(u->ns.part, blocks, 1, d.eps, u->ns_scale + 2 * l, st);
    }
    if (rc) return rc;
    if (!own) continue;
    r.m = m;
    r.n = nn;
    r.batch = 1;
    r.ldx = u->ns.ldx;
    r.xbs = (long)m * u->ns.ldx;
    r.out = u->xres[l];
    r.ld_out = nn;
    r.obs = (long)m * nn;
    r.small = small;
    r.scale = u->ns_scale + 2 * l;
    runs.push_back(r);
    ns_flops += (double)u->iters * (4.0 * m * (double)m * nn + 2.0 * m * (double)m * m);
  }
  if (!runs.empty()) {
    Span sp(u, 4, st, ns_flops);
    rc = ns_run_groups(u, runs, st);
    if (rc) return rc;
  }
  {
    Span sp(u, 7, st, 0);
    std::vector<float*> bufs;
    std::vector<size_t> counts;
    std::vector<int> roots;
    for (size_t l = 0; l < u->layers.size(); l++) {
      bufs.push_back(u->xres[l]);
      counts.push_back((size_t)u->layers[l].out * u->layers[l].in);
      roots.push_back(u->owner[l]);
    }
    rc = comm_broadcast_group(d.comm, bufs, counts, roots, st);
    if (rc) return rc;
  }
  for (const auto& grp : u->ns_groups) {
    const Layer& g0 = u->layers[grp[0]];
    const int nn = std::max(g0.out, g0.in);
    const int blocks = muon_group_blocks(g0.out, g0.in, (int)grp.size());
    Span sp(u, 6, st, 0);
    for (int q0 = 0; q0 < (int)grp.size() && !rc; q0 += kMuonGroupMax)
      rc = launch_muon_finalize(muon_args(u, grp, q0, nn, [](int) { return (__nv_bfloat16*)nullptr; },
                                          [&](int q) { return (const float*)u->xres[grp[q]]; }),
                                blocks, lr, d.wd, d.mu, muon_shape_scale(g0), u->cc, st);
    if (rc) return rc;
  }
  return PL_OK;
}

// Data parallel: the summed gradient of layer l's block [W_l | b_l] (contiguous in the flat layout) is
// all-reduced on the comm stream once the compute stream has finished it. b_l is complete before
// W_l: the head's bias in the PPO epilogue, every other bias in the data-gradient epilogue of the layer
// above. The compute stream only waits for the all-reduces before the gradient norm (comm_wait).
static int comm_block(pl_update* u, int l, cudaStream_t st) {
  const Layer& ly = u->layers[l];
  const size_t n = (size_t)ly.out * ly.in + (size_t)ly.out;
  PL_CUDA(cudaEventRecord(u->aev[l], st));
  PL_CUDA(cudaStreamWaitEvent(u->ast, u->aev[l], 0));
  if (u->prof) {
    while (u->comm_ev.size() <= u->comm_ev_used) {
      cudaEvent_t a, b;
      cudaEventCreate(&a);
      cudaEventCreate(&b);
      u->comm_ev.push_back({a, b});
      u->comm_ev_bytes.push_back(0);
    }
    cudaEventRecord(u->comm_ev[u->comm_ev_used].first, u->ast);
  }
  int rc = comm_allreduce_f32(u->d.comm, u->grad + ly.oW, n, u->ast);
  if (u->prof) {
    cudaEventRecord(u->comm_ev[u->comm_ev_used].second, u->ast);
    u->comm_ev_bytes[u->comm_ev_used] = (double)n * sizeof(float);
    u->comm_ev_used++;
  }
  return rc;
}
static int comm_wait(pl_update* u, cudaStream_t st) {
  const int nl = (int)u->layers.size();
  PL_CUDA(cudaEventRecord(u->aev[nl], u->ast));
  Span sp(u, 7, st, 0);  // time the compute stream is held by the collectives it could not hide
  PL_CUDA(cudaStreamWaitEvent(st, u->aev[nl], 0));
  return PL_OK;
}

// The minibatch's rows of the resident columns (row k = column row idx[k]; its observation row is
// oidx[k] when obs is not in column order; xdirect: the observation rows are already contiguous and
// only the scalars are gathered), with the advantage statistics of the minibatch (all ranks' rows
// under data parallelism).
static int gather_step(pl_update* u, const int* idx, const int* oidx, const void* xdirect, int Nmb, cudaStream_t st) {
  const bool fast = u->fast;
  int rc = launch_gather(fast, idx, Nmb, xdirect ? nullptr : u->obs, fast ? u->Dp : (int)u->d.D, u->X, u->act_c,
                         u->adv_c, u->ret_c, u->olp_c, u->ov_c, u->mb_act, u->mb_adv, u->mb_ret, u->mb_olp, u->mb_ov,
                         u->adv_part, u->ms, st, u->dp ? u->adv_sums : nullptr, fast ? oidx : nullptr);
  // data parallel: the normalisation statistics are those of the whole (all-rank) minibatch
  if (!rc && u->dp) rc = comm_allreduce_f64(u->d.comm, u->adv_sums, 3, st);
  if (!rc && u->dp) rc = launch_adv_ms_from_sums(u->adv_sums, u->ms, st);
  return rc;
}

// Minibatch m of epoch e: rows [lo, lo + Nmb) of that epoch's shuffle, mbSize = NT / numMB and the
// last minibatch taking the remainder (ffi/puffercuda.cu:1236-1241); false when it is empty. idx, oidx
// and xdirect are what gather_step reads for it.
struct MbRows {
  long lo = 0;
  int Nmb = 0;
  long nglob = 0;  // rows of the minibatch over all ranks
  const int* idx = nullptr;
  const int* oidx = nullptr;
  const void* xdirect = nullptr;
};
static bool minibatch_rows(const pl_update* u, size_t e, size_t m, MbRows* r) {
  const pl_update_desc& d = u->d;
  const long lo = (long)m * u->mbSize;
  long hi = (m + 1 == d.numMB) ? (long)d.NT : (long)(m + 1) * u->mbSize;
  if (hi > (long)d.NT) hi = (long)d.NT;
  if (hi <= lo) return false;
  long a = lo, b = hi;
  r->nglob = hi - lo;
  if (u->dp && u->split) {  // this rank's share of the one global minibatch
    a = lo + (hi - lo) * d.rank / d.world;
    b = lo + (hi - lo) * (d.rank + 1) / d.world;
  } else if (u->dp) {  // every rank its own rollout: the all-rank minibatch is world equal parts
    r->nglob = (hi - lo) * d.world;
  }
  r->lo = a;
  r->Nmb = (int)(b - a);
  r->idx = u->perm + e * d.NT + a;
  r->oidx = nullptr;
  r->xdirect = nullptr;
  if (u->obs_epoch0) {
    if (e == 0)
      r->xdirect = (const __nv_bfloat16*)u->obs + a * u->Dp;
    else
      r->oidx = u->operm + e * d.NT + a;
  }
  return true;
}

// oidx: observation rows when obs is not in column order; xdirect: the minibatch's rows already
// contiguous in obs (no observation gather).
static int minibatch_fast(pl_update* u, const int* idx, const int* oidx, const void* xdirect, int Nmb, double lr,
                          bool last, cudaStream_t st) {
  const pl_update_desc& d = u->d;
  const int L = u->L;
  const int act = d.arch.act;
  const int mt = (int)ceil_div(Nmb, 128);
  int rc;
  {
    Span sp(u, 5, st, 0);
    rc = gather_step(u, idx, oidx, xdirect, Nmb, st);
  }
  if (rc) return rc;
  // ---- forward
  const void* xin = xdirect ? xdirect : u->X;
  const void* hin = xin;
  long ldin = u->Dp;
  for (int l = 0; l < L; l++) {
    const Layer& ly = u->layers[l];
    Operand A{hin, Nmb, ly.in, ldin, 1, 0};
    Operand B{u->Wb[l], ly.out, ly.in, ly.in_p, 1, 0};
    EpiArgs e{};
    e.out = u->Hs[l];
    e.ldo = u->Hp;
    e.out_rows = Nmb;
    e.out_cols = ly.out;
    e.bias = u->bf[l];
    e.out2 = u->Zs[l];
    e.ldo2 = u->Hp;
    e.act = act;
    {
      Span sp(u, 0, st, gf(Nmb, ly.out, ly.in));
      rc = gemm_launch(pick_bn(ly.out), EPI_FWD, false, false, A, B, Nmb, ly.out, ly.in, 1, e, st);
    }
    if (rc) return rc;
    hin = u->Hs[l];
    ldin = u->Hp;
  }
  // ---- PPO head: logits + value -> objective gradient dOut
  const Layer& hd = u->layers[L];
  if (u->head_mode != 0) {
    // wide heads: fp32 logits from a plain GEMM, then the row kernel (objective gradient, column
    // partial sums for the bias gradient, loss sums)
    rc = launch_gather_rows_f32(idx, Nmb, u->actw_c, u->W, u->mb_actw, st);
    if (rc) return rc;
    Operand A{hin, Nmb, hd.in, ldin, 1, 0};
    Operand B{u->Wb[L], hd.out, hd.in, hd.in_p, 1, 0};
    EpiArgs e{};
    e.out = u->Outw;
    e.ldo = u->Op;
    e.out_rows = Nmb;
    e.out_cols = hd.out;
    e.alpha = 1.f;
    {
      Span sp(u, 1, st, gf(Nmb, hd.out, hd.in));
      rc = gemm_launch(128, EPI_F32, false, false, A, B, Nmb, hd.out, hd.in, 1, e, st);
      if (!rc)
        rc = launch_ppo_rows_wide(true, u->Outw, u->Op, u->bf[L], Nmb, u->O, u->Op, u->head_mode, u->W, u->hs_dev,
                                  u->mb_actw, u->mb_adv, u->grad_only ? nullptr : u->ms, u->mb_ret, u->mb_olp,
                                  u->mb_ov, (float)d.vfCoef, (float)d.entCoef, (float)d.clipEps, (float)d.vfClip,
                                  kContLogStdLo, kContLogStdHi, u->dOut, u->colpart,
                                  last && u->loss_on ? u->loss_part : nullptr, st);
    }
    if (rc) return rc;
    {
      Span sp(u, 6, st, 0);
      rc = launch_colsum_reduce(u->colpart, mt, u->Op, hd.out, u->grad + hd.ob, st);
    }
    if (rc) return rc;
  } else {
    Operand A{hin, Nmb, hd.in, ldin, 1, 0};
    Operand B{u->Wb[L], hd.out, hd.in, hd.in_p, 1, 0};
    EpiArgs e{};
    e.out = u->dOut;
    e.ldo = u->Op;
    e.out_rows = Nmb;
    e.out_cols = hd.out;
    e.bias = u->bf[L];
    e.colsum = u->colpart;
    e.ld_colsum = u->Op;
    e.act_idx = u->mb_act;
    e.adv = u->mb_adv;
    e.adv_ms = u->grad_only ? nullptr : u->ms;
    e.ret = u->mb_ret;
    e.olp = u->mb_olp;
    e.ov = u->mb_ov;
    e.A = (int)d.A;
    e.vf = (float)d.vfCoef;
    e.ent = (float)d.entCoef;
    e.clip = (float)d.clipEps;
    e.vfclip = (float)d.vfClip;
    e.loss_part = last && u->loss_on ? u->loss_part : nullptr;
    {
      Span sp(u, 1, st, gf(Nmb, hd.out, hd.in));
      rc = gemm_launch(u->Op, EPI_PPO, false, false, A, B, Nmb, hd.out, hd.in, 1, e, st);
    }
    if (rc) return rc;
    {
      Span sp(u, 6, st, 0);
      rc = launch_colsum_reduce(u->colpart, mt, u->Op, hd.out, u->grad + hd.ob, st);
    }
    if (rc) return rc;
  }
  // ---- backward
  const void* dcur = u->dOut;
  long ldd = u->Op;
  int dsel = 0;
  for (int l = L; l >= 0; l--) {
    const Layer& ly = u->layers[l];
    const void* hprev = l == 0 ? xin : u->Hs[l - 1];
    const long ldprev = l == 0 ? u->Dp : u->Hp;
    {
      Span sp(u, 3, st, gf(ly.out, ly.in, Nmb));
      rc = wgrad_fast(u, dcur, ldd, ly.out, hprev, ldprev, ly.in, Nmb, u->grad + ly.oW, st);
    }
    if (!rc && u->dp && u->overlap && !u->grad_only) rc = comm_block(u, l, st);
    if (rc) return rc;
    if (l == 0) break;
    // dZ_{l-1} = (dcur W_l) * act'(Z_{l-1})
    const Layer& lp = u->layers[l - 1];
    Operand A{dcur, Nmb, ly.out, ldd, 1, 0};
    Operand B{u->Wb[l], ly.out, ly.in, ly.in_p, 1, 0};  // MN-major: rows = K (= out), cols = N (= in)
    EpiArgs e{};
    e.out = u->dZ[dsel];
    e.ldo = u->Hp;
    e.out_rows = Nmb;
    e.out_cols = lp.out;
    e.aux = (const __nv_bfloat16*)(act == 1 ? u->Zs[l - 1] : u->Hs[l - 1]);
    e.ld_aux = u->Hp;
    e.act = act;
    e.colsum = u->colpart;
    e.ld_colsum = u->Hp;
    {
      Span sp(u, 2, st, gf(Nmb, lp.out, ly.out));
      rc = gemm_launch(pick_bn(lp.out), EPI_DGRAD, false, true, A, B, Nmb, lp.out, ly.out, 1, e, st);
    }
    if (rc) return rc;
    {
      Span sp(u, 6, st, 0);
      rc = launch_colsum_reduce(u->colpart, mt, u->Hp, lp.out, u->grad + lp.ob, st);
    }
    if (rc) return rc;
    dcur = u->dZ[dsel];
    ldd = u->Hp;
    dsel ^= 1;
  }
  if (u->grad_only) return PL_OK;
  const long Nglob = u->dp ? u->nglob : Nmb;
  if (u->dp) {
    // ---- data parallel: the gradient summed over ranks (the mean is over the all-rank minibatch)
    if (u->overlap) {
      rc = comm_wait(u, st);
    } else {
      Span sp(u, 7, st, 0);
      rc = comm_allreduce_f32(d.comm, u->grad, u->P, st);
    }
    if (rc) return rc;
  }
  // ---- clip to the mean gradient, then Muon on every layer
  {
    Span sp(u, 6, st, 0);
    rc = launch_gradnorm(u->grad, (long)u->P, 1.0 / (double)Nglob, d.maxGradNorm, u->gn_part, u->cc, st);
  }
  if (rc) return rc;
  if (u->dp) return muon_sharded(u, lr, st);
  // Muon per group of equal-shape layers: the Nesterov step writes the unscaled Newton-Schulz input
  // (and the sums of u^2 whose factor the first step applies, or the fused short-matrix kernel
  // normalises in place); the groups that take the persistent chain run in one launch, so that the
  // short dependent products of the small groups overlap the large group's; then one finalisation of
  // weights and biases per group
  const size_t ngr = u->ns_groups.size();
  std::vector<NsGroupRun> runs(ngr);
  std::vector<int> blocks(ngr);
  double ns_flops = 0.0;
  for (size_t gi = 0; gi < ngr; gi++) {
    const auto& grp = u->ns_groups[gi];
    const Layer& g0 = u->layers[grp[0]];
    const int m = std::min(g0.out, g0.in), nn = std::max(g0.out, g0.in);
    const int nb = (int)grp.size();
    const long s0 = u->ns_slot0[gi];
    const long xstride = (long)m * u->ns.ldx;  // one wide m x ldx matrix per batch slot
    NsGroupRun& r = runs[gi];
    r.w = ns_slots(u, s0);
    r.m = m;
    r.n = nn;
    r.batch = nb;
    r.ldx = u->ns.ldx;
    r.xbs = xstride;
    r.out = r.w.Xf;
    r.ld_out = u->ns.ldx;
    r.obs = xstride;
    r.small = ns_small_eligible(m, nn, nb, u->iters);
    r.scale = u->ns_scale + 2 * s0;
    blocks[gi] = muon_group_blocks(g0.out, g0.in, nb);
    // algorithmic Newton-Schulz flops per step and matrix: 4 m^2 n + 2 m^3
    ns_flops += (double)nb * u->iters * (4.0 * m * (double)m * nn + 2.0 * m * (double)m * m);
    Span sp(u, 6, st, 0);
    for (int q0 = 0; q0 < nb && !rc; q0 += kMuonGroupMax)
      rc = launch_muon_x0(muon_args(u, grp, q0, u->ns.ldx, [&](int q) { return r.w.X0 + q * xstride; },
                                    [&](int q) { return (const float*)(r.w.Xf + q * xstride); }),
                          blocks[gi], u->cc, d.mu, r.small ? nullptr : u->ns.part + (long)q0 * blocks[gi], st);
    if (!rc && !r.small) rc = launch_muon_scale(u->ns.part, blocks[gi], nb, d.eps, r.scale, st);
    if (rc) return rc;
  }
  {
    Span sp(u, 4, st, ns_flops);
    rc = ns_run_groups(u, runs, st);
  }
  if (rc) return rc;
  for (size_t gi = 0; gi < ngr; gi++) {
    const auto& grp = u->ns_groups[gi];
    const Layer& g0 = u->layers[grp[0]];
    const long xstride = (long)std::min(g0.out, g0.in) * u->ns.ldx;
    const NsWork& w = runs[gi].w;
    Span sp(u, 6, st, 0);
    for (int q0 = 0; q0 < (int)grp.size() && !rc; q0 += kMuonGroupMax)
      rc = launch_muon_finalize(muon_args(u, grp, q0, u->ns.ldx, [&](int q) { return w.X0 + q * xstride; },
                                          [&](int q) { return (const float*)(w.Xf + q * xstride); }),
                                blocks[gi], lr, d.wd, d.mu, muon_shape_scale(g0), u->cc, st);
    if (rc) return rc;
  }
  return PL_OK;
}

static int minibatch_tight(pl_update* u, const int* idx, int Nmb, double lr, bool last, cudaStream_t st) {
  (void)last;
  const pl_update_desc& d = u->d;
  const int L = u->L, act = d.arch.act, D = (int)d.D, H = (int)d.H, O = u->O;
  int rc = gather_step(u, idx, nullptr, nullptr, Nmb, st);
  if (rc) return rc;
  const float* hin = (const float*)u->X;
  int nin = D;
  for (int l = 0; l < L; l++) {
    // Z = hin W^T + b and H = act(Z) in the product's epilogue
    rc = launch_sgemm_bias_act(Nmb, H, nin, hin, nin, u->Wf[l], u->bf[l], (float*)u->Zs[l], (float*)u->Hs[l], act, st);
    if (rc) return rc;
    hin = (const float*)u->Hs[l];
    nin = H;
  }
  if (skinny_rows_ok(H, O)) {  // a few head outputs: one warp per row instead of 64 x 64 tiles
    rc = launch_skinny_rows(hin, Nmb, H, u->Wf[L], u->bf[L], O, u->Out, st);
  } else {
    rc = launch_sgemm(Nmb, O, H, hin, H, 1, u->Wf[L], H, 1, u->Out, O, 1.f, st);
    if (!rc) rc = launch_bias_act_f32(u->Out, nullptr, u->bf[L], Nmb, O, 0, st);
  }
  if (rc) return rc;
  if (u->head_mode != 0) {
    rc = launch_gather_rows_f32(idx, Nmb, u->actw_c, u->W, u->mb_actw, st);
    if (!rc)
      rc = launch_ppo_rows_wide(false, u->Out, O, nullptr, Nmb, O, O, u->head_mode, u->W, u->hs_dev, u->mb_actw,
                                u->mb_adv, u->grad_only ? nullptr : u->ms, u->mb_ret, u->mb_olp, u->mb_ov,
                                (float)d.vfCoef, (float)d.entCoef, (float)d.clipEps, (float)d.vfClip, kContLogStdLo,
                                kContLogStdHi, u->dOut, u->colpart, nullptr, st);
  } else {
    rc = launch_ppo_rows_f32(u->Out, Nmb, (int)d.A, u->mb_act, u->mb_adv, u->grad_only ? nullptr : u->ms, u->mb_ret,
                             u->mb_olp, u->mb_ov, (float)d.vfCoef, (float)d.entCoef, (float)d.clipEps,
                             (float)d.vfClip, (float*)u->dOut, nullptr, nullptr, st);
  }
  if (rc) return rc;
  const float* dcur = (const float*)u->dOut;
  int nd = O;
  int dsel = 0;
  for (int l = L; l >= 0; l--) {
    const Layer& ly = u->layers[l];
    const float* hprev = l == 0 ? (const float*)u->X : (const float*)u->Hs[l - 1];
    // dW[o, i] = sum_n dcur[n, o] hprev[n, i] and the bias gradient db[o] = sum_n dcur[n, o], as one
    // split-K product with a column of ones
    rc = launch_wgrad_bias_f32(ly.out, ly.in, Nmb, dcur, nd, hprev, ly.in, u->grad + ly.oW, u->grad + ly.ob,
                               u->splitk, (long)u->splitk_elems, st);
    if (rc) return rc;
    if (l == 0) break;
    // dZ_{l-1}[n, i] = (sum_o dcur[n, o] W[o, i]) * act'(Z_{l-1}[n, i])
    float* dn = (float*)u->dZ[dsel];
    rc = launch_sgemm_act_grad(Nmb, ly.in, ly.out, dcur, nd, u->Wf[l], (const float*)u->Zs[l - 1], dn, act, st);
    if (rc) return rc;
    dcur = dn;
    nd = ly.in;
    dsel ^= 1;
  }
  if (u->grad_only) return PL_OK;
  const long Nglob = u->dp ? u->nglob : Nmb;
  if (u->dp) {
    rc = comm_allreduce_f32(d.comm, u->grad, u->P, st);
    if (rc) return rc;
  }
  rc = launch_gradnorm(u->grad, (long)u->P, 1.0 / (double)Nglob, d.maxGradNorm, u->gn_part, u->cc, st);
  if (rc) return rc;
  // f64 tight Muon (the parity tier runs it redundantly on every rank); the clip scale stays on the
  // device (u->cc[0]), read there by the Muon kernels. Small layers: one launch for every matrix and
  // bias, which also refreshes the f32 copies.
  if (u->exact_group.size() == u->layers.size())
    return muon_group_exact(u->exact_group.data(), (int)u->exact_group.size(), u->pm, (long)u->P, u->grad, lr, d.wd,
                            d.mu, d.eps, u->iters, u->cc, st);
  double* g64 = u->stage;  // P <= stage size is checked at creation
  rc = launch_f32_to_f64(u->grad, (long)u->P, g64, st);
  if (rc) return rc;
  for (size_t l = 0; l < u->layers.size(); l++) {
    const Layer& ly = u->layers[l];
    rc = muon_mat_exact(ly.out, ly.in, u->pm + ly.oW, u->pm + u->P + ly.oW, g64 + ly.oW, 0.0, lr, d.wd, d.mu, d.eps,
                        u->iters, u->exact_ws, st, u->cc);
    if (rc) return rc;
    rc = stepvec_launch(u->pm + ly.ob, u->pm + u->P + ly.ob, g64 + ly.ob, lr, d.wd, d.mu, 0.0, ly.out, st, u->cc);
    if (rc) return rc;
  }
  return refresh_shadows(u, st);
}

static int reduce_losses(pl_update* u, int Nmb, cudaStream_t st) {
  const int mt = (int)ceil_div(Nmb, 128);
  std::vector<float> h((size_t)mt * 8);
  PL_CUDA(cudaMemcpyAsync(h.data(), u->loss_part, sizeof(float) * h.size(), cudaMemcpyDeviceToHost, st));
  PL_CUDA(cudaStreamSynchronize(st));
  double s[6] = {0, 0, 0, 0, 0, 0};
  for (int t = 0; t < mt; t++)
    for (int q = 0; q < 6; q++) s[q] += h[(size_t)t * 8 + q];
  for (int q = 0; q < 6; q++) s[q] /= (double)Nmb;
  const pl_update_desc& d = u->d;
  // [policy, value, entropy, total, old_kl, kl, clipfrac]
  u->losses[0] = s[0];
  u->losses[1] = s[1];
  u->losses[2] = s[2];
  u->losses[3] = s[0] + d.vfCoef * s[1] - d.entCoef * s[2];
  u->losses[4] = s[4];
  u->losses[5] = s[3];
  u->losses[6] = s[5];
  std::lock_guard<std::mutex> g(g_mu);
  memcpy(g_losses, u->losses, sizeof(g_losses));
  return PL_OK;
}

}  // namespace

// ================================================================================ C ABI
extern "C" {

size_t pl_mlp_param_count(size_t D, size_t H, size_t A, size_t L) {
  if (L == 0) L = 1;
  return H * D + H + (L - 1) * (H * H + H) + (A + 1) * H + A + 1;
}

int pl_update_create(size_t handle, const pl_update_desc* desc, pl_update** out) {
  int rc = require_device();
  if (rc) return rc;
  PL_REQUIRE(desc && out, PL_ERR_INVALID, "pl_update_create: NULL argument");
  PL_REQUIRE(handle != 0, PL_ERR_INVALID, "pl_update_create: policy handle is 0");
  const pl_update_desc& d = *desc;
  PL_REQUIRE(d.NT > 0 && d.D > 0 && d.H > 0 && d.A > 0 && d.epochs > 0 && d.numMB > 0, PL_ERR_INVALID,
             "empty update shape (NT=%zu D=%zu H=%zu A=%zu epochs=%zu numMB=%zu)", d.NT, d.D, d.H, d.A, d.epochs,
             d.numMB);
  PL_REQUIRE(d.A + 1 <= 128, PL_ERR_UNSUPPORTED, "at most 127 discrete actions (A=%zu)", d.A);
  PL_REQUIRE(d.NT < (1ul << 31) && d.epochs * d.NT < (1ul << 31), PL_ERR_UNSUPPORTED, "NT x epochs must fit int32");
  PL_REQUIRE(d.arch.act == 0 || d.arch.act == 1, PL_ERR_INVALID, "activation must be 0 (ReLU) or 1 (GELU)");
  pl_update* u = new pl_update();
  u->d = d;
  u->fast = d.bf16 != 0;
  cudaGetDevice(&u->dev);
  u->pm = (double*)handle;
  if (d.arch.ns_coeffs && d.arch.ns_iters) {
    u->coeffs.assign(d.arch.ns_coeffs, d.arch.ns_coeffs + 3 * d.arch.ns_iters);
    u->iters = (int)d.arch.ns_iters;
  } else {
    u->coeffs.assign(&kMuonCoeffs[0][0], &kMuonCoeffs[0][0] + 15);
    u->iters = 5;
  }
  build_layout(u);
  u->dp = d.world > 1;
  if (u->dp) {
    if (!d.comm || d.rank < 0 || d.rank >= d.world || pl_comm_aborted(d.comm) != 0) {
      delete u;
      return set_error(PL_ERR_INVALID, "data-parallel session needs a live communicator from pl_comm_create and "
                                       "0 <= rank < world");
    }
    std::vector<size_t> rows, cols;
    for (auto& ly : u->layers) {
      rows.push_back((size_t)ly.out);
      cols.push_back((size_t)ly.in);
    }
    u->owner.assign(u->layers.size(), 0);
    pl_muon_shard_plan(rows.data(), cols.data(), rows.size(), d.world, u->owner.data());
    u->overlap = g_dp_overlap;
    cudaStreamCreateWithFlags(&u->ast, cudaStreamNonBlocking);
    u->aev.resize(u->layers.size() + 1);
    for (auto& e : u->aev) cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
  } else {
    u->owner.assign(u->layers.size(), 0);
  }
  rc = alloc_session(u);
  if (!rc && !u->fast && u->stage_elems < u->P) rc = set_error(PL_ERR_UNSUPPORTED, "tight tier staging too small");
  if (!rc) rc = refresh_shadows(u, 0);
  if (!rc) rc = (cudaDeviceSynchronize() == cudaSuccess) ? PL_OK : check_cuda(cudaGetLastError(), "session init");
  if (rc) {
    free_all(u);
    delete u;
    return rc;
  }
  *out = u;
  return PL_OK;
}

int pl_update_destroy(pl_update* u) {
  if (!u) return PL_OK;
  cudaDeviceSynchronize();
  for (cudaEvent_t e : u->ev) cudaEventDestroy(e);
  for (cudaEvent_t e : u->aev) cudaEventDestroy(e);
  for (auto& p : u->comm_ev) {
    cudaEventDestroy(p.first);
    cudaEventDestroy(p.second);
  }
  if (u->ast) cudaStreamDestroy(u->ast);
  if (u->cev) cudaEventDestroy(u->cev);
  if (u->sev) cudaEventDestroy(u->sev);
  if (u->cst) cudaStreamDestroy(u->cst);
  u->hstage.release();
  free_all(u);
  delete u;
  return PL_OK;
}

uint64_t pl_update_last_launches(const pl_update* u) { return u ? u->launches : 0; }
uint64_t pl_update_last_upload_bytes(void) { return g_upload_bytes.load(); }

}  // extern "C"

// Uploads n doubles from host through the staging buffer into dst via `fn(stage, count, offset)`.
template <typename F>
static int staged(pl_update* u, const double* host, size_t n, cudaStream_t st, F fn) {
  for (size_t off = 0; off < n; off += u->stage_elems) {
    const size_t c = std::min(u->stage_elems, n - off);
    PL_CUDA(cudaMemcpyAsync(u->stage, host + off, c * sizeof(double), cudaMemcpyHostToDevice, st));
    int rc = fn(u->stage, c, off);
    if (rc) return rc;
  }
  return PL_OK;
}

extern "C" {

int pl_update_set_head(pl_update* u, int mode, size_t W, const double* head_sizes) {
  PL_REQUIRE(u != nullptr, PL_ERR_INVALID, "pl_update_set_head: NULL session");
  PL_REQUIRE(mode >= 0 && mode <= 2, PL_ERR_INVALID, "pl_update_set_head: mode %d (0, 1 or 2)", mode);
  if (mode == 0) {
    u->head_mode = 0;
    return PL_OK;
  }
  const long A = (long)u->d.A;
  PL_REQUIRE(W >= 1 && W <= 4096, PL_ERR_INVALID, "pl_update_set_head: W = %zu", W);
  PL_REQUIRE(u->O <= 128, PL_ERR_UNSUPPORTED, "wide heads need A + 1 <= 128 outputs (A = %ld)", A);
  std::vector<int> hs((size_t)W, 0);
  if (mode == 1) {
    PL_REQUIRE(head_sizes != nullptr, PL_ERR_INVALID, "multi-discrete heads need their sizes");
    long sum = 0;
    for (size_t i = 0; i < W; i++) {
      hs[i] = (int)head_sizes[i];
      PL_REQUIRE(hs[i] >= 1, PL_ERR_INVALID, "head %zu has size %d", i, hs[i]);
      sum += hs[i];
    }
    PL_REQUIRE(sum == A, PL_ERR_INVALID, "head sizes sum to %ld, the network has A = %ld logits", sum, A);
  } else {
    PL_REQUIRE((long)(2 * W) == A, PL_ERR_INVALID, "a Gaussian head of %zu dims needs A = %zu (got %ld)", W, 2 * W, A);
  }
  if (u->W != (int)W || !u->actw_c) {
    u->actw_c = dalloc<float>(u, (size_t)u->d.NT * W);
    u->mb_actw = dalloc<float>(u, (size_t)u->mbMax * W);
    u->hs_dev = dalloc<int>(u, W);
    if (u->fast && !u->Outw) u->Outw = dalloc<float>(u, (size_t)u->mbMax * u->Op);
    if (u->alloc_failed) return PL_ERR_NOMEM;
  }
  PL_CUDA(cudaMemcpy(u->hs_dev, hs.data(), sizeof(int) * W, cudaMemcpyHostToDevice));
  u->head_mode = mode;
  u->W = (int)W;
  return PL_OK;
}

}  // extern "C"

// defer: the observation rows are left on the host for pl_update_run to upload in the first epoch's
// order (the caller runs the update before touching them again).
static int set_columns(pl_update* u, const double* obs, const double* acts, const double* adv, const double* ret,
                       const double* olp, const double* oldVal, const double* perm, void* stream, bool defer) {
  PL_REQUIRE(u && obs && acts && adv && ret && olp && perm, PL_ERR_INVALID, "pl_update_set_columns: NULL column");
  u->pend_obs = u->pend_perm = nullptr;
  u->obs_epoch0 = false;
  PL_REQUIRE(!u->d.use_old_values || oldVal, PL_ERR_INVALID, "value clip needs the old-value column");
  cudaStream_t st = (cudaStream_t)stream;
  const pl_update_desc& d = u->d;
  const long NT = (long)d.NT;
  const int D = (int)d.D;
  // obs: in the bf16 tier the host threads round the rows to bf16 and a quarter of the f64 bytes
  // cross the host link (pinned double buffering, conversion of chunk k + 1 overlapping the copy of
  // chunk k); otherwise whole rows per chunk through the device staging buffer, converted there
  bool host_done = false;
  uint64_t bytes = 0;
  long dev_rows_n = 0;
  if (defer && u->fast && g_host_bf16 && d.D >= 64 && d.epochs > 0 && (size_t)NT * d.D >= ((size_t)1 << 20) &&
      u->hstage.init((size_t)16 << 20) == 0) {
    if (!u->operm) {
      u->pos0 = dalloc<int>(u, (size_t)NT);
      u->operm = dalloc<int>(u, (size_t)d.epochs * NT);
      if (!u->pos0 || !u->operm) return PL_ERR_NOMEM;
    }
    u->pend_obs = obs;
    u->pend_perm = perm;
    u->obs_epoch0 = true;
    bytes += (uint64_t)NT * u->Dp * 2;
    host_done = true;
  }
  if (!host_done && u->fast && g_host_bf16 && (size_t)NT * d.D >= ((size_t)1 << 20) &&
      u->hstage.init((size_t)16 << 20) == 0) {
    // from pinned memory a share of the rows also goes as f64 through the device staging buffer
    cudaPointerAttributes at{};
    const bool pinned = cudaPointerGetAttributes(&at, obs) == cudaSuccess && at.type == cudaMemoryTypeHost;
    cudaGetLastError();
    std::function<int(long, long)> dev;
    if (pinned)
      dev = [&](long r0, long nr) -> int {
        const long per = std::max<long>(1, (long)(u->stage_elems / d.D));
        for (long r = r0; r < r0 + nr; r += per) {
          const long n = std::min(per, r0 + nr - r);
          if (cudaMemcpyAsync(u->stage, obs + r * D, (size_t)n * D * sizeof(double), cudaMemcpyHostToDevice, st) !=
              cudaSuccess)
            return -1;
          bytes += (uint64_t)n * D * sizeof(double);
          dev_rows_n += n;
          if (launch_obs_to_bf16_f64(u->stage, n, D, u->Dp, (__nv_bfloat16*)u->obs + r * u->Dp, st) != PL_OK)
            return -1;
        }
        return 0;
      };
    if (upload_rows_bf16(u->hstage, obs, NT, D, u->Dp, u->obs, st, dev) != 0)
      return check_cuda(cudaGetLastError(), "host bf16 observation upload");
    bytes += (uint64_t)(NT - dev_rows_n) * u->Dp * 2;
    host_done = true;
  }
  const size_t rows_per = std::max<size_t>(1, u->stage_elems / d.D);
  for (size_t r0 = 0; r0 < (size_t)NT && !host_done; r0 += rows_per) {
    const size_t nr = std::min(rows_per, (size_t)NT - r0);
    PL_CUDA(cudaMemcpyAsync(u->stage, obs + r0 * D, nr * D * sizeof(double), cudaMemcpyHostToDevice, st));
    bytes += (uint64_t)nr * D * sizeof(double);
    int rc = u->fast ? launch_obs_to_bf16_f64(u->stage, (long)nr, D, u->Dp, (__nv_bfloat16*)u->obs + r0 * u->Dp, st)
                     : launch_obs_to_f32_f64(u->stage, (long)nr * D, (float*)u->obs + r0 * D, st);
    if (rc) return rc;
  }
  PL_CUDA(cudaMemcpyAsync(u->adv_c, adv, NT * sizeof(double), cudaMemcpyHostToDevice, st));
  bytes += (uint64_t)NT * sizeof(double);
  if (u->head_mode != 0) {
    // wide action rows (NT x W) -> fp32 through staging; the categorical column is unused
    const size_t n = (size_t)NT * u->W;
    for (size_t off = 0; off < n; off += u->stage_elems) {
      const size_t c = std::min(u->stage_elems, n - off);
      PL_CUDA(cudaMemcpyAsync(u->stage, acts + off, c * 8, cudaMemcpyHostToDevice, st));
      bytes += c * 8;
      int rc = launch_f64_to_f32_rows(u->stage, (long)c, u->actw_c + off, st);
      if (rc) return rc;
    }
    acts = ret;  // the column pass below then fills the unused integer column from ret
  }
  // act/ret/olp/ov -> int32 / f32 through staging (4 columns)
  double* s = u->stage;
  const size_t per = u->stage_elems / 4;
  for (size_t off = 0; off < (size_t)NT; off += per) {
    const size_t c = std::min(per, (size_t)NT - off);
    PL_CUDA(cudaMemcpyAsync(s, acts + off, c * 8, cudaMemcpyHostToDevice, st));
    PL_CUDA(cudaMemcpyAsync(s + per, ret + off, c * 8, cudaMemcpyHostToDevice, st));
    PL_CUDA(cudaMemcpyAsync(s + 2 * per, olp + off, c * 8, cudaMemcpyHostToDevice, st));
    if (u->ov_c) PL_CUDA(cudaMemcpyAsync(s + 3 * per, oldVal + off, c * 8, cudaMemcpyHostToDevice, st));
    bytes += c * 8 * (u->ov_c ? 4 : 3);
    int rc = launch_columns(s, s + per, s + 2 * per, u->ov_c ? s + 3 * per : nullptr, (long)c, u->act_c + off,
                            u->ret_c + off, u->olp_c + off, u->ov_c ? u->ov_c + off : nullptr, st);
    if (rc) return rc;
  }
  bytes += (uint64_t)d.epochs * d.NT * sizeof(double);
  g_upload_bytes.store(bytes);
  int rc = staged(u, perm, d.epochs * d.NT, st, [&](double* sp, size_t c, size_t off) {
    return launch_perm(sp, (long)c, u->perm + off, st);
  });
  if (!rc && u->obs_epoch0) rc = launch_perm_positions(u->perm, NT, (long)(d.epochs * NT), u->pos0, u->operm, st);
  return rc;
}

extern "C" {

int pl_update_set_columns(pl_update* u, const double* obs, const double* acts, const double* adv, const double* ret,
                          const double* olp, const double* oldVal, const double* perm, void* stream) {
  return set_columns(u, obs, acts, adv, ret, olp, oldVal, perm, stream, false);
}

int pl_update_set_columns_dev(pl_update* u, const float* obs, const double* acts, const double* adv,
                              const double* ret, const double* olp, const double* oldVal, const double* perm,
                              void* stream) {
  // adv / ret / oldVal may be NULL when pl_update_set_advantages_dev provides them
  PL_REQUIRE(u && obs && acts && olp && perm, PL_ERR_INVALID, "pl_update_set_columns_dev: NULL column");
  u->pend_obs = u->pend_perm = nullptr;
  u->obs_epoch0 = false;
  cudaStream_t st = (cudaStream_t)stream;
  const pl_update_desc& d = u->d;
  const long NT = (long)d.NT;
  int rc;
  if (u->fast)
    rc = launch_obs_to_bf16_f32(obs, NT, (int)d.D, u->Dp, (__nv_bfloat16*)u->obs, st);
  else {
    PL_CUDA(cudaMemcpyAsync(u->obs, obs, sizeof(float) * NT * d.D, cudaMemcpyDeviceToDevice, st));
    rc = PL_OK;
  }
  if (rc) return rc;
  if (adv) PL_CUDA(cudaMemcpyAsync(u->adv_c, adv, NT * sizeof(double), cudaMemcpyDeviceToDevice, st));
  if (u->head_mode != 0) {
    rc = launch_f64_to_f32_rows(acts, NT * u->W, u->actw_c, st);
    if (rc) return rc;
    acts = olp;  // the integer column is unused with wide heads
  }
  rc = launch_columns(acts, ret, olp, (u->ov_c && oldVal) ? oldVal : nullptr, NT, u->act_c, ret ? u->ret_c : nullptr,
                      u->olp_c, (u->ov_c && oldVal) ? u->ov_c : nullptr, st);
  if (rc) return rc;
  return launch_perm(perm, (long)(d.epochs * NT), u->perm, st);
}

__global__ void adv_columns_kernel(const float* __restrict__ a, const float* __restrict__ val, long n, double* adv_c,
                                   float* ret_c, float* ov_c) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float ad = a[i];
    adv_c[i] = (double)ad;
    ret_c[i] = ad + val[i];
    if (ov_c) ov_c[i] = val[i];
  }
}

int pl_update_set_advantages_dev(pl_update* u, const float* rew, const float* val, const float* term,
                                 const float* imp, size_t T, double gamma, double lam, double rhoClip, double cClip,
                                 void* stream) {
  PL_REQUIRE(u && rew && val && term && T > 0, PL_ERR_INVALID, "pl_update_set_advantages_dev: bad arguments");
  PL_REQUIRE(u->d.NT % T == 0, PL_ERR_INVALID, "NT=%zu is not a whole number of T=%zu segments", u->d.NT, T);
  cudaStream_t st = (cudaStream_t)stream;
  if (!u->adv_f) {
    u->adv_f = dalloc<float>(u, u->d.NT);
    if (!u->adv_f) return PL_ERR_NOMEM;
  }
  int rc = pl_vtrace_f32_dev(rew, val, term, imp, nullptr, u->d.NT / T, T, gamma, lam, rhoClip, cClip, u->adv_f,
                             nullptr, stream);
  if (rc) return rc;
  adv_columns_kernel<<<(unsigned)std::min<long>(ceil_div((long)u->d.NT, 256), 148 * 16), 256, 0, st>>>(
      u->adv_f, val, (long)u->d.NT, u->adv_c, u->ret_c, u->ov_c);
  count_launch();
  PL_LAUNCH("adv_columns_kernel");
  return PL_OK;
}

int pl_update_profile(pl_update* u, int on) {
  PL_REQUIRE(u != nullptr, PL_ERR_INVALID, "pl_update_profile: NULL session");
  if (on && !u->prof) {
    for (int i = 0; i < 8; i++) u->prof_ms[i] = u->prof_flops[i] = u->prof_launch[i] = 0;
    u->ev_used = 0;
    u->ev_cls.clear();
    u->comm_ms = u->comm_bytes = u->comm_launches = 0;
    u->comm_ev_used = 0;
  }
  u->prof = on != 0;
  return PL_OK;
}

int pl_update_profile_read(pl_update* u, double ms[8], double flops[8], double launches[8]) {
  PL_REQUIRE(u != nullptr, PL_ERR_INVALID, "pl_update_profile_read: NULL session");
  prof_collect(u);
  for (int i = 0; i < 8; i++) {
    if (ms) ms[i] = u->prof_ms[i];
    if (flops) flops[i] = u->prof_flops[i];
    if (launches) launches[i] = u->prof_launch[i];
  }
  return PL_OK;
}

int pl_update_comm_profile_read(pl_update* u, double* ms, double* bytes, double* launches) {
  PL_REQUIRE(u != nullptr, PL_ERR_INVALID, "pl_update_comm_profile_read: NULL session");
  prof_collect(u);
  if (ms) *ms = u->comm_ms;
  if (bytes) *bytes = u->comm_bytes;
  if (launches) *launches = u->comm_launches;
  return PL_OK;
}

int pl_update_split_minibatch(pl_update* u, int on) {
  PL_REQUIRE(u != nullptr, PL_ERR_INVALID, "pl_update_split_minibatch: NULL session");
  if (on && u->dp)
    PL_REQUIRE(u->mbSize >= u->d.world, PL_ERR_INVALID,
               "split minibatch: %ld rows per minibatch for %d ranks", u->mbSize, u->d.world);
  u->split = on != 0;
  return PL_OK;
}

int pl_update_run(pl_update* u, double lr, void* stream) {
  PL_REQUIRE(u != nullptr, PL_ERR_INVALID, "pl_update_run: NULL session");
  PL_REQUIRE(!u->dp || pl_comm_aborted(u->d.comm) == 0, PL_ERR_COMM,
             "pl_update_run: the session's communicator was aborted (or is not one of this library)");
  cudaStream_t st = (cudaStream_t)stream;
  const pl_update_desc& d = u->d;
  const uint64_t l0 = pl_kernel_launch_count();
  u->loss_on = g_loss_on;
  int lastNmb = 0;
  if (!u->fast) {  // the f64 Newton-Schulz table of the tight tier, once per update
    int rc0 = set_ns_coeffs(u->coeffs.data(), u->iters, st);
    if (rc0) return rc0;
  }
  // pending host observations: each first-epoch minibatch's rows are rounded and copied on the copy
  // stream just before its kernels are queued, and the compute stream waits for exactly those rows
  const bool upl = u->pend_obs != nullptr;
  struct Done {
    pl_update* u;
    ~Done() { u->pend_obs = u->pend_perm = nullptr; }
  } done{u};
  if (upl) {
    if (!u->cst) PL_CUDA(cudaStreamCreateWithFlags(&u->cst, cudaStreamNonBlocking));
    if (!u->cev) PL_CUDA(cudaEventCreateWithFlags(&u->cev, cudaEventDisableTiming));
    if (!u->sev) PL_CUDA(cudaEventCreateWithFlags(&u->sev, cudaEventDisableTiming));
    PL_CUDA(cudaEventRecord(u->sev, st));  // earlier work on obs is done before it is overwritten
    PL_CUDA(cudaStreamWaitEvent(u->cst, u->sev, 0));
  }
  for (size_t e = 0; e < d.epochs; e++)
    for (size_t m = 0; m < d.numMB; m++) {
      MbRows mr;
      if (!minibatch_rows(u, e, m, &mr)) continue;
      u->nglob = mr.nglob;
      // the first-epoch upload brings every row of the minibatch (later epochs read them all)
      const long lo = (long)m * u->mbSize, hi = (m + 1 == d.numMB) ? (long)d.NT : (long)(m + 1) * u->mbSize;
      const int Nmb = mr.Nmb;
      const bool last = (e + 1 == d.epochs) && (m + 1 == d.numMB);
      if (upl && e == 0) {
        const int r = upload_rows_bf16_order(u->hstage, u->pend_obs, u->pend_perm, (long)d.NT, lo, hi, (int)d.D, u->Dp,
                                             u->obs, u->cst);
        PL_REQUIRE(r != -2, PL_ERR_INVALID, "shuffle entry is not a row index in [0, %zu)", d.NT);
        if (r) return check_cuda(cudaGetLastError(), "host bf16 observation upload");
        PL_CUDA(cudaEventRecord(u->cev, u->cst));
        PL_CUDA(cudaStreamWaitEvent(st, u->cev, 0));
      }
      int rc = u->fast ? minibatch_fast(u, mr.idx, mr.oidx, mr.xdirect, Nmb, lr, last, st)
                       : minibatch_tight(u, mr.idx, Nmb, lr, last, st);
      if (rc) return rc;
      lastNmb = Nmb;
    }
  u->launches = pl_kernel_launch_count() - l0;
  if (u->prof && u->ev_used > 16384) prof_collect(u);
  if (u->loss_on && u->fast && lastNmb > 0) return reduce_losses(u, lastNmb, st);
  return PL_OK;
}

extern "C" int pl_update_run_columns(pl_update* u, const double* obs, const double* acts, const double* adv,
                                     const double* ret, const double* olp, const double* oldVal, const double* perm,
                                     double lr, void* stream) {
  int rc = set_columns(u, obs, acts, adv, ret, olp, oldVal, perm, stream, true);
  return rc ? rc : pl_update_run(u, lr, stream);
}

// ---------------------------------------------------------------- policy handle
int pl_policy_load(const double* pm, size_t P, size_t* handle) {
  int rc = require_device();
  if (rc) return rc;
  PL_REQUIRE(pm && handle && P > 0, PL_ERR_INVALID, "pl_policy_load: bad arguments");
  double* d = nullptr;
  PL_CUDA(cudaMalloc(&d, 2 * P * sizeof(double)));
  cudaError_t e = cudaMemcpy(d, pm, 2 * P * sizeof(double), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return check_cuda(e, "pl_policy_load upload");
  }
  *handle = (size_t)d;
  return PL_OK;
}

int pl_policy_download(size_t handle, size_t P, double* pm_out) {
  PL_REQUIRE(handle && pm_out, PL_ERR_INVALID, "pl_policy_download: bad arguments");
  PL_CUDA(cudaDeviceSynchronize());
  PL_CUDA(cudaMemcpy(pm_out, (const void*)handle, 2 * P * sizeof(double), cudaMemcpyDeviceToHost));
  return PL_OK;
}

// ---------------------------------------------------------------- cached sessions for the
// reference-shaped entry points (one per handle and shape)
struct CachedSession {
  size_t handle;
  pl_update_desc d;
  std::vector<double> coeffs;
  pl_update* u;
};
static std::vector<CachedSession> g_sessions;

static bool same_desc(const pl_update_desc& a, const pl_update_desc& b) {
  return a.NT == b.NT && a.D == b.D && a.H == b.H && a.A == b.A && a.epochs == b.epochs && a.numMB == b.numMB &&
         a.arch.L == b.arch.L && a.arch.act == b.arch.act && a.bf16 == b.bf16 && a.use_old_values == b.use_old_values &&
         a.arch.ns_iters == b.arch.ns_iters;
}

static int session_for(size_t handle, const pl_update_desc& d, pl_update** out) {
  std::lock_guard<std::mutex> g(g_mu);
  std::vector<double> co;
  if (d.arch.ns_coeffs && d.arch.ns_iters) co.assign(d.arch.ns_coeffs, d.arch.ns_coeffs + 3 * d.arch.ns_iters);
  for (auto it = g_sessions.begin(); it != g_sessions.end(); ++it) {
    if (it->handle != handle) continue;
    if (same_desc(it->d, d) && it->coeffs == co) {
      it->u->d = d;  // hyperparameters may change between calls
      it->u->d.arch.ns_coeffs = nullptr;
      *out = it->u;
      return PL_OK;
    }
    pl_update_destroy(it->u);
    g_sessions.erase(it);
    break;
  }
  pl_update* u = nullptr;
  int rc = pl_update_create(handle, &d, &u);
  if (rc) return rc;
  u->d.arch.ns_coeffs = nullptr;
  g_sessions.push_back({handle, d, co, u});
  *out = u;
  return PL_OK;
}

int pl_policy_free(size_t handle) {
  if (!handle) return PL_OK;
  {
    std::lock_guard<std::mutex> g(g_mu);
    for (auto it = g_sessions.begin(); it != g_sessions.end();) {
      if (it->handle == handle) {
        pl_update_destroy(it->u);
        it = g_sessions.erase(it);
      } else
        ++it;
    }
  }
  PL_CUDA(cudaDeviceSynchronize());
  PL_CUDA(cudaFree((void*)handle));
  return PL_OK;
}

static int resident_update(size_t handle, const pl_mlp_arch* arch, const double* obs, const double* acts,
                           const double* adv, const double* ret, const double* olp, const double* oldVal,
                           size_t oldValN, const double* perm, size_t NT, size_t D, size_t H, size_t A, size_t epochs,
                           size_t numMB, double lr, double wd, double mu, double eps, double vfCoef, double entCoef,
                           double clipEps, double vfClip, double maxGradNorm, uint8_t bf16, bool grad_only,
                           float* grad_out, int head_mode = 0, size_t W = 1, const double* head_sizes = nullptr) {
  int rc = require_device();
  if (rc) return rc;
  pl_update_desc d{};
  d.NT = NT;
  d.D = D;
  d.H = H;
  d.A = A;
  d.epochs = epochs;
  d.numMB = numMB;
  if (arch) d.arch = *arch;
  if (d.arch.L == 0) d.arch.L = 1;
  d.wd = wd;
  d.mu = mu;
  d.eps = eps;
  d.vfCoef = vfCoef;
  d.entCoef = entCoef;
  d.clipEps = clipEps;
  d.vfClip = vfClip;
  d.maxGradNorm = maxGradNorm;
  d.bf16 = bf16;
  d.use_old_values = (vfClip > 0.0 && oldVal != nullptr && oldValN >= NT) ? 1 : 0;
  d.world = 1;
  pl_update* u = nullptr;
  rc = session_for(handle, d, &u);
  if (rc) return rc;
  u->grad_only = grad_only;
  rc = pl_update_set_head(u, head_mode, W, head_sizes);
  if (rc) return rc;
  rc = refresh_shadows(u, 0);
  if (rc) return rc;
  rc = set_columns(u, obs, acts, adv, ret, olp, d.use_old_values ? oldVal : nullptr, perm, nullptr, true);
  if (rc) return rc;
  rc = pl_update_run(u, lr, nullptr);
  if (rc) return rc;
  if (grad_only && grad_out) PL_CUDA(cudaMemcpy(grad_out, u->grad, sizeof(float) * u->P, cudaMemcpyDeviceToHost));
  PL_CUDA(cudaDeviceSynchronize());
  return device_error_check();
}

int pl_train_update_resident_deep(size_t handle, const pl_mlp_arch* arch, const double* obs, const double* acts,
                                  const double* adv, const double* ret, const double* olp, const double* oldVal,
                                  size_t oldValN, const double* perm, size_t NT, size_t D, size_t H, size_t A,
                                  size_t epochs, size_t numMB, double lr, double wd, double mu, double eps,
                                  double vfCoef, double entCoef, double clipEps, double vfClip, double maxGradNorm,
                                  uint8_t bf16, double* params0_out) {
  PL_REQUIRE(handle && obs && acts && adv && ret && olp && perm, PL_ERR_INVALID, "update: NULL argument");
  int rc = resident_update(handle, arch, obs, acts, adv, ret, olp, oldVal, oldValN, perm, NT, D, H, A, epochs, numMB, lr,
                           wd, mu, eps, vfCoef, entCoef, clipEps, vfClip, maxGradNorm, bf16, false, nullptr);
  if (rc) return rc;
  if (params0_out) PL_CUDA(cudaMemcpy(params0_out, (const void*)handle, sizeof(double), cudaMemcpyDeviceToHost));
  return PL_OK;
}

int pl_train_update_wide_resident(size_t handle, const double* obs, const double* acts, const double* adv,
                                  const double* ret, const double* olp, const double* oldVal, size_t oldValN,
                                  const double* perm, const double* head_sizes, size_t NT, size_t D, size_t H,
                                  size_t O, size_t W, uint32_t mode, size_t epochs, size_t numMB, double lr, double wd,
                                  double mu, double eps, double vfCoef, double entCoef, double clipEps, double vfClip,
                                  double maxGradNorm, uint8_t bf16, double* params0_out) {
  PL_REQUIRE(handle && obs && acts && adv && ret && olp && perm, PL_ERR_INVALID, "wide update: NULL argument");
  PL_REQUIRE(mode == 1 || mode == 2, PL_ERR_INVALID, "wide update: mode %u (1 multi-discrete, 2 Gaussian)", mode);
  PL_REQUIRE(O >= 2, PL_ERR_INVALID, "wide update: O = %zu", O);
  int rc = resident_update(handle, nullptr, obs, acts, adv, ret, olp, oldVal, oldValN, perm, NT, D, H, O - 1, epochs,
                           numMB, lr, wd, mu, eps, vfCoef, entCoef, clipEps, vfClip, maxGradNorm, bf16, false,
                           nullptr, (int)mode, W, head_sizes);
  if (rc) return rc;
  if (params0_out) PL_CUDA(cudaMemcpy(params0_out, (const void*)handle, sizeof(double), cudaMemcpyDeviceToHost));
  return PL_OK;
}

int pl_mlp_ppo_grad_wide(const double* params, const double* obs, const double* acts, const double* advs,
                         const double* rets, const double* oldlps, const double* oldVal, size_t N, size_t H, size_t D,
                         size_t O, size_t W, uint32_t mode, const double* head_sizes, double vfCoef, double entCoef,
                         double clipEps, double vfClip, uint8_t bf16, double* g) {
  PL_REQUIRE(params && obs && acts && advs && rets && oldlps && g, PL_ERR_INVALID, "wide gradient: NULL argument");
  PL_REQUIRE(mode == 1 || mode == 2, PL_ERR_INVALID, "wide gradient: mode %u (1 multi-discrete, 2 Gaussian)", mode);
  const size_t P = pl_mlp_param_count(D, H, O - 1, 1);
  std::vector<double> pm(2 * P, 0.0);
  memcpy(pm.data(), params, sizeof(double) * P);
  std::vector<double> perm(N);
  for (size_t i = 0; i < N; i++) perm[i] = (double)i;
  size_t h = 0;
  int rc = pl_policy_load(pm.data(), P, &h);
  if (rc) return rc;
  std::vector<float> gf(P);
  rc = resident_update(h, nullptr, obs, acts, advs, rets, oldlps, oldVal, oldVal ? N : 0, perm.data(), N, D, H, O - 1,
                       1, 1, 0.0, 0.0, 0.0, 1e-7, vfCoef, entCoef, clipEps, vfClip, 0.0, bf16, true, gf.data(),
                       (int)mode, W, head_sizes);
  pl_policy_free(h);
  if (rc) return rc;
  for (size_t i = 0; i < P; i++) g[i] = (double)gf[i];
  return PL_OK;
}

// One Muon step of the resident one-hidden-layer MLP from a raw summed gradient: the exact f64 tier
// (the reference's muon_mat_dev / k_stepvec, the same folds as muon_mat_cpu / stepvec_cpu with the
// gradient scale applied in the momentum update).
int pl_muon_step_mlp_resident(size_t handle, const double* gRaw, size_t H, size_t D, size_t O, double gscale,
                              double lr, double wd, double mu, double eps, double* params_out) {
  PL_REQUIRE(handle && gRaw, PL_ERR_INVALID, "pl_muon_step_mlp_resident: NULL argument");
  int rc = require_device();
  if (rc) return rc;
  const size_t P = H * D + H + O * H + O;
  double* pm = (double*)handle;
  double* g = (double*)scratch(23, sizeof(double) * P);
  double* ws = (double*)scratch(24, sizeof(double) * std::max(exact_ws_doubles((int)H, (int)D),
                                                               exact_ws_doubles((int)O, (int)H)));
  if (!g || !ws) return PL_ERR_NOMEM;
  PL_CUDA(cudaMemcpy(g, gRaw, sizeof(double) * P, cudaMemcpyHostToDevice));
  rc = set_ns_coeffs(&kMuonCoeffs[0][0], 5, 0);
  const size_t oW1 = 0, ob1 = H * D, oW2 = H * D + H, ob2 = H * D + H + O * H;
  if (!rc) rc = muon_mat_exact((int)H, (int)D, pm + oW1, pm + P + oW1, g + oW1, gscale, lr, wd, mu, eps, 5, ws, 0);
  if (!rc) rc = stepvec_launch(pm + ob1, pm + P + ob1, g + ob1, lr, wd, mu, gscale, (long)H, 0);
  if (!rc) rc = muon_mat_exact((int)O, (int)H, pm + oW2, pm + P + oW2, g + oW2, gscale, lr, wd, mu, eps, 5, ws, 0);
  if (!rc) rc = stepvec_launch(pm + ob2, pm + P + ob2, g + ob2, lr, wd, mu, gscale, (long)O, 0);
  if (rc) return rc;
  // sessions holding shadows of this handle refresh them at their next call (resident_update)
  if (params_out) PL_CUDA(cudaMemcpy(params_out, pm, sizeof(double) * P, cudaMemcpyDeviceToHost));
  PL_CUDA(cudaDeviceSynchronize());
  return device_error_check();
}

int pl_train_update_resident(size_t handle, const double* obs, const double* acts, const double* adv,
                             const double* ret, const double* olp, const double* oldVal, size_t oldValN,
                             const double* perm, size_t NT, size_t D, size_t H, size_t A, size_t epochs, size_t numMB,
                             double lr, double wd, double mu, double eps, double vfCoef, double entCoef,
                             double clipEps, double vfClip, double maxGradNorm, uint8_t bf16, double* params0_out) {
  return pl_train_update_resident_deep(handle, nullptr, obs, acts, adv, ret, olp, oldVal, oldValN, perm, NT, D, H, A,
                                       epochs, numMB, lr, wd, mu, eps, vfCoef, entCoef, clipEps, vfClip, maxGradNorm,
                                       bf16, params0_out);
}

int pl_train_update(const double* pm, const double* obs, const double* acts, const double* adv, const double* ret,
                    const double* olp, const double* perm, size_t NT, size_t D, size_t H, size_t A, size_t epochs,
                    size_t numMB, double lr, double wd, double mu, double eps, double vfCoef, double entCoef,
                    double clipEps, uint8_t bf16, double* pm_out) {
  PL_REQUIRE(pm && pm_out, PL_ERR_INVALID, "pl_train_update: NULL argument");
  const size_t P = pl_mlp_param_count(D, H, A, 1);
  size_t h = 0;
  int rc = pl_policy_load(pm, P, &h);
  if (rc) return rc;
  rc = pl_train_update_resident(h, obs, acts, adv, ret, olp, nullptr, 0, perm, NT, D, H, A, epochs, numMB, lr, wd, mu,
                                eps, vfCoef, entCoef, clipEps, 0.0, 0.0, bf16, nullptr);
  if (!rc) rc = pl_policy_download(h, P, pm_out);
  pl_policy_free(h);
  return rc;
}

int pl_train_step(const double* pm, const double* obs, const double* acts, const double* advRaw, const double* rets,
                  const double* oldlps, size_t N, size_t H, size_t D, size_t A, double lr, double wd, double mu,
                  double eps, double vfCoef, double entCoef, double clipEps, uint8_t bf16, double* pm_out) {
  std::vector<double> perm(N);
  for (size_t i = 0; i < N; i++) perm[i] = (double)i;
  return pl_train_update(pm, obs, acts, advRaw, rets, oldlps, perm.data(), N, D, H, A, 1, 1, lr, wd, mu, eps, vfCoef,
                         entCoef, clipEps, bf16, pm_out);
}

int pl_mlp_ppo_grad(const double* params, const double* obs, const double* acts, const double* advs,
                    const double* rets, const double* oldlps, size_t N, size_t H, size_t D, size_t A, double vfCoef,
                    double entCoef, double clipEps, uint8_t bf16, double* g) {
  PL_REQUIRE(params && g, PL_ERR_INVALID, "pl_mlp_ppo_grad: NULL argument");
  const size_t P = pl_mlp_param_count(D, H, A, 1);
  std::vector<double> pm(2 * P, 0.0);
  memcpy(pm.data(), params, P * sizeof(double));
  size_t h = 0;
  int rc = pl_policy_load(pm.data(), P, &h);
  if (rc) return rc;
  std::vector<double> perm(N);
  for (size_t i = 0; i < N; i++) perm[i] = (double)i;
  std::vector<float> gf(P);
  rc = resident_update(h, nullptr, obs, acts, advs, rets, oldlps, nullptr, 0, perm.data(), N, D, H, A, 1, 1, 0.0, 0.0,
                       0.0, 1e-7, vfCoef, entCoef, clipEps, 0.0, 0.0, bf16, true, gf.data());
  pl_policy_free(h);
  if (rc) return rc;
  for (size_t i = 0; i < P; i++) g[i] = (double)gf[i];
  return PL_OK;
}

// f64 sequential folds, one thread: bit-identical to normalizeAdv (Puffer/RL/NNTrain.lean:274-279).
}  // extern "C"

__global__ void adv_normalize_exact_kernel(const double* __restrict__ a, long n, double* out) {
  if (threadIdx.x || blockIdx.x) return;
  double s = 0.0;
  for (long i = 0; i < n; i++) s = __dadd_rn(s, a[i]);
  const double mean = __ddiv_rn(s, (double)n);
  double v = 0.0;
  for (long i = 0; i < n; i++) {
    const double d = __dsub_rn(a[i], mean);
    v = __dadd_rn(v, __dmul_rn(d, d));
  }
  const double den = __dadd_rn(__dsqrt_rn(__ddiv_rn(v, (double)n)), 1e-8);
  for (long i = 0; i < n; i++) out[i] = __ddiv_rn(__dsub_rn(a[i], mean), den);
}

extern "C" {

int pl_adv_normalize(const double* adv, size_t n, double* out) {
  int rc = require_device();
  if (rc) return rc;
  PL_REQUIRE(adv && out, PL_ERR_INVALID, "pl_adv_normalize: NULL buffer");
  if (n == 0) return PL_OK;
  double* d = (double*)scratch(2, 2 * n * sizeof(double));
  if (!d) return PL_ERR_NOMEM;
  PL_CUDA(cudaMemcpy(d, adv, n * 8, cudaMemcpyHostToDevice));
  adv_normalize_exact_kernel<<<1, 32>>>(d, (long)n, d + n);
  count_launch();
  PL_LAUNCH("adv_normalize_exact_kernel");
  PL_CUDA(cudaMemcpy(out, d + n, n * 8, cudaMemcpyDeviceToHost));
  return PL_OK;
}

}  // extern "C"

namespace pl {
// The one dashboard-loss channel every trainer writes (the MinGRU path included).
bool loss_channel_on() {
  std::lock_guard<std::mutex> g(g_mu);
  return g_loss_on;
}
void loss_channel_store(const double v[7]) {
  std::lock_guard<std::mutex> g(g_mu);
  memcpy(g_losses, v, sizeof(g_losses));
}
}  // namespace pl

extern "C" {

int pl_loss_enable(uint8_t on) {
  std::lock_guard<std::mutex> g(g_mu);
  g_loss_on = on != 0;
  return PL_OK;
}

int pl_read_losses(double out[7]) {
  PL_REQUIRE(out != nullptr, PL_ERR_INVALID, "pl_read_losses: NULL");
  std::lock_guard<std::mutex> g(g_mu);
  memcpy(out, g_losses, sizeof(g_losses));
  return PL_OK;
}

}  // extern "C"

// Test hook: 1 = in the bf16 tier, host observations are rounded to bf16 on the host threads before
// the copy (the default), 0 = f64 rows copied and converted on the device; a negative mode only
// queries. Returns the previous mode.
extern "C" int pl_test_host_bf16(int mode) {
  const int prev = g_host_bf16 ? 1 : 0;
  if (mode >= 0) g_host_bf16 = mode != 0;
  return prev;
}

// Test hook: the gather of minibatch (epoch, mb) exactly as pl_update_run runs it before that
// minibatch's forward pass, with its outputs copied to the host.
extern "C" int pl_test_update_gather(pl_update* u, size_t epoch, size_t mb, void* rows, size_t* row_elems, int* act,
                                     float* adv, float* ret, float* olp, float* ov, size_t* nmb, void* stream) {
  PL_REQUIRE(u && nmb, PL_ERR_INVALID, "pl_test_update_gather: NULL argument");
  PL_REQUIRE(epoch < u->d.epochs && mb < u->d.numMB, PL_ERR_INVALID, "pl_test_update_gather: no minibatch (%zu, %zu)",
             epoch, mb);
  PL_REQUIRE(u->pend_obs == nullptr, PL_ERR_INVALID, "pl_test_update_gather: observations not uploaded yet");
  cudaStream_t st = (cudaStream_t)stream;
  MbRows mr;
  *nmb = 0;
  if (!minibatch_rows(u, epoch, mb, &mr)) return PL_OK;
  u->nglob = mr.nglob;
  int rc = gather_step(u, mr.idx, mr.oidx, mr.xdirect, mr.Nmb, st);
  if (rc) return rc;
  PL_CUDA(cudaStreamSynchronize(st));
  const size_t re = u->fast ? (size_t)u->Dp : (size_t)u->d.D, es = u->fast ? 2 : 4;
  *nmb = (size_t)mr.Nmb;
  if (row_elems) *row_elems = re;
  const size_t n = (size_t)mr.Nmb;
  if (rows) PL_CUDA(cudaMemcpy(rows, mr.xdirect ? mr.xdirect : u->X, n * re * es, cudaMemcpyDeviceToHost));
  if (act) PL_CUDA(cudaMemcpy(act, u->mb_act, n * sizeof(int), cudaMemcpyDeviceToHost));
  if (adv) PL_CUDA(cudaMemcpy(adv, u->mb_adv, n * sizeof(float), cudaMemcpyDeviceToHost));
  if (ret) PL_CUDA(cudaMemcpy(ret, u->mb_ret, n * sizeof(float), cudaMemcpyDeviceToHost));
  if (olp) PL_CUDA(cudaMemcpy(olp, u->mb_olp, n * sizeof(float), cudaMemcpyDeviceToHost));
  if (ov && u->mb_ov) PL_CUDA(cudaMemcpy(ov, u->mb_ov, n * sizeof(float), cudaMemcpyDeviceToHost));
  return PL_OK;
}

// Test hook: 1 = sessions created afterwards all-reduce the gradient per layer on a second stream under
// the backward pass (the default), 0 = one all-reduce of the whole gradient after it; < 0 queries.
extern "C" int pl_test_dp_overlap(int mode) {
  const int prev = g_dp_overlap ? 1 : 0;
  if (mode >= 0) g_dp_overlap = mode != 0;
  return prev;
}
// Test hook: 1 = the bf16 tier's Newton-Schulz chains of all layer groups run in one launch per Muon step
// (the default), 0 = one launch per group; < 0 queries. Returns the previous mode.
extern "C" int pl_test_ns_group_launch(int mode) {
  const int prev = g_ns_one_launch ? 1 : 0;
  if (mode >= 0) g_ns_one_launch = mode != 0;
  return prev;
}
// Test hook: 1 = tight-tier sessions created afterwards run the Muon step of small layers as one launch
// (the default), 0 = one launch sequence per matrix and bias; < 0 queries. Returns the previous mode.
extern "C" int pl_test_exact_group(int mode) {
  const int prev = g_exact_group ? 1 : 0;
  if (mode >= 0) g_exact_group = mode != 0;
  return prev;
}
