// Data-parallel communication over NCCL (NVLink 5 / NVSwitch within a node).
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, reusing the copy the process already has if
// any, e.g. the one torch loaded), so the library keeps no link-time dependency on it and a
// single-GPU caller never touches it. One communicator per process and GPU; the caller creates it
// from a unique id it distributes itself (any side channel: a file, a TCP store, MPI).
//
// Failure handling. Communicators are created non-blocking (ncclConfig_t.blocking = 0): creation and
// every call that answers ncclInProgress are polled with ncclCommGetAsyncError until they settle or a
// deadline passes (pl_comm_set_timeout; 600 s by default). A deadline that passes, or an asynchronous
// error (a peer that died, a network error), aborts the communicator (ncclCommAbort, which also makes
// NCCL kernels still waiting on a peer return) and the call fails with PL_ERR_COMM. pl_comm_wait is the
// watchdog of enqueued work: it waits for a stream with the same deadline and error checks. An aborted
// communicator fails every later call at once, before anything is enqueued. A test hook replaces the
// NCCL entry points and the stream query with fakes (a peer that never joins, a peer that fails, a
// collective that never completes), so all of this is tested on the host without a GPU.
//
// Also here: the ownership plan of the sharded Newton-Schulz (which rank orthogonalises which
// matrix), a pure host function so every rank computes the same plan without communicating.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <numeric>
#include <vector>

#include "../../include/pufferlean_b200.h"
#include "pl_comm.h"

namespace pl {
int set_error(int code, const char* fmt, ...);
int require_device();

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  // stream completion: cudaStreamQuery, or the fake's
  int (*StreamDone)(cudaStream_t) = nullptr;
  bool ok = false;
};

static int real_stream_done(cudaStream_t st) {
  const cudaError_t e = cudaStreamQuery(st);
  if (e == cudaErrorNotReady) return 0;
  return e == cudaSuccess ? 1 : -1;
}

static NcclApi g_nccl;
static std::once_flag g_nccl_once;

// ---------------------------------------------------------------- fakes (host-side failure tests)
// 1: creation never completes (a peer that never joins); 2: a peer fails once the communicator is up
// (every asynchronous-error query after the one that completes creation reports ncclRemoteError);
// 3: enqueued work never completes (the stream query never reports done); 4: a healthy communicator.
// 0: the real library.
static std::atomic<int> g_fake{0};
static std::atomic<int> g_fake_aborts{0};
static std::atomic<int> g_fake_queries{0};
static char g_fake_comm_obj[64][8];
static std::atomic<int> g_fake_next{0};
namespace fake {
static ncclResult_t GetUniqueId(ncclUniqueId* u) {
  memset(u, 7, sizeof(*u));
  return ncclSuccess;
}
static ncclResult_t CommInitRankConfig(ncclComm_t* c, int, ncclUniqueId, int, ncclConfig_t*) {
  *c = (ncclComm_t)g_fake_comm_obj[g_fake_next.fetch_add(1) & 63];
  g_fake_queries.store(0);
  return g_fake.load() == 1 ? ncclInProgress : ncclSuccess;
}
static ncclResult_t CommDestroy(ncclComm_t) { return ncclSuccess; }
static ncclResult_t CommAbort(ncclComm_t) {
  g_fake_aborts.fetch_add(1);
  return ncclSuccess;
}
static ncclResult_t CommGetAsyncError(ncclComm_t, ncclResult_t* r) {
  const int m = g_fake.load();
  const int q = g_fake_queries.fetch_add(1);
  *r = m == 1 ? ncclInProgress : ((m == 2 && q > 0) ? ncclRemoteError : ncclSuccess);
  return ncclSuccess;
}
static ncclResult_t AllReduce(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) {
  return ncclSuccess;
}
static ncclResult_t Broadcast(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) {
  return ncclSuccess;
}
static ncclResult_t AllGather(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) {
  return ncclSuccess;
}
static ncclResult_t GroupStart() { return ncclSuccess; }
static ncclResult_t GroupEnd() { return ncclSuccess; }
static const char* GetErrorString(ncclResult_t r) {
  return r == ncclRemoteError ? "remote process exited or there was a network error (fake)" : "fake NCCL error";
}
static int StreamDone(cudaStream_t) { return g_fake.load() == 3 ? 0 : 1; }
}  // namespace fake

static NcclApi make_fake() {
  NcclApi a;
  a.GetUniqueId = fake::GetUniqueId;
  a.CommInitRankConfig = fake::CommInitRankConfig;
  a.CommDestroy = fake::CommDestroy;
  a.CommAbort = fake::CommAbort;
  a.CommGetAsyncError = fake::CommGetAsyncError;
  a.AllReduce = fake::AllReduce;
  a.Broadcast = fake::Broadcast;
  a.AllGather = fake::AllGather;
  a.GroupStart = fake::GroupStart;
  a.GroupEnd = fake::GroupEnd;
  a.GetErrorString = fake::GetErrorString;
  a.StreamDone = fake::StreamDone;
  a.ok = true;
  return a;
}
static NcclApi g_fake_api = make_fake();

static const NcclApi* nccl() {
  if (g_fake.load()) return &g_fake_api;
  std::call_once(g_nccl_once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
#define PL_SYM(f) g_nccl.f = (decltype(g_nccl.f))dlsym(h, "nccl" #f)
    PL_SYM(GetUniqueId);
    PL_SYM(CommInitRankConfig);
    PL_SYM(CommDestroy);
    PL_SYM(CommAbort);
    PL_SYM(CommGetAsyncError);
    PL_SYM(AllReduce);
    PL_SYM(Broadcast);
    PL_SYM(AllGather);
    PL_SYM(GroupStart);
    PL_SYM(GroupEnd);
    PL_SYM(GetErrorString);
#undef PL_SYM
    g_nccl.StreamDone = real_stream_done;
    g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRankConfig && g_nccl.CommDestroy && g_nccl.CommAbort &&
                g_nccl.CommGetAsyncError && g_nccl.AllReduce && g_nccl.Broadcast && g_nccl.AllGather && g_nccl.GroupStart &&
                g_nccl.GroupEnd && g_nccl.GetErrorString;
  });
  return g_nccl.ok ? &g_nccl : nullptr;
}

// ---------------------------------------------------------------- communicator object
static constexpr uint64_t kCommMagic = 0x706c636f6d6d3031ULL;
struct PlComm {
  uint64_t magic = kCommMagic;
  ncclComm_t nc = nullptr;
  int rank = 0, world = 1;
  std::atomic<bool> aborted{false};
  bool fake = false;
};
static std::atomic<double> g_timeout_s{600.0};

static double now_s() {
  timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

static PlComm* as_comm(void* c) {
  PlComm* p = (PlComm*)c;
  return (p && p->magic == kCommMagic) ? p : nullptr;
}

static int nccl_err(ncclResult_t r, const char* what) {
  const NcclApi* n = nccl();
  return set_error(PL_ERR_COMM, "%s: %s", what, n ? n->GetErrorString(r) : "NCCL unavailable");
}

static int abort_comm(PlComm* c, const char* why) {
  if (!c->aborted.exchange(true)) {
    const NcclApi* a = nccl();
    if (a && c->nc) a->CommAbort(c->nc);
  }
  return set_error(PL_ERR_COMM, "communicator of rank %d/%d aborted: %s", c->rank, c->world, why);
}

// Between polls: a few thousand immediate retries (an enqueue usually settles within microseconds),
// then 0.2 ms sleeps.
static void pause(long polls) {
  if (polls < 4096) return;
  struct timespec ts = {0, 200000};
  nanosleep(&ts, nullptr);
}

// Polls the communicator's asynchronous state until it leaves ncclInProgress; the deadline or an
// error aborts it.
static int settle(PlComm* c, const char* what) {
  const NcclApi* a = nccl();
  const double t_end = now_s() + g_timeout_s.load();
  long polls = 0;
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = a->CommGetAsyncError(c->nc, &st);
    if (r != ncclSuccess) st = r;
    if (st == ncclSuccess) return PL_OK;
    if (st != ncclInProgress) {
      char buf[256];
      snprintf(buf, sizeof buf, "%s: %s", what, a->GetErrorString(st));
      return abort_comm(c, buf);
    }
    if (now_s() > t_end) {
      char buf[256];
      snprintf(buf, sizeof buf, "%s did not complete within %.3g s", what, g_timeout_s.load());
      return abort_comm(c, buf);
    }
    pause(++polls);
  }
}

// Result of one enqueue call in non-blocking mode: success, in progress (settled by polling) or error.
static int after_call(PlComm* c, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return PL_OK;
  if (r == ncclInProgress) return settle(c, what);
  char buf[256];
  snprintf(buf, sizeof buf, "%s: %s", what, nccl()->GetErrorString(r));
  return abort_comm(c, buf);
}

static int usable(void* comm, PlComm** out) {
  PlComm* c = as_comm(comm);
  if (!c) return set_error(PL_ERR_INVALID, "not a communicator from pl_comm_create");
  if (c->aborted.load()) return set_error(PL_ERR_COMM, "communicator of rank %d/%d was aborted", c->rank, c->world);
  if (!nccl()) return set_error(PL_ERR_COMM, "NCCL library not found");
  *out = c;
  return PL_OK;
}

int comm_allreduce_f32(void* comm, float* buf, size_t n, cudaStream_t st) {
  PlComm* c = nullptr;
  int rc = usable(comm, &c);
  if (rc) return rc;
  return after_call(c, nccl()->AllReduce(buf, buf, n, ncclFloat32, ncclSum, c->nc, st), "ncclAllReduce(f32)");
}
int comm_allreduce_f64(void* comm, double* buf, size_t n, cudaStream_t st) {
  PlComm* c = nullptr;
  int rc = usable(comm, &c);
  if (rc) return rc;
  return after_call(c, nccl()->AllReduce(buf, buf, n, ncclFloat64, ncclSum, c->nc, st), "ncclAllReduce(f64)");
}
int comm_allgather_bf16(void* comm, const void* send, void* recv, size_t count, cudaStream_t st) {
  PlComm* c = nullptr;
  int rc = usable(comm, &c);
  if (rc) return rc;
  return after_call(c, nccl()->AllGather(send, recv, count, ncclBfloat16, c->nc, st), "ncclAllGather(bf16)");
}
int comm_rank_world(void* comm, int* rank, int* world) {
  PlComm* c = nullptr;
  int rc = usable(comm, &c);
  if (rc) return rc;
  *rank = c->rank;
  *world = c->world;
  return PL_OK;
}
int comm_broadcast_group(void* comm, const std::vector<float*>& bufs, const std::vector<size_t>& counts,
                         const std::vector<int>& roots, cudaStream_t st) {
  PlComm* c = nullptr;
  int rc = usable(comm, &c);
  if (rc) return rc;
  const NcclApi* a = nccl();
  ncclResult_t r = a->GroupStart();
  if (r != ncclSuccess) return after_call(c, r, "ncclGroupStart");
  for (size_t i = 0; i < bufs.size(); i++) {
    r = a->Broadcast(bufs[i], bufs[i], counts[i], ncclFloat32, roots[i], c->nc, st);
    if (r != ncclSuccess && r != ncclInProgress) {
      a->GroupEnd();
      return after_call(c, r, "ncclBroadcast");
    }
  }
  return after_call(c, a->GroupEnd(), "ncclGroupEnd (broadcasts)");
}

}  // namespace pl

extern "C" {

int pl_comm_unique_id(uint8_t id[128]) {
  if (!id) return pl::set_error(PL_ERR_INVALID, "pl_comm_unique_id: NULL");
  const pl::NcclApi* a = pl::nccl();
  if (!a) return pl::set_error(PL_ERR_COMM, "NCCL library (libnccl.so.2) not found");
  ncclUniqueId u;
  ncclResult_t r = a->GetUniqueId(&u);
  if (r != ncclSuccess) return pl::nccl_err(r, "ncclGetUniqueId");
  static_assert(sizeof(u.internal) == 128, "NCCL unique id size");
  memcpy(id, u.internal, 128);
  return PL_OK;
}

int pl_comm_create(int rank, int world, const uint8_t id[128], void** comm) {
  const bool fake = pl::g_fake.load() != 0;
  if (!fake) {
    int rc = pl::require_device();
    if (rc) return rc;
  }
  if (!id || !comm || world < 1 || rank < 0 || rank >= world)
    return pl::set_error(PL_ERR_INVALID, "pl_comm_create: bad rank %d / world %d", rank, world);
  *comm = nullptr;
  const pl::NcclApi* a = pl::nccl();
  if (!a) return pl::set_error(PL_ERR_COMM, "NCCL library (libnccl.so.2) not found");
  ncclUniqueId u;
  memcpy(u.internal, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // creation and collectives return at once; progress is polled with a deadline
  pl::PlComm* c = new pl::PlComm();
  c->rank = rank;
  c->world = world;
  c->fake = fake;
  ncclResult_t r = a->CommInitRankConfig(&c->nc, world, u, rank, &cfg);
  int rc = (r == ncclSuccess || r == ncclInProgress) ? pl::settle(c, "ncclCommInitRankConfig")
                                                      : pl::nccl_err(r, "ncclCommInitRankConfig");
  if (rc) {
    // an aborted communicator is released by the abort; one that failed outright never existed
    delete c;
    return rc;
  }
  *comm = (void*)c;
  return PL_OK;
}

int pl_comm_destroy(void* comm) {
  if (!comm) return PL_OK;
  pl::PlComm* c = pl::as_comm(comm);
  if (!c) return pl::set_error(PL_ERR_INVALID, "pl_comm_destroy: not a communicator from pl_comm_create");
  int rc = PL_OK;
  if (!c->aborted.load()) {
    const pl::NcclApi* a = pl::nccl();
    if (!a) return pl::set_error(PL_ERR_COMM, "NCCL library not found");
    ncclResult_t r = a->CommDestroy(c->nc);
    if (r != ncclSuccess && r != ncclInProgress) rc = pl::nccl_err(r, "ncclCommDestroy");
  }
  c->magic = 0;
  delete c;
  return rc;
}

int pl_comm_set_timeout(double seconds) {
  if (!(seconds > 0)) return pl::set_error(PL_ERR_INVALID, "pl_comm_set_timeout: %g s", seconds);
  pl::g_timeout_s.store(seconds);
  return PL_OK;
}

int pl_comm_wait(void* comm, void* stream) {
  pl::PlComm* c = nullptr;
  int rc = pl::usable(comm, &c);
  if (rc) return rc;
  const pl::NcclApi* a = pl::nccl();
  const double t_end = pl::now_s() + pl::g_timeout_s.load();
  long polls = 0;
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = a->CommGetAsyncError(c->nc, &st);
    if (r != ncclSuccess) st = r;
    if (st != ncclSuccess && st != ncclInProgress) {
      char buf[256];
      snprintf(buf, sizeof buf, "asynchronous error: %s", a->GetErrorString(st));
      return pl::abort_comm(c, buf);
    }
    const int done = a->StreamDone((cudaStream_t)stream);
    if (done > 0) return PL_OK;
    if (done < 0) return pl::set_error(PL_ERR_CUDA, "pl_comm_wait: stream query failed");
    if (pl::now_s() > t_end) {
      char buf[256];
      snprintf(buf, sizeof buf, "enqueued work did not complete within %.3g s", pl::g_timeout_s.load());
      return pl::abort_comm(c, buf);
    }
    pl::pause(++polls);
  }
}

int pl_comm_abort(void* comm) {
  pl::PlComm* c = pl::as_comm(comm);
  if (!c) return pl::set_error(PL_ERR_INVALID, "pl_comm_abort: not a communicator from pl_comm_create");
  pl::abort_comm(c, "requested by the caller");
  return PL_OK;
}

int pl_comm_aborted(void* comm) {
  pl::PlComm* c = pl::as_comm(comm);
  return c ? (c->aborted.load() ? 1 : 0) : -1;
}

int pl_test_comm_fake(int mode) {
  const int prev = pl::g_fake.load();
  if (mode >= 0) pl::g_fake.store(mode);
  return prev;
}

int pl_test_comm_fake_aborts(void) { return pl::g_fake_aborts.load(); }

// Longest-processing-time assignment of matrices to ranks by Newton-Schulz cost
// iters * (4 m^2 n + 2 m^3), m = min(rows, cols), n = max: matrices in decreasing cost (ties by
// index), each to the currently least-loaded rank (ties to the lower rank). Deterministic, so every
// rank derives the same plan locally.
int pl_muon_shard_plan(const size_t* rows, const size_t* cols, size_t nmat, int world, int* owner) {
  if ((!rows || !cols || !owner) && nmat) return pl::set_error(PL_ERR_INVALID, "pl_muon_shard_plan: NULL");
  if (world < 1) return pl::set_error(PL_ERR_INVALID, "pl_muon_shard_plan: world %d", world);
  std::vector<double> cost(nmat);
  for (size_t i = 0; i < nmat; i++) {
    const double m = (double)std::min(rows[i], cols[i]), n = (double)std::max(rows[i], cols[i]);
    cost[i] = 4.0 * m * m * n + 2.0 * m * m * m;
  }
  std::vector<size_t> order(nmat);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return cost[a] > cost[b]; });
  std::vector<double> load((size_t)world, 0.0);
  for (size_t i : order) {
    int best = 0;
    for (int r = 1; r < world; r++)
      if (load[r] < load[best]) best = r;
    owner[i] = best;
    load[best] += cost[i];
  }
  return PL_OK;
}

}  // extern "C"
