// Data-parallel communication over NCCL (NVLink 5 / NVSwitch within a node).
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, reusing the copy the process already has if
// any, e.g. the one torch loaded), so the library keeps no link-time dependency on it and a
// single-GPU caller never touches it. One communicator per process and GPU; the caller creates it
// from a unique id it distributes itself (any side channel: a file, a TCP store, MPI).
//
// Also here: the ownership plan of the sharded Newton-Schulz (which rank orthogonalises which
// matrix), a pure host function so every rank computes the same plan without communicating.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
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
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

static NcclApi g_nccl;
static std::once_flag g_nccl_once;

static const NcclApi* nccl() {
  std::call_once(g_nccl_once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
#define PL_SYM(f) g_nccl.f = (decltype(g_nccl.f))dlsym(h, "nccl" #f)
    PL_SYM(GetUniqueId);
    PL_SYM(CommInitRank);
    PL_SYM(CommDestroy);
    PL_SYM(CommAbort);
    PL_SYM(CommGetAsyncError);
    PL_SYM(AllReduce);
    PL_SYM(Broadcast);
    PL_SYM(GroupStart);
    PL_SYM(GroupEnd);
    PL_SYM(GetErrorString);
#undef PL_SYM
    g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRank && g_nccl.CommDestroy && g_nccl.AllReduce &&
                g_nccl.Broadcast && g_nccl.GroupStart && g_nccl.GroupEnd && g_nccl.GetErrorString;
  });
  return g_nccl.ok ? &g_nccl : nullptr;
}

static int nccl_err(ncclResult_t r, const char* what) {
  const NcclApi* n = nccl();
  return set_error(PL_ERR_COMM, "%s: %s", what, n ? n->GetErrorString(r) : "NCCL unavailable");
}

int comm_allreduce_f32(void* comm, float* buf, size_t n, cudaStream_t st) {
  const NcclApi* a = nccl();
  if (!a) return set_error(PL_ERR_COMM, "NCCL library not found");
  ncclResult_t r = a->AllReduce(buf, buf, n, ncclFloat32, ncclSum, (ncclComm_t)comm, st);
  return r == ncclSuccess ? PL_OK : nccl_err(r, "ncclAllReduce(f32)");
}
int comm_allreduce_f64(void* comm, double* buf, size_t n, cudaStream_t st) {
  const NcclApi* a = nccl();
  if (!a) return set_error(PL_ERR_COMM, "NCCL library not found");
  ncclResult_t r = a->AllReduce(buf, buf, n, ncclFloat64, ncclSum, (ncclComm_t)comm, st);
  return r == ncclSuccess ? PL_OK : nccl_err(r, "ncclAllReduce(f64)");
}
int comm_broadcast_group(void* comm, const std::vector<float*>& bufs, const std::vector<size_t>& counts,
                         const std::vector<int>& roots, cudaStream_t st) {
  const NcclApi* a = nccl();
  if (!a) return set_error(PL_ERR_COMM, "NCCL library not found");
  ncclResult_t r = a->GroupStart();
  if (r != ncclSuccess) return nccl_err(r, "ncclGroupStart");
  for (size_t i = 0; i < bufs.size(); i++) {
    r = a->Broadcast(bufs[i], bufs[i], counts[i], ncclFloat32, roots[i], (ncclComm_t)comm, st);
    if (r != ncclSuccess) {
      a->GroupEnd();
      return nccl_err(r, "ncclBroadcast");
    }
  }
  r = a->GroupEnd();
  return r == ncclSuccess ? PL_OK : nccl_err(r, "ncclGroupEnd");
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
  int rc = pl::require_device();
  if (rc) return rc;
  if (!id || !comm || world < 1 || rank < 0 || rank >= world)
    return pl::set_error(PL_ERR_INVALID, "pl_comm_create: bad rank %d / world %d", rank, world);
  const pl::NcclApi* a = pl::nccl();
  if (!a) return pl::set_error(PL_ERR_COMM, "NCCL library (libnccl.so.2) not found");
  ncclUniqueId u;
  memcpy(u.internal, id, 128);
  ncclComm_t c = nullptr;
  ncclResult_t r = a->CommInitRank(&c, world, u, rank);
  if (r != ncclSuccess) return pl::nccl_err(r, "ncclCommInitRank");
  *comm = (void*)c;
  return PL_OK;
}

int pl_comm_destroy(void* comm) {
  if (!comm) return PL_OK;
  const pl::NcclApi* a = pl::nccl();
  if (!a) return pl::set_error(PL_ERR_COMM, "NCCL library not found");
  ncclResult_t r = a->CommDestroy((ncclComm_t)comm);
  return r == ncclSuccess ? PL_OK : pl::nccl_err(r, "ncclCommDestroy");
}

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
