// Batched Newton-Schulz sharded over the ranks of a communicator, the results all-gathered (the
// batched Newton-Schulz benchmark at N > 1: "matrices are sharded across 1/2/4/8 GPUs, followed by an
// all-gather"; the reference has no multi-GPU code).
//
// Every rank holds the same batch of inputs and ends with every result. The batch is cut into C
// chunks of R * cs matrices (R ranks, cs per rank and chunk); in chunk c rank r orthogonalises
// matrices [c R cs + r cs, c R cs + (r + 1) cs) in place with the single-GPU batched kernels, then an
// in-place all-gather of chunk c runs on a second stream while chunk c + 1 is orthogonalised. The
// remainder of the batch that does not fill a chunk (fewer than R C matrices, or all of them when the
// batch has fewer than R) is orthogonalised on every rank, last, under the final all-gather. A
// matrix's result depends only on that matrix (the batched kernels take the same path whatever the
// batch size), so the sharded result is bit-identical to one GPU's.
//
// Matrices with a short side of at most 128 and a long side of at most 512 are not sharded: the fused
// kernel that takes them (one CTA per matrix, all steps in shared memory) is latency-bound, its time does not shrink with the batch
// (configs[2]'s 64 x 128^2: 55 us for all 64 on one GPU, 50 us for 32), so sharding would only add
// the all-gather. Chunks overlap little in practice: the persistent Newton-Schulz kernel is a
// cooperative launch over every SM, so a chunk's all-gather kernels get SMs only between chunks
// (2 GPUs, 64 x 512 x 2048: one chunk 566 us, two 694 us, against 779 us on one GPU).
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/pufferlean_b200.h"
#include "pl_comm.h"
#include "pl_common.cuh"
#include "pl_runtime.h"

namespace pl {
namespace {

constexpr int kMaxShardChunks = 16;

// The all-gather stream of a device and its events (one per chunk, one for the end), made once.
struct ShardStreams {
  cudaStream_t cs = nullptr;
  cudaEvent_t ev[kMaxShardChunks + 1] = {};
  bool ready = false;
};
ShardStreams g_shard[64];
std::mutex g_shard_mu;

int shard_streams(ShardStreams** out) {
  int dev = 0;
  PL_CUDA(cudaGetDevice(&dev));
  PL_REQUIRE(dev >= 0 && dev < 64, PL_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_shard_mu);
  ShardStreams& s = g_shard[dev];
  if (!s.ready) {
    PL_CUDA(cudaStreamCreateWithFlags(&s.cs, cudaStreamNonBlocking));
    for (auto& e : s.ev) PL_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    s.ready = true;
  }
  *out = &s;
  return PL_OK;
}

}  // namespace
}  // namespace pl

extern "C" int pl_ns_shard_chunks(size_t batch, size_t world, size_t chunks, size_t* per_rank, size_t* used) {
  if (!per_rank || !used || world == 0) return pl::set_error(PL_ERR_INVALID, "pl_ns_shard_chunks: bad arguments");
  size_t c = chunks < 1 ? 1 : (chunks > (size_t)pl::kMaxShardChunks ? (size_t)pl::kMaxShardChunks : chunks);
  while (c > 1 && batch / (world * c) == 0) c--;
  *per_rank = batch / (world * c);
  *used = *per_rank ? c : 0;
  return PL_OK;
}

extern "C" int pl_ns_batched_bf16_dev_sharded(void* Xv, size_t batch, size_t rows, size_t cols, double eps,
                                              const double* coeffs, size_t iters, void* comm, size_t chunks,
                                              void* stream) {
  using namespace pl;
  if (batch == 0 || rows == 0 || cols == 0) return PL_OK;
  int rank = 0, world = 1;
  int rc = comm_rank_world(comm, &rank, &world);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  __nv_bfloat16* X = (__nv_bfloat16*)Xv;
  const size_t per = rows * cols;
  size_t cs = 0, nch = 0;
  rc = pl_ns_shard_chunks(batch, (size_t)world, chunks, &cs, &nch);
  if (rc) return rc;
  const size_t mside = rows < cols ? rows : cols, nside = rows < cols ? cols : rows;
  if (nch == 0 || (mside <= 128 && nside <= 512))  // nothing to shard, or the latency-bound fused kernel
    return pl_ns_batched_bf16_dev(Xv, batch, rows, cols, eps, coeffs, iters, stream);
  ShardStreams* ss = nullptr;
  rc = shard_streams(&ss);
  if (rc) return rc;
  const size_t span = (size_t)world * cs;  // matrices per chunk
  for (size_t c = 0; c < nch; c++) {
    __nv_bfloat16* mine = X + (c * span + (size_t)rank * cs) * per;
    rc = pl_ns_batched_bf16_dev(mine, cs, rows, cols, eps, coeffs, iters, st);
    if (rc) return rc;
    PL_CUDA(cudaEventRecord(ss->ev[c], st));
    PL_CUDA(cudaStreamWaitEvent(ss->cs, ss->ev[c], 0));
    rc = comm_allgather_bf16(comm, mine, X + c * span * per, cs * per, ss->cs);
    if (rc) return rc;
  }
  const size_t done = nch * span;
  if (done < batch) {  // the remainder, on every rank, under the last all-gather
    rc = pl_ns_batched_bf16_dev(X + done * per, batch - done, rows, cols, eps, coeffs, iters, st);
    if (rc) return rc;
  }
  PL_CUDA(cudaEventRecord(ss->ev[kMaxShardChunks], ss->cs));
  PL_CUDA(cudaStreamWaitEvent(st, ss->ev[kMaxShardChunks], 0));
  return PL_OK;
}
