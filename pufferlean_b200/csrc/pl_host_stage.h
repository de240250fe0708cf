// Pinned double-buffered staging for uploading f64 observation rows as bf16 (pl_host_stage.cpp).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include <functional>

namespace pl {

struct HostStage {
  void* buf[2] = {nullptr, nullptr};  // pinned, `cap` bytes each
  cudaEvent_t done[2] = {nullptr, nullptr};
  bool used[2] = {false, false};
  int next = 0;  // the buffer the next chunked upload starts with
  size_t cap = 0;
  int init(size_t bytes);  // 0 = ready (allocates once); -1 = no pinned memory (use another path)
  void release();
};

// Rounds the NT x D f64 rows of host `obs` to bf16 on the host threads (Dp wide, zero padded) and
// copies them to dst_dev on stream st through the two staging buffers, converting chunk k + 1 while
// chunk k is in flight. With dev_rows (obs pinned), a share of the rows is instead handed to
// dev_rows(r0, nr), which enqueues their f64 copy and device conversion on st, interleaved so that
// the host threads and the host link finish together. Returns 0, or -1 on an error.
int upload_rows_bf16(HostStage& hs, const double* obs, long NT, int D, int Dp, void* dst_dev, cudaStream_t st,
                     const std::function<int(long, long)>& dev_rows = nullptr);
// Rounds rows k in [k0, k1) of a shuffle order -- host row order[k] of the nrows x D f64 `obs` (f64
// indices) -- to bf16 rows k of dst_dev (Dp wide, zero padded), through the staging buffers on stream
// st; a later call continues with the other buffer, so consecutive calls overlap as one upload.
// Returns 0, -1 on a CUDA error, or -2 when an order entry is not an integer in [0, nrows) (its row
// is left zero).
int upload_rows_bf16_order(HostStage& hs, const double* obs, const double* order, long nrows, long k0, long k1, int D,
                           int Dp, void* dst_dev, cudaStream_t st);
// Threads of the conversion pool (the calling thread included).
int host_threads();
// Runs fn(t, T) on the pool's T threads (the caller is thread 0); returns when all have returned.
void host_parallel(const std::function<void(int, int)>& fn);

}  // namespace pl
