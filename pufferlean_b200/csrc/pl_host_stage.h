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
// Threads of the conversion pool (the calling thread included).
int host_threads();
// Runs fn(t, T) on the pool's T threads (the caller is thread 0); returns when all have returned.
void host_parallel(const std::function<void(int, int)>& fn);

}  // namespace pl
