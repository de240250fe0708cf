// Host side of the observation upload: f64 rows (the reference ABI's column form) rounded to bf16 by a
// small pool of host threads into pinned staging buffers, which the copy engine then moves to the
// device while the next chunk is converted. The device keeps observations in bf16, so sending bf16
// over the host link moves a quarter of the bytes of the f64 rows; the rounding is the device
// conversion's (f64 -> f32 to nearest, then f32 -> bf16 to nearest even), so the device copy is
// bit-identical to converting there.
#pragma GCC optimize("O3")
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <sched.h>
#include <stdlib.h>

#include <thread>
#include <vector>

#include "pl_host_stage.h"

namespace pl {

namespace {

// Threads of the pool: the cores this process may run on, shared with the other processes of the node
// that upload at the same time (one per GPU: LOCAL_WORLD_SIZE, as torch.distributed launchers set it),
// at most 16; PL_HOST_THREADS overrides. Eight ranks on one host then split its cores instead of each
// starting 16 threads that compete for them.
static int pool_threads() {
  if (const char* e = getenv("PL_HOST_THREADS")) {
    const int v = atoi(e);
    if (v >= 1) return std::min(v, 64);
  }
  int cores = 0;
  cpu_set_t set;
  if (sched_getaffinity(0, sizeof(set), &set) == 0) cores = CPU_COUNT(&set);
  if (cores <= 0) cores = (int)std::thread::hardware_concurrency();
  int local = 1;
  if (const char* e = getenv("LOCAL_WORLD_SIZE")) local = std::max(1, atoi(e));
  return std::max(1, std::min(16, std::max(1, cores) / local));
}

// Fork-join pool: run(fn) calls fn(t, T) on T threads (the caller is thread 0) and returns when all
// have returned.
class Pool {
 public:
  Pool() {
    n_ = pool_threads();
    for (int t = 1; t < n_; t++) th_.emplace_back([this, t] { loop(t); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
      gen_++;
    }
    cv_.notify_all();
    for (auto& t : th_) t.join();
  }
  int size() const { return n_; }
  void run(const std::function<void(int, int)>& fn) {
    {
      std::lock_guard<std::mutex> g(mu_);
      fn_ = &fn;
      left_ = n_ - 1;
      gen_++;
    }
    cv_.notify_all();
    fn(0, n_);
    std::unique_lock<std::mutex> g(mu_);
    done_.wait(g, [this] { return left_ == 0; });
    fn_ = nullptr;
  }

 private:
  void loop(int t) {
    uint64_t seen = 0;
    for (;;) {
      const std::function<void(int, int)>* fn;
      {
        std::unique_lock<std::mutex> g(mu_);
        cv_.wait(g, [&] { return gen_ != seen; });
        seen = gen_;
        if (stop_) return;
        fn = fn_;
      }
      (*fn)(t, n_);
      {
        std::lock_guard<std::mutex> g(mu_);
        if (--left_ == 0) done_.notify_one();
      }
    }
  }
  int n_ = 1;
  std::vector<std::thread> th_;
  std::mutex mu_;
  std::condition_variable cv_, done_;
  const std::function<void(int, int)>* fn_ = nullptr;
  uint64_t gen_ = 0;
  int left_ = 0;
  bool stop_ = false;
};

Pool& pool() {
  static Pool p;
  return p;
}

// f32 -> bf16 bits, round to nearest even; NaN -> the canonical 0x7FFF (branch-free, so the row loop
// vectorises)
inline uint16_t bf16_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  const uint32_t r = (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
  const bool nan = (u & 0x7FFFFFFFu) > 0x7F800000u;
  return (uint16_t)(nan ? 0x7FFFu : r);
}

// Cloned for AVX-512 and AVX2 with run-time dispatch (the library is built for baseline x86-64).
__attribute__((target_clones("avx512f", "avx2", "default"))) void rows_to_bf16(const double* src, long r0, long r1,
                                                                               int D, int Dp, uint16_t* dst) {
  for (long r = r0; r < r1; r++) {
    const double* s = src + r * D;
    uint16_t* o = dst + r * Dp;
    for (int c = 0; c < D; c++) o[c] = bf16_bits((float)s[c]);
    for (int c = D; c < Dp; c++) o[c] = 0;
  }
}

// Rows k in [k0, k1) of the order: src row order[k] (an f64 row index, as the reference's shuffles are
// stored) -> dst row k - k0. An entry that is not an integer in [0, nrows) leaves a zero row and sets
// *bad. The next row's first lines are prefetched while this one is rounded (rows are visited in the
// shuffle's random order).
__attribute__((target_clones("avx512f", "avx2", "default"))) void rows_to_bf16_order(
    const double* src, const double* order, long nrows, long k0, long k1, int D, int Dp, uint16_t* dst, int* bad) {
  for (long k = k0; k < k1; k++) {
    const double f = order[k];
    const long r = (long)f;
    uint16_t* o = dst + (k - k0) * Dp;
    if (!(f >= 0.0 && f < (double)nrows) || (double)r != f) {
      for (int c = 0; c < Dp; c++) o[c] = 0;
      *bad = 1;
      continue;
    }
    if (k + 1 < k1) {
      const double fn = order[k + 1];
      if (fn >= 0.0 && fn < (double)nrows) {
        const char* nx = (const char*)(src + (long)fn * D);
        for (int b = 0; b < 4 && b * 64 < D * 8; b++) __builtin_prefetch(nx + b * 64);
      }
    }
    const double* s = src + r * D;
    for (int c = 0; c < D; c++) o[c] = bf16_bits((float)s[c]);
    for (int c = D; c < Dp; c++) o[c] = 0;
  }
}

}  // namespace

int host_threads() { return pool().size(); }
void host_parallel(const std::function<void(int, int)>& fn) { pool().run(fn); }

int HostStage::init(size_t bytes) {
  if (buf[0] && cap >= bytes) return 0;
  release();
  for (int b = 0; b < 2; b++) {
    if (cudaHostAlloc(&buf[b], bytes, cudaHostAllocDefault) != cudaSuccess) {
      cudaGetLastError();
      release();
      return -1;
    }
    if (cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      release();
      return -1;
    }
  }
  cap = bytes;
  used[0] = used[1] = false;
  return 0;
}

void HostStage::release() {
  for (int b = 0; b < 2; b++) {
    if (buf[b]) cudaFreeHost(buf[b]);
    if (done[b]) cudaEventDestroy(done[b]);
    buf[b] = nullptr;
    done[b] = nullptr;
    used[b] = false;
  }
  cap = 0;
}

int upload_rows_bf16(HostStage& hs, const double* obs, long NT, int D, int Dp, void* dst_dev, cudaStream_t st,
                     const std::function<int(long, long)>& dev_rows) {
  const size_t row_bytes = (size_t)Dp * 2;
  const long rows = std::max<long>(1, (long)(hs.cap / row_bytes));
  uint16_t* dst = (uint16_t*)dst_dev;
  Pool& P = pool();
  // Host share: with H the host threads' f64 read rate (about 6 GB/s per thread, at most ~90 GB/s)
  // and L the link rate (~50 GB/s), rounding a share a on the host takes a S / H and the link moves
  // (a / 4 + 1 - a) S, so both end together at a = H / (L + 0.75 H).
  long NH = NT;
  if (dev_rows) {
    const double H = std::min(6.0 * P.size(), 90.0), L = 50.0;
    NH = std::min(NT, std::max(0L, (long)(NT * (H / (L + 0.75 * H)))));
  }
  long dnext = NH;  // next row handed to the device
  int k = 0;
  for (long r0 = 0; r0 < NH; r0 += rows, k ^= 1) {
    const long nr = std::min(rows, NH - r0);
    if (hs.used[k] && cudaEventSynchronize(hs.done[k]) != cudaSuccess) return -1;  // its last copy has left
    uint16_t* b = (uint16_t*)hs.buf[k];
    const double* s = obs + r0 * D;
    P.run([&](int t, int T) {
      const long a = nr * t / T, e = nr * (t + 1) / T;
      rows_to_bf16(s, a, e, D, Dp, b);
    });
    if (cudaMemcpyAsync(dst + r0 * Dp, b, (size_t)nr * row_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess) return -1;
    if (cudaEventRecord(hs.done[k], st) != cudaSuccess) return -1;
    hs.used[k] = true;
    if (dev_rows && dnext < NT) {  // the device's rows in proportion, queued behind this chunk's copy
      const long want = NH > 0 ? (long)((double)(NT - NH) * (double)(r0 + nr) / (double)NH) + NH : NT;
      const long upto = (r0 + nr >= NH) ? NT : std::min(NT, want);
      if (upto > dnext) {
        if (dev_rows(dnext, upto - dnext) != 0) return -1;
        dnext = upto;
      }
    }
  }
  if (dev_rows && dnext < NT && dev_rows(dnext, NT - dnext) != 0) return -1;
  return 0;
}

int upload_rows_bf16_order(HostStage& hs, const double* obs, const double* order, long nrows, long k0, long k1, int D,
                           int Dp, void* dst_dev, cudaStream_t st) {
  const size_t row_bytes = (size_t)Dp * 2;
  const long rows = std::max<long>(1, (long)(hs.cap / row_bytes));
  uint16_t* dst = (uint16_t*)dst_dev;
  Pool& P = pool();
  int bad = 0;
  int k = hs.next;
  for (long r0 = k0; r0 < k1; r0 += rows, k ^= 1) {
    const long nr = std::min(rows, k1 - r0);
    if (hs.used[k] && cudaEventSynchronize(hs.done[k]) != cudaSuccess) return -1;  // its last copy has left
    uint16_t* b = (uint16_t*)hs.buf[k];
    P.run([&](int t, int T) {
      int tb = 0;
      rows_to_bf16_order(obs, order, nrows, r0 + nr * t / T, r0 + nr * (t + 1) / T, D, Dp, b + (nr * t / T) * Dp, &tb);
      if (tb) __atomic_store_n(&bad, 1, __ATOMIC_RELAXED);
    });
    if (cudaMemcpyAsync(dst + r0 * Dp, b, (size_t)nr * row_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess) return -1;
    if (cudaEventRecord(hs.done[k], st) != cudaSuccess) return -1;
    hs.used[k] = true;
  }
  hs.next = k;
  return bad ? -2 : 0;
}

}  // namespace pl

// Test hook: the host rounding of rows x D f64 values into Dp-wide bf16 rows (no device involved).
extern "C" int pl_test_round_rows_bf16(const double* src, long rows, int D, int Dp, uint16_t* dst) {
  if (!src || !dst || rows < 0 || D < 0 || Dp < D) return -1;
  pl::pool().run([&](int t, int T) { pl::rows_to_bf16(src, rows * t / T, rows * (t + 1) / T, D, Dp, dst); });
  return 0;
}
