// Batched Newton-Schulz that allocates no device memory.
//
// Some callers cannot call cudaMalloc: a host whose device memory is owned by another allocator or
// handed out from a fixed budget at start-up (a framework's caching allocator, an embedded runtime
// that forbids allocation once it runs), or a loop that must never reach the driver's allocator,
// whose calls can block and synchronise the device. For them this entry point takes the
// Newton-Schulz workspace from a fixed array compiled into the library instead of from the
// allocator. The caller still owns X (input and output).
//
// Limit: kNoAllocBytes (32 MiB) per device, which every GPU that loads the library holds until the
// process exits. A request needs, each region rounded up to 256 bytes: 2 * batch*m*n bf16 values
// (two iterates) + 2 * batch*m*m bf16 values (Gram and polynomial) + batch * ceil(m*n / 16384)
// doubles (norm partials) + (3 * batch + 1) 32-bit tile counters + 2 * batch floats (per-matrix
// scale) + 256 bytes (the error word), with m = min(rows, cols) and n = max(rows, cols). Larger
// requests are rejected with PL_ERR_INVALID before anything runs.
//
// Sharing: every call on a device uses the same array and leaves its contents behind, so two calls
// whose work overlaps on the GPU (different streams, or different host threads) race on it and
// corrupt each other's results; serialise them. Two things in it must start at zero: the tile
// counters of the persistent chain, which the chain launcher clears before every launch, and the
// bounded-wait error word, cleared when the array is first set up on a device and again after a
// failure has been reported.
//
// Errors: the call waits for its own work on `stream` to finish and then reads the error word, so
// a device-side wait that ran out comes back from this same call as PL_ERR_DEVICE_TIMEOUT (X is
// then not valid), not silently.
//
// Set-up: the first call on each device looks up the array's device address with
// cudaGetSymbolAddress (with that device current) and clears the error word.
#include <mutex>

#include "pl_gemm.cuh"
#include "pl_mlp.cuh"
#include "pl_runtime.h"

namespace pl {
int launch_transpose_bf16(const __nv_bfloat16* src, long batch, int rows, int cols, __nv_bfloat16* dst,
                          cudaStream_t st);
}  // namespace pl

namespace {
constexpr size_t kNoAllocBytes = (size_t)32 << 20;
static __device__ __align__(256) unsigned char g_ns_noalloc_scratch[kNoAllocBytes];
static void* g_scratch_addr[64];
static std::mutex g_scratch_mu;

inline size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

// Device address of the array on the current device (looked up once per device; the error word at
// its start is cleared then, on the caller's stream, ahead of the call's kernels).
int scratch_address(void** out, cudaStream_t st) {
  int dev = 0;
  PL_CUDA(cudaGetDevice(&dev));
  PL_REQUIRE(dev >= 0 && dev < 64, PL_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> g(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_ns_noalloc_scratch);
    if (e != cudaSuccess) return pl::check_cuda(e, "cudaGetSymbolAddress(no-alloc Newton-Schulz workspace)");
    e = cudaMemsetAsync(p, 0, 256, st);
    if (e != cudaSuccess) return pl::check_cuda(e, "clearing the no-alloc Newton-Schulz error word");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return PL_OK;
}

// The kernels of one call, on stream st, with the workspace regions in w / part / scale.
int run(pl::NsWork& w, __nv_bfloat16* X, size_t batch, size_t rows, size_t cols, int m, int n, long per,
        double eps, const double* coeffs, size_t iters, double* part, float* scale, cudaStream_t st) {
  using namespace pl;
  const bool tall = rows > cols;
  __nv_bfloat16* res = nullptr;
  int rc;
  if (!tall && m > 128 && iters >= 2) {  // normalisation folded into the first step, as in the allocating entry
    return ns_run_batched(m, n, (int)batch, coeffs, (int)iters, w, X, n, per, nullptr, 0, 0, st, X, &res, scale, eps);
  }
  if (!tall && m <= 128 && n <= 512 && ns_set_small_mode(-1))  // normalised by the fused kernel, as above
    return ns_run_batched(m, n, (int)batch, coeffs, (int)iters, w, X, n, per, nullptr, 0, 0, st, X, &res, nullptr, eps);
  rc = launch_ns_prepare(X, (long)batch, (int)rows, (int)cols, eps, part, w.X0, st);
  if (rc) return rc;
  rc = ns_run_batched(m, n, (int)batch, coeffs, (int)iters, w, w.X0, n, per, nullptr, 0, 0, st, tall ? nullptr : X,
                      &res);
  if (rc) return rc;
  if (tall) return launch_transpose_bf16(res, (long)batch, (int)cols, (int)rows, X, st);
  return PL_OK;
}

// Waits for the call's work on st, then reports (and clears) a bounded wait that ran out.
int check_error_word(unsigned* err, cudaStream_t st) {
  unsigned v = 0;
  PL_CUDA(cudaMemcpyAsync(&v, err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  PL_CUDA(cudaStreamSynchronize(st));
  if (v == 0) return PL_OK;
  PL_CUDA(cudaMemsetAsync(err, 0, sizeof(unsigned), st));
  PL_CUDA(cudaStreamSynchronize(st));
  return pl::set_error(PL_ERR_DEVICE_TIMEOUT,
                       "no-alloc Newton-Schulz: a device-side bounded wait ran out (code 0x%x); X is not valid", v);
}
}  // namespace

extern "C" int pl_ns_batched_bf16_dev_noalloc(void* Xv, size_t batch, size_t rows, size_t cols, double eps,
                                              const double* coeffs, size_t iters, void* stream) {
  using namespace pl;
  if (batch == 0 || rows == 0 || cols == 0) return PL_OK;
  PL_REQUIRE(Xv != nullptr, PL_ERR_INVALID, "no-alloc Newton-Schulz: X is NULL");
  PL_REQUIRE(coeffs && iters > 0 && iters <= 64, PL_ERR_INVALID, "Newton-Schulz needs a coefficient table");
  PL_REQUIRE(rows % 8 == 0 && cols % 8 == 0, PL_ERR_INVALID, "batched NS needs rows and cols multiples of 8");
  const int m = (int)(rows < cols ? rows : cols), n = (int)(rows < cols ? cols : rows);
  const long per = (long)m * n;
  const size_t xbytes = align256((size_t)per * batch * 2), gbytes = align256((size_t)m * m * batch * 2);
  const size_t pbytes = align256((size_t)batch * ns_prepare_parts(per) * sizeof(double));
  const size_t cbytes = align256(sizeof(unsigned) * (size_t)ns_chain_counter_words((long)batch));
  const size_t sbytes = align256(sizeof(float) * 2 * batch);
  const size_t need = 256 + 2 * xbytes + 2 * gbytes + pbytes + cbytes + sbytes;
  PL_REQUIRE(need <= kNoAllocBytes, PL_ERR_INVALID,
             "no-alloc Newton-Schulz: %zu matrices of %zux%zu need %zu bytes of workspace, above the fixed %zu-byte "
             "limit (use pl_ns_batched_bf16_dev, which allocates)",
             batch, rows, cols, need, kNoAllocBytes);
  cudaStream_t st = (cudaStream_t)stream;
  void* base = nullptr;
  int rc = scratch_address(&base, st);
  if (rc) return rc;
  unsigned char* b = (unsigned char*)base;
  NsWork w;
  w.err = (unsigned*)b;
  w.X0 = (__nv_bfloat16*)(b + 256);
  w.X1 = (__nv_bfloat16*)(b + 256 + xbytes);
  w.G = (__nv_bfloat16*)(b + 256 + 2 * xbytes);
  w.B = (__nv_bfloat16*)(b + 256 + 2 * xbytes + gbytes);
  double* part = (double*)(b + 256 + 2 * xbytes + 2 * gbytes);
  w.cnt = (unsigned*)(b + 256 + 2 * xbytes + 2 * gbytes + pbytes);
  float* scale = (float*)(b + 256 + 2 * xbytes + 2 * gbytes + pbytes + cbytes);
  w.ldx = n;
  w.ldg = m;
  rc = run(w, (__nv_bfloat16*)Xv, batch, rows, cols, m, n, per, eps, coeffs, iters, part, scale, st);
  if (rc) return rc;
  return check_error_word(w.err, st);
}
