// Library runtime: error reporting, device selection, launch accounting, the per-device error
// word that bounded device-side waits write to.
#include <stdarg.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "pl_common.cuh"
#include "pl_runtime.h"

namespace pl {

static thread_local char g_err[1024] = "";
static std::atomic<uint64_t> g_launches{0};

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
void clear_error() { g_err[0] = 0; }

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
    return set_error(PL_ERR_NO_DEVICE, "%s: %s (no usable CUDA device; this library has no CPU fallback)", what,
                     cudaGetErrorString(e));
  if (e == cudaErrorMemoryAllocation) return set_error(PL_ERR_NOMEM, "%s: %s", what, cudaGetErrorString(e));
  return set_error(PL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

static unsigned* g_err_word[64];
static std::mutex g_err_mu;

unsigned* device_error_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> g(g_err_mu);
  if (!g_err_word[dev]) {
    unsigned* p = nullptr;
    if (cudaMalloc(&p, sizeof(unsigned)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(unsigned));
    g_err_word[dev] = p;
  }
  return g_err_word[dev];
}

int device_error_check() {
  unsigned* w = device_error_word();
  if (!w) return PL_OK;
  unsigned v = 0;
  PL_CUDA(cudaMemcpy(&v, w, sizeof(unsigned), cudaMemcpyDeviceToHost));
  if (v) {
    cudaMemset(w, 0, sizeof(unsigned));
    return set_error(PL_ERR_DEVICE_TIMEOUT, "a device-side bounded wait ran out (code 0x%x)", v);
  }
  return PL_OK;
}

// Requires a usable device; the library never computes on the host in place of the GPU.
int require_device() {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return set_error(PL_ERR_NO_DEVICE, "no usable CUDA device (%s); this library has no CPU fallback",
                     e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
  return PL_OK;
}

}  // namespace pl

extern "C" {

const char* pl_last_error(void) { return pl::g_err; }

int pl_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int pl_set_device(int device) {
  PL_CUDA(cudaSetDevice(device));
  return PL_OK;
}

uint64_t pl_kernel_launch_count(void) { return pl::g_launches.load(); }

}  // extern "C"

namespace pl {
static void* g_scratch[64][64];
static size_t g_scratch_sz[64][64];
static std::mutex g_scratch_mu;

void* scratch(int slot, size_t bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || slot < 0 || slot >= 64) {
    set_error(PL_ERR_INVALID, "scratch slot %d / device %d out of range", slot, dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> g(g_scratch_mu);
  if (bytes == 0) bytes = 16;
  if (g_scratch_sz[dev][slot] < bytes) {
    if (g_scratch[dev][slot]) cudaFree(g_scratch[dev][slot]);
    g_scratch[dev][slot] = nullptr;
    g_scratch_sz[dev][slot] = 0;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      check_cuda(e, "cudaMalloc(scratch)");
      return nullptr;
    }
    g_scratch[dev][slot] = p;
    g_scratch_sz[dev][slot] = bytes;
  }
  return g_scratch[dev][slot];
}
}  // namespace pl
