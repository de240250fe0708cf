// Shared definitions for the B200 PPO+Muon update library: status codes, the per-thread
// error message behind pl_last_error(), launch checks, and small device helpers.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/pufferlean_b200.h"

namespace pl {

// Records a formatted message as this thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();
int check_cuda(cudaError_t e, const char* what);

#define PL_CUDA(call)                                          \
  do {                                                         \
    cudaError_t _e = (call);                                   \
    if (_e != cudaSuccess) return ::pl::check_cuda(_e, #call); \
  } while (0)

#define PL_LAUNCH(what)                                        \
  do {                                                         \
    cudaError_t _e = cudaGetLastError();                       \
    if (_e != cudaSuccess) return ::pl::check_cuda(_e, what);  \
  } while (0)

#define PL_REQUIRE(cond, code, ...)                            \
  do {                                                         \
    if (!(cond)) return ::pl::set_error((code), __VA_ARGS__);  \
  } while (0)

static inline long ceil_div(long a, long b) { return (a + b - 1) / b; }
static inline long round_up(long a, long b) { return (a + b - 1) / b * b; }

// Per-device word that kernels with bounded waits set when a wait runs out (0 = none).
unsigned* device_error_word();
// Reads and clears the word (synchronizes the device). Returns PL_OK or PL_ERR_DEVICE_TIMEOUT.
int device_error_check();

}  // namespace pl

#define PL_ERR_MBAR_TIMEOUT 0x100u
