// Rollout-side column producer: the device scatters that turn a rollout's per-step outputs into the
// update's resident columns (row e*T + t, env-major), so the columns never pass through the host.
// The reference stamps its MinGRU columns the same way (ffi/puffercuda.cu:242-309: k_mg_cols_alv per
// rollout step, k_mg_cols_rt_all for the whole-update reward / terminal planes) and scatters the obs
// trajectory per step into g_dObsTraj (ffi/puffercuda.cu:975-983).
#include "../../include/pufferlean_b200.h"
#include "pl_common.cuh"
#include "pl_mlp.cuh"
#include "pl_runtime.h"

namespace pl {

// col[((e0 + i / width) * T + step) * width + i % width] = src[i], i < ne * width
template <typename V>
__global__ void stamp_rows_kernel(V* __restrict__ col, long width, long T, long step, long e0, long ne,
                                  const V* __restrict__ src) {
  const long n = ne * width;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long e = e0 + i / width, c = i - (i / width) * width;
    col[(e * T + step) * width + c] = src[i];
  }
}
// col[e * T + s] = plane[s * N + e]: a step-major [T x N] plane into the env-major column
__global__ void stamp_plane_kernel(double* __restrict__ col, long N, long T, const double* __restrict__ plane) {
  const long n = N * T;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long s = i / N, e = i - s * N;
    col[e * T + s] = plane[i];
  }
}
static inline unsigned grid_of(long n) {
  long g = (n + 255) / 256;
  if (g < 1) g = 1;
  if (g > 148 * 16) g = 148 * 16;
  return (unsigned)g;
}

int launch_stamp_rows_f64(double* col, long width, long T, long step, long e0, long ne, const double* src,
                          cudaStream_t st) {
  if (ne <= 0 || width <= 0) return PL_OK;
  stamp_rows_kernel<double><<<grid_of(ne * width), 256, 0, st>>>(col, width, T, step, e0, ne, src);
  count_launch();
  PL_LAUNCH("stamp_rows_kernel");
  return PL_OK;
}
int launch_stamp_rows_f32(float* col, long width, long T, long step, long e0, long ne, const float* src,
                          cudaStream_t st) {
  if (ne <= 0 || width <= 0) return PL_OK;
  stamp_rows_kernel<float><<<grid_of(ne * width), 256, 0, st>>>(col, width, T, step, e0, ne, src);
  count_launch();
  PL_LAUNCH("stamp_rows_kernel");
  return PL_OK;
}
int launch_stamp_plane(double* col, long N, long T, const double* plane, cudaStream_t st) {
  if (N <= 0 || T <= 0) return PL_OK;
  stamp_plane_kernel<<<grid_of(N * T), 256, 0, st>>>(col, N, T, plane);
  count_launch();
  PL_LAUNCH("stamp_plane_kernel");
  return PL_OK;
}

}  // namespace pl

extern "C" {

int pl_stamp_rows_f64(double* col, size_t width, size_t N, size_t T, size_t step, size_t e0, size_t ne,
                      const double* src, void* stream) {
  using namespace pl;
  PL_REQUIRE(col && src && width > 0, PL_ERR_INVALID, "pl_stamp_rows_f64: NULL column or source");
  PL_REQUIRE(step < T && e0 + ne <= N, PL_ERR_INVALID, "pl_stamp_rows_f64: step %zu / envs [%zu, %zu) outside %zu x %zu",
             step, e0, e0 + ne, N, T);
  return launch_stamp_rows_f64(col, (long)width, (long)T, (long)step, (long)e0, (long)ne, src, (cudaStream_t)stream);
}

int pl_stamp_rows_f32(float* col, size_t width, size_t N, size_t T, size_t step, size_t e0, size_t ne,
                      const float* src, void* stream) {
  using namespace pl;
  PL_REQUIRE(col && src && width > 0, PL_ERR_INVALID, "pl_stamp_rows_f32: NULL column or source");
  PL_REQUIRE(step < T && e0 + ne <= N, PL_ERR_INVALID, "pl_stamp_rows_f32: step %zu / envs [%zu, %zu) outside %zu x %zu",
             step, e0, e0 + ne, N, T);
  return launch_stamp_rows_f32(col, (long)width, (long)T, (long)step, (long)e0, (long)ne, src, (cudaStream_t)stream);
}

int pl_stamp_plane_f64(double* col, size_t N, size_t T, const double* plane, void* stream) {
  using namespace pl;
  PL_REQUIRE(col && plane, PL_ERR_INVALID, "pl_stamp_plane_f64: NULL column or plane");
  return launch_stamp_plane(col, (long)N, (long)T, plane, (cudaStream_t)stream);
}

}  // extern "C"
