// Collectives used by the data-parallel update (NCCL, resolved at run time).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include <vector>

namespace pl {
int comm_allreduce_f32(void* comm, float* buf, size_t n, cudaStream_t st);
int comm_allreduce_f64(void* comm, double* buf, size_t n, cudaStream_t st);
// One grouped broadcast per buffer, buffer i from rank roots[i].
int comm_broadcast_group(void* comm, const std::vector<float*>& bufs, const std::vector<size_t>& counts,
                         const std::vector<int>& roots, cudaStream_t st);
}  // namespace pl
