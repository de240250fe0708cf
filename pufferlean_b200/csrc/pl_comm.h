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
// All-gather of count bf16 values per rank: rank r's send lands at recv + r * count (in place when
// send == recv + rank * count).
int comm_allgather_bf16(void* comm, const void* send, void* recv, size_t count, cudaStream_t st);
// Rank and world size of a live communicator.
int comm_rank_world(void* comm, int* rank, int* world);
}  // namespace pl
