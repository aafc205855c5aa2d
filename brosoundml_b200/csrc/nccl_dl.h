// NCCL through dlopen (see nccl.cpp): communicator set-up and the gradient all-reduce.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace bsml {

void nccl_unique_id(void* out128);
void* nccl_comm_init(int nranks, const void* id128, int rank, int device, int timeout_ms);
void nccl_comm_destroy(void* comm);
void nccl_allreduce(void* comm, float* grads, int64_t n, bool average, cudaStream_t st);
// waits (bounded by the communicator's timeout) for the stream's work; aborts the
// communicator and raises on an NCCL error or when the deadline passes
void nccl_sync(void* comm, cudaStream_t st);
int nccl_version();

}  // namespace bsml
