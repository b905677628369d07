// nccl_plain.h — a plain NCCL communicator (float sum all-reduce) on the library's run-time loaded
// NCCL (comm.cpp), for contexts other than the generator's bucketed one.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>

namespace wb {
int nccl_plain_init(void** comm, int rank, int world, const void* id128);
int nccl_plain_allreduce_sum(void* comm, float* buf, size_t n, cudaStream_t st);
int nccl_plain_async_error(void* comm);  // 0 or WUBU_B200_ERR_COMM
void nccl_plain_abort(void* comm);
void nccl_plain_destroy(void* comm);
}  // namespace wb
