// Internal view of the NCCL communicator (fg_comm.cu) for the MLP step.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include "../../include/ferro_cuda.h"

namespace fg {
int comm_allreduce_mean(fg_comm *c, float *buf, size_t count, cudaStream_t st);
int comm_allreduce_sum(fg_comm *c, float *buf, size_t count, cudaStream_t st);
int comm_nranks(const fg_comm *c);
}  // namespace fg
