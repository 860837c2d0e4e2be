// Internal view of the NCCL communicator (fg_comm.cu) for the MLP step.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include "../../include/ferro_cuda.h"

namespace fg {
int comm_allreduce_mean(fg_comm *c, float *buf, size_t count, cudaStream_t st);
int comm_allreduce_sum(fg_comm *c, float *buf, size_t count, cudaStream_t st);
int comm_nranks(const fg_comm *c);
// SMs the data-parallel step leaves to the collective while its backward
// GEMMs run (FG_COMM_SM_RESERVE, default kCommSmReserve); the communicator
// is created with at most that many CTAs per collective.
constexpr int kCommSmReserve = 20;
int comm_sm_reserve();
}  // namespace fg
