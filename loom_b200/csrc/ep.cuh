// ep.cuh -- expert parallelism: the NCCL communicator of the backend (one
// process per GPU) and the combine of the ranks' partial MoE outputs.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include <string>

namespace loom {

bool ep_active();
int ep_rank();
int ep_size();
// out[i] = sum over ranks of out[i] (in place), on stream st
int ep_allreduce_sum(float *buf, size_t n, cudaStream_t st, std::string &err);

}  // namespace loom
