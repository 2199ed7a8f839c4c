// Block-size-independent row reduction: the caller stores one partial per
// 8-element vector i in part[i] (i in [0, n)); lane j of warp 0 adds
// part[j], part[j + 32], ... in index order, then the 32 lane sums meet in a
// fixed xor butterfly. The result depends only on the partials, never on the
// number of threads that produced them, so a norm computed by kernels with
// different block sizes (the standalone RMSNorm, the NVLink collective, the
// GEMM that runs the collective as its last phase) rounds identically.
#pragma once
#include <cuda_runtime.h>

namespace b200 {

__device__ __forceinline__ float canonical_block_sum(const float* part, int n, float* bcast) {
  __syncthreads();  // every partial stored
  if (threadIdx.x < 32) {
    float a = 0.f;
    for (int i = threadIdx.x; i < n; i += 32) a += part[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (threadIdx.x == 0) *bcast = a;
  }
  __syncthreads();
  return *bcast;
}

}  // namespace b200
