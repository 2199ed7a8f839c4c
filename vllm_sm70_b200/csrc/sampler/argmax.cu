// Greedy sampling: row-wise argmax over bf16/fp32 logits.
// Tie rule: NaN wins (first NaN), otherwise the largest value, lowest index on
// ties -- the same total order as the reference's top-1 exchange
// (sm70/csrc/custom_ar/top1_custom_ar.cu:52-101), so a per-rank partial
// argmax merged in rank order gives the same token as a full-vocab argmax.
// Also emits the row's max value, which the vocab-parallel path exchanges.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>

#include "ops_api.h"
#include "common/launch.h"

namespace b200 {
namespace {

struct VI {
  float v;
  int i;
};

__device__ __forceinline__ bool better(const VI& a, const VI& b) {
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an != bn) return an;
  if (an && bn) return a.i < b.i;
  if (a.v != b.v) return a.v > b.v;
  return a.i < b.i;
}

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }

template <typename T>
__global__ void argmax_kernel(const T* __restrict__ logits, int V, int ld, int* __restrict__ ids,
                              float* __restrict__ vals, int id_offset) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const T* x = logits + (size_t)row * ld;
  VI best{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    VI c{to_f(x[i]), i};
    if (better(c, best)) best = c;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    VI other{__shfl_xor_sync(0xffffffff, best.v, o), __shfl_xor_sync(0xffffffff, best.i, o)};
    if (better(other, best)) best = other;
  }
  __shared__ VI red[32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    VI b = red[0];
    for (int w = 1; w < (int)blockDim.x / 32; ++w)
      if (better(red[w], b)) b = red[w];
    ids[row] = b.i + id_offset;
    if (vals) vals[row] = b.v;
  }
}

}  // namespace

void argmax_launch(const void* logits, bool is_bf16, int rows, int V, int ld, int* ids,
                   float* vals, int id_offset, cudaStream_t stream) {
  if (rows <= 0) return;
  if (is_bf16)
    launch_pdl(argmax_kernel<__nv_bfloat16>, dim3(rows), dim3(1024), 0, stream, nullptr,
               (const __nv_bfloat16*)logits, V, ld, ids, vals, id_offset);
  else
    launch_pdl(argmax_kernel<float>, dim3(rows), dim3(1024), 0, stream, nullptr,
               (const float*)logits, V, ld, ids, vals, id_offset);
}

}  // namespace b200
