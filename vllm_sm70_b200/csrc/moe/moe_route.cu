// MoE routing kernels: router top-k, deterministic token->expert permutation,
// and the weighted combine.
//
//   moe_topk      logits [T, E] (bf16/fp32) -> softmax or sigmoid scores,
//                 top-k (ties -> lower expert id, NaN -> 0), optional
//                 renormalisation; weights fp32 [T, k], ids int32 [T, k].
//   moe_permute   ids [T, k] -> per-expert counts / offsets [E + 1] and, for
//                 every (token, slot) pair, its row in the expert-sorted
//                 buffer: pos [T, k]; rows inside one expert keep (token,
//                 slot) order, so the permutation is deterministic. Also
//                 gathers x rows into x_perm [T*k, H] and writes the inverse
//                 map src_row [T*k] (token index of each sorted row).
//   moe_combine   out[t] = sum_j w[t, j] * y[pos[t, j]] (+ shared[t]), summed
//                 in slot order in fp32 (no float atomics).
//
// Reference parity: the fused router (K13: sm70/csrc/router/flint_router.cuh:
// 1-186 -- sigmoid top-6, ties to the lower id, NaN -> 0, renormalise by the
// last CTA) and the TurboMind MoE helpers (strided tables, weighted reduce:
// sm70/csrc/turbomind/ops/tm_moe_sm70.cu:105-1407). Here: softmax or sigmoid,
// E <= 1024, k <= 16, plus an explicit expert-sorted layout for the grouped
// tcgen05 GEMM.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>

#include "moe/moe_api.h"

namespace b200 {
namespace {

constexpr int kMaxK = 16;

template <typename T>
__device__ __forceinline__ float ldf(const T* p, size_t i);
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) {
  return __bfloat162float(p[i]);
}
template <>
__device__ __forceinline__ float ldf<float>(const float* p, size_t i) { return p[i]; }

// One warp per token. Each lane scans E/32 experts; k rounds of warp argmax.
template <typename T>
__global__ void topk_kernel(const T* __restrict__ logits, int ld, int Tn, int E, int k,
                            bool use_sigmoid, bool renorm, const float* __restrict__ bias,
                            float* __restrict__ w_out, int* __restrict__ id_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= Tn) return;
  const T* row = logits + (size_t)warp * ld;
  // softmax denominator (max-subtracted) or sigmoid scores
  float mx = -INFINITY;
  for (int e = lane; e < E; e += 32) {
    float v = ldf(row, e);
    if (v != v) v = -INFINITY;
    mx = fmaxf(mx, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o));
  float den = 0.f;
  if (!use_sigmoid) {
    for (int e = lane; e < E; e += 32) {
      float v = ldf(row, e);
      den += (v != v) ? 0.f : __expf(v - mx);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffff, den, o);
  }
  float sel_w[kMaxK];
  int sel_id[kMaxK];
  float taken_sum = 0.f;
  for (int j = 0; j < k; ++j) {
    // best (score, -id) among experts not yet taken
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      bool taken = false;
      for (int q = 0; q < j; ++q) taken |= (sel_id[q] == e);
      if (taken) continue;
      float v = ldf(row, e);
      float sc = (v != v) ? 0.f : (use_sigmoid ? 1.f / (1.f + __expf(-v)) : __expf(v - mx) / den);
      const float key = sc + (bias ? bias[e] : 0.f);  // selection key (bias only selects)
      if (key > bv || (key == bv && e < bi)) {
        bv = key;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffff, bv, o);
      const int oi = __shfl_xor_sync(0xffffffff, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    sel_id[j] = bi;
    float v = ldf(row, bi);
    float sc = (v != v) ? 0.f : (use_sigmoid ? 1.f / (1.f + __expf(-v)) : __expf(v - mx) / den);
    sel_w[j] = sc;
    taken_sum += sc;
  }
  if (lane == 0) {
    const float inv = (renorm && taken_sum > 0.f) ? 1.f / taken_sum : 1.f;
    for (int j = 0; j < k; ++j) {
      w_out[(size_t)warp * k + j] = sel_w[j] * inv;
      id_out[(size_t)warp * k + j] = sel_id[j];
    }
  }
}

// One CTA per expert: counts the (token, slot) pairs routed to it and their
// order (block-wide prefix over the pair index), deterministic.
__global__ void expert_count_kernel(const int* __restrict__ ids, int pairs, int* __restrict__ counts,
                                    int* __restrict__ rank_in_expert, int E, int e_base) {
  const int e = blockIdx.x + e_base;
  __shared__ int warp_sums[32];
  __shared__ int running;
  if (threadIdx.x == 0) running = 0;
  __syncthreads();
  for (int base = 0; base < pairs; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const bool hit = i < pairs && ids[i] == e;
    const unsigned m = __ballot_sync(0xffffffff, hit);
    const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    const int before_in_warp = __popc(m & ((1u << lane) - 1u));
    if (lane == 0) warp_sums[warp] = __popc(m);
    __syncthreads();
    int before = running;
    for (int w = 0; w < warp; ++w) before += warp_sums[w];
    if (hit) rank_in_expert[i] = before + before_in_warp;
    __syncthreads();
    if (threadIdx.x == 0) {
      int tot = 0;
      for (int w = 0; w < (int)(blockDim.x / 32); ++w) tot += warp_sums[w];
      running += tot;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[e - e_base] = running;
}

// Expert start offsets; with align > 1 every expert's block starts at a
// multiple of `align` rows (the NVFP4 grouped GEMM reads its activation
// scales in 128-row atoms).
__global__ void offsets_kernel(const int* __restrict__ counts, int E, int* __restrict__ offsets,
                               int align) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = acc;
      acc += (counts[e] + align - 1) / align * align;
    }
    offsets[E] = acc;
  }
}

// pos[i] = offsets[ids[i] - e_base] + rank; gather x rows. Pairs routed to an
// expert outside [e_base, e_base + E) get pos = -1 (not local: EP).
__global__ void scatter_kernel(const int* __restrict__ ids, const int* __restrict__ rank_in_expert,
                               const int* __restrict__ offsets, int pairs, int k, int E, int e_base,
                               const __nv_bfloat16* __restrict__ x, int H,
                               __nv_bfloat16* __restrict__ x_perm, int* __restrict__ pos,
                               int* __restrict__ src_row) {
  const int i = blockIdx.x;  // pair index
  if (i >= pairs) return;
  const int e = ids[i] - e_base;
  const bool local = e >= 0 && e < E;
  const int p = local ? offsets[e] + rank_in_expert[i] : -1;
  if (threadIdx.x == 0) {
    pos[i] = p;
    if (local) src_row[p] = i / k;
  }
  if (!local || x == nullptr) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(i / k) * H);
  uint4* dst = reinterpret_cast<uint4*>(x_perm + (size_t)p * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}

__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ pos,
                               const float* __restrict__ w, int k, int H,
                               const __nv_bfloat16* __restrict__ shared, float shared_scale,
                               __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < H / 2; c += blockDim.x) {
    float a0 = 0.f, a1 = 0.f;
    for (int j = 0; j < k; ++j) {
      const int p = pos[(size_t)t * k + j];
      if (p < 0) continue;
      const float wj = w[(size_t)t * k + j];
      const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(y + (size_t)p * H)[c];
      a0 += wj * __low2float(v);
      a1 += wj * __high2float(v);
    }
    if (shared) {
      const __nv_bfloat162 s = reinterpret_cast<const __nv_bfloat162*>(shared + (size_t)t * H)[c];
      a0 += shared_scale * __low2float(s);
      a1 += shared_scale * __high2float(s);
    }
    reinterpret_cast<__nv_bfloat162*>(out + (size_t)t * H)[c] = __floats2bfloat162_rn(a0, a1);
  }
}

}  // namespace

void moe_topk_launch(const void* logits, bool bf16, int ld, int T, int E, int k, bool sigmoid,
                     bool renorm, const float* bias, float* w, int* ids, cudaStream_t stream) {
  if (T <= 0) return;
  if (k > kMaxK || k > E) throw std::runtime_error("moe_topk: k must be <= 16 and <= E");
  const int threads = 256;
  const int blocks = (T * 32 + threads - 1) / threads;
  if (bf16)
    topk_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(
        (const __nv_bfloat16*)logits, ld, T, E, k, sigmoid, renorm, bias, w, ids);
  else
    topk_kernel<float><<<blocks, threads, 0, stream>>>((const float*)logits, ld, T, E, k, sigmoid,
                                                       renorm, bias, w, ids);
}

void moe_permute_launch(const int* ids, int T, int k, int E, int e_base, const void* x, int H,
                        void* x_perm, int* counts, int* offsets, int* rank_scratch, int* pos,
                        int* src_row, cudaStream_t stream, int align) {
  const int pairs = T * k;
  if (E <= 0) return;
  expert_count_kernel<<<E, 256, 0, stream>>>(ids, pairs, counts, rank_scratch, E, e_base);
  offsets_kernel<<<1, 32, 0, stream>>>(counts, E, offsets, align < 1 ? 1 : align);
  if (pairs > 0)
    scatter_kernel<<<pairs, 128, 0, stream>>>(ids, rank_scratch, offsets, pairs, k, E, e_base,
                                               (const __nv_bfloat16*)x, H,
                                               (__nv_bfloat16*)x_perm, pos, src_row);
}

void moe_combine_launch(const void* y, const int* pos, const float* w, int T, int k, int H,
                        const void* shared, float shared_scale, void* out, cudaStream_t stream) {
  if (T <= 0) return;
  combine_kernel<<<T, 256, 0, stream>>>((const __nv_bfloat16*)y, pos, w, k, H,
                                        (const __nv_bfloat16*)shared, shared_scale,
                                        (__nv_bfloat16*)out);
}

}  // namespace b200
