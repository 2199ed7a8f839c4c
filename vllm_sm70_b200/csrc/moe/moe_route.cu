// MoE routing kernels: router top-k, deterministic token->expert permutation,
// and the weighted combine.
//
//   moe_router    x [T, H] bf16, router weight [E, H] -> fp32 logits and the
//                 top-k below in one kernel (small T: decode steps).
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
#include <string>

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

// One warp selects one token's experts: softmax (max-subtracted) or sigmoid
// scores, k rounds of warp argmax over the experts not yet taken (ties to the
// lower id, NaN logits score 0, `bias` only shifts the selection key), then
// the optional renormalisation; lane 0 writes the row.
template <typename T>
__device__ void warp_topk(const T* __restrict__ row, int E, int k, bool use_sigmoid, bool renorm,
                          const float* __restrict__ bias, float* __restrict__ w_row,
                          int* __restrict__ id_row) {
  const int lane = threadIdx.x % 32;
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
      w_row[j] = sel_w[j] * inv;
      id_row[j] = sel_id[j];
    }
  }
}

// One warp per token.
template <typename T>
__global__ void topk_kernel(const T* __restrict__ logits, int ld, int Tn, int E, int k,
                            bool use_sigmoid, bool renorm, const float* __restrict__ bias,
                            float* __restrict__ w_out, int* __restrict__ id_out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  if (warp >= Tn) return;
  warp_topk(logits + (size_t)warp * ld, E, k, use_sigmoid, renorm, bias,
            w_out + (size_t)warp * k, id_out + (size_t)warp * k);
}

// Fused router for small token counts: logits = x @ wr^T in fp32 and the
// top-k selection in one kernel. Grid (token tiles of kRtTok, expert chunks
// of 32); 8 warps, warp w computes experts chunk * 32 + 4w .. + 3 for the
// tile's tokens (x tile staged in shared memory, each lane 8 columns of H
// per step, fixed summation order), a 31-shuffle reduce-scatter leaves
// (token, expert) = lane's sum in that lane. Every CTA stores its fp32
// logits; the last CTA of a token tile (arrival counter, re-armed by that
// CTA) runs warp_topk for the tile's tokens on them. Deterministic: the
// logits do not depend on which CTA arrives last.
constexpr int kRtTok = 8;

__global__ void __launch_bounds__(256) router_kernel(
    const __nv_bfloat16* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ wr, int Tn,
    int E, int H, int k, bool use_sigmoid, bool renorm, const float* __restrict__ bias,
    float* __restrict__ logits, int* __restrict__ tile_ctr, float* __restrict__ w_out,
    int* __restrict__ id_out) {
  extern __shared__ uint4 xs4[];  // [kRtTok][H / 8]
  __shared__ int s_last;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int t0 = blockIdx.x * kRtTok;
  const int nt = min(kRtTok, Tn - t0);
  const int hv = H / 8;
  for (int i = threadIdx.x; i < kRtTok * hv; i += blockDim.x) {
    const int t = i / hv, c = i - t * hv;
    xs4[i] = t < nt ? *reinterpret_cast<const uint4*>(x + (size_t)(t0 + t) * ldx + c * 8)
                    : make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int e0 = blockIdx.y * 32 + warp * 4;
  float acc[kRtTok * 4];
#pragma unroll
  for (int i = 0; i < kRtTok * 4; ++i) acc[i] = 0.f;
  for (int c = lane; c < hv; c += 32) {
    float wf[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + j;
      const uint4 u = e < E ? *reinterpret_cast<const uint4*>(wr + (size_t)e * H + c * 8)
                            : make_uint4(0, 0, 0, 0);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h2[q]);
        wf[j][2 * q] = f.x;
        wf[j][2 * q + 1] = f.y;
      }
    }
#pragma unroll
    for (int t = 0; t < kRtTok; ++t) {
      const uint4 u = xs4[t * hv + c];
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
      float xf[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h2[q]);
        xf[2 * q] = f.x;
        xf[2 * q + 1] = f.y;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a = acc[t * 4 + j];
#pragma unroll
        for (int q = 0; q < 8; ++q) a = fmaf(xf[q], wf[j][q], a);
        acc[t * 4 + j] = a;
      }
    }
  }
  // Reduce-scatter over the warp: afterwards lane l holds the sum of acc[l].
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? acc[i] : acc[i + o];
      const float keep = upper ? acc[i + o] : acc[i];
      acc[i] = keep + __shfl_xor_sync(0xffffffff, send, o);
    }
  }
  {
    const int t = lane / 4, e = e0 + (lane & 3);
    if (t < nt && e < E) logits[(size_t)(t0 + t) * E + e] = acc[0];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(&tile_ctr[blockIdx.x], 1);
    s_last = old == (int)gridDim.y - 1;
    if (s_last) tile_ctr[blockIdx.x] = 0;  // re-arm for the next launch
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (!s_last) return;
  __threadfence();
  if (warp < nt)
    warp_topk(logits + (size_t)(t0 + warp) * E, E, k, use_sigmoid, renorm, bias,
              w_out + (size_t)(t0 + warp) * k, id_out + (size_t)(t0 + warp) * k);
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

void moe_router_launch(const void* x, int ldx, const void* wr, int T, int E, int H, int k,
                       bool sigmoid, bool renorm, const float* bias, float* logits,
                       int* tile_ctr, float* w, int* ids, cudaStream_t stream) {
  if (T <= 0) return;
  if (k > kMaxK || k > E) throw std::runtime_error("moe_router: k must be <= 16 and <= E");
  if (H % 8) throw std::runtime_error("moe_router: H must be a multiple of 8");
  const size_t smem = (size_t)kRtTok * H * 2;
  if (smem > 96 * 1024) throw std::runtime_error("moe_router: hidden size too large");
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)((T + kRtTok - 1) / kRtTok), (unsigned)((E + 31) / 32), 1);
  lc.blockDim = dim3(256, 1, 1);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&lc, router_kernel, (const __nv_bfloat16*)x, ldx,
                                     (const __nv_bfloat16*)wr, T, E, H, k, sigmoid, renorm, bias,
                                     logits, tile_ctr, w, ids);
  if (e != cudaSuccess) throw std::runtime_error(std::string("moe_router: ") + cudaGetErrorString(e));
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
