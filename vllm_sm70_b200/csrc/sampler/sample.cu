// Random sampling kernels.
//
// * gumbel_argmax: exact sampling from softmax(logits / T) by the Gumbel-max
//   trick: token = argmax_i(logit_i / T + G_i), G_i = -log(-log(u_i)), u_i from
//   Philox4x32-10 keyed by (seed, row) at counter (offset, i). Rows with
//   T <= 0 are greedy. Because it is an argmax, the vocab-parallel merge of
//   per-rank (value, id) pairs (the greedy merge) gives the exact global
//   sample with one tiny all-gather.
// * topk_candidates: per-row top-K (K <= 64) of a logit shard by a two-pass
//   radix select on the order-preserving 16/32-bit key, ties to the lower id,
//   sorted descending -- the candidate set for top-k / top-p sampling.
// * sample_candidates: temperature, top-k, top-p (nucleus) over the candidate
//   set, then an exponential race (argmax p_i / E_i, E_i ~ Exp(1) from Philox).
//
// Philox4x32-10 follows Salmon et al., "Parallel random numbers: as easy as
// 1, 2, 3" (SC'11): 10 rounds of the published multiply/xor round function
// and Weyl key schedule.
//
// Reference parity: the top-k candidate sampler (K16:
// sm70/csrc/sampler/topk_candidates_sampler.cu:80-448: local top-32 per rank,
// all-gather, temperature/top-k/top-p/exponential race) and the greedy F12
// path. Here the candidate count is K <= 64 per rank and TP <= 8.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>

#include "sampler/sampler_api.h"
#include "common/launch.h"

namespace b200 {
namespace {

__device__ __forceinline__ void mulhilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  const unsigned long long p = (unsigned long long)a * b;
  hi = (uint32_t)(p >> 32);
  lo = (uint32_t)p;
}

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo(M0, c.x, hi0, lo0);
    mulhilo(M1, c.z, hi1, lo1);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += W0;
    k.y += W1;
  }
  return c;
}

// Uniform in (0, 1): 24 random bits, centred in their interval (never 0 or 1).
__device__ __forceinline__ float u01(uint32_t x) {
  return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ float rand_u01(uint64_t seed, uint64_t row, uint64_t offset,
                                          uint32_t i) {
  const uint4 c = make_uint4(i, (uint32_t)offset, (uint32_t)(offset >> 32), (uint32_t)row);
  const uint2 k = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
  return u01(philox4x32_10(c, k).x);
}

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }

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
__global__ void gumbel_argmax_kernel(const T* __restrict__ logits, int V, int ld,
                                     const float* __restrict__ temperature,
                                     const int64_t* __restrict__ seeds, uint64_t offset,
                                     const int64_t* __restrict__ row_offsets, int id_offset,
                                     int* __restrict__ ids, float* __restrict__ vals) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const T* x = logits + (size_t)row * ld;
  const float t = temperature[row];
  const uint64_t seed = (uint64_t)seeds[row];
  if (row_offsets) offset += (uint64_t)row_offsets[row];
  VI best{-INFINITY, 0x7fffffff};
  auto visit = [&](float v, int i) {
    if (t > 0.f && v == v) {
      const float u = rand_u01(seed, 0, offset, (uint32_t)(i + id_offset));
      v = v / t - __logf(-__logf(u));
    }
    const VI c{v, i};
    if (better(c, best)) best = c;
  };
  // 16-byte vector loads when the row allows them (the row is read once, so
  // the load width sets the rate).
  constexpr int E = 16 / sizeof(T);
  int done = 0;
  if (ld % E == 0 && (reinterpret_cast<uintptr_t>(logits) & 15u) == 0) {
    const int nv = V / E;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int j = threadIdx.x; j < nv; j += blockDim.x) {
      const uint4 raw = __ldg(xv + j);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int k = 0; k < E; ++k) visit(to_f(e[k]), j * E + k);
    }
    done = nv * E;
  }
  for (int i = done + threadIdx.x; i < V; i += blockDim.x) visit(to_f(x[i]), i);
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
    vals[row] = b.v;
  }
}

// Order-preserving 32-bit key of a float (larger float -> larger key; NaN
// treated as -inf so it is never a candidate).
__device__ __forceinline__ uint32_t fkey(float f) {
  if (f != f) f = -INFINITY;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// One CTA per row: radix select of the K-th largest key over 4 passes of 8
// bits, then collect keys > threshold and the lowest-index keys == threshold.
template <typename T>
__global__ void topk_candidates_kernel(const T* __restrict__ logits, int V, int ld, int K,
                                       int id_offset, float* __restrict__ out_v,
                                       int* __restrict__ out_i) {
  pdl_wait();
  pdl_trigger();
  __shared__ int hist[256];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int s_need;
  __shared__ int s_cnt_gt, s_cnt_eq;
  __shared__ float cv[64];
  __shared__ int ci[64];
  const int row = blockIdx.x;
  const T* x = logits + (size_t)row * ld;
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_need = K;
  }
  __syncthreads();
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const uint32_t key = fkey(to_f(x[i]));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xff], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int need = s_need;
      int b = 255;
      for (; b > 0; --b) {
        if (hist[b] >= need) break;
        need -= hist[b];
      }
      s_prefix = prefix | ((uint32_t)b << shift);
      s_mask = mask | (0xffu << shift);
      s_need = need;  // how many keys equal to the final threshold to take
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;
  if (threadIdx.x == 0) {
    s_cnt_gt = 0;
    s_cnt_eq = 0;
  }
  __syncthreads();
  // keys strictly greater than the threshold: exactly K - need of them
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float f = to_f(x[i]);
    if (fkey(f) > thr) {
      const int slot = atomicAdd(&s_cnt_gt, 1);
      cv[slot] = f;
      ci[slot] = i;
    }
  }
  __syncthreads();
  // ties at the threshold: take the lowest indices (serial scan, deterministic)
  if (threadIdx.x == 0) {
    int n = s_cnt_gt;
    for (int i = 0; i < V && n < K; ++i) {
      const float f = to_f(x[i]);
      if (fkey(f) == thr) {
        cv[n] = f;
        ci[n] = i;
        ++n;
      }
    }
    // insertion sort descending (value, then lower id) -- K <= 64
    for (int a = 1; a < n; ++a) {
      const float v = cv[a];
      const int id = ci[a];
      int b = a - 1;
      while (b >= 0 && (cv[b] < v || (cv[b] == v && ci[b] > id))) {
        cv[b + 1] = cv[b];
        ci[b + 1] = ci[b];
        --b;
      }
      cv[b + 1] = v;
      ci[b + 1] = id;
    }
    for (int a = 0; a < K; ++a) {
      out_v[(size_t)row * K + a] = a < n ? cv[a] : -INFINITY;
      out_i[(size_t)row * K + a] = a < n ? ci[a] + id_offset : -1;
    }
  }
}

// One CTA (256 threads) per row over C <= 512 candidates (merged across
// ranks): bitonic sort by (value desc, id asc) in smem, softmax of the top-k
// at temperature T, nucleus cut (keep the smallest prefix whose mass reaches
// top_p), then an exponential race over the kept prefix.
__global__ void sample_candidates_kernel(const float* __restrict__ cand_v,
                                         const int* __restrict__ cand_i, int C,
                                         const float* __restrict__ temperature,
                                         const int* __restrict__ top_k,
                                         const float* __restrict__ top_p,
                                         const int64_t* __restrict__ seeds, uint64_t offset,
                                         int* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  constexpr int CMAX = 512;
  __shared__ float sv[CMAX];
  __shared__ int si[CMAX];
  __shared__ float sp[CMAX];
  __shared__ int s_keep;
  __shared__ float s_best[8];
  __shared__ int s_besti[8];
  const int row = blockIdx.x;
  int P = 1;
  while (P < C) P <<= 1;
  for (int j = threadIdx.x; j < P; j += blockDim.x) {
    const bool ok = j < C && cand_i[(size_t)row * C + j] >= 0;
    sv[j] = ok ? cand_v[(size_t)row * C + j] : -INFINITY;
    si[j] = ok ? cand_i[(size_t)row * C + j] : 0x7fffffff;
  }
  __syncthreads();
  // bitonic sort, "before" = larger value, then smaller id
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int j = threadIdx.x; j < P; j += blockDim.x) {
        const int partner = j ^ stride;
        if (partner > j) {
          const bool desc = (j & size) == 0;
          const bool j_before = sv[j] > sv[partner] || (sv[j] == sv[partner] && si[j] < si[partner]);
          if (desc != j_before) {
            const float tv = sv[j]; sv[j] = sv[partner]; sv[partner] = tv;
            const int ti = si[j]; si[j] = si[partner]; si[partner] = ti;
          }
        }
      }
      __syncthreads();
    }
  }
  int valid = 0;
  for (int j = 0; j < C; ++j) valid += (si[j] != 0x7fffffff);  // uniform across threads
  const float t = temperature[row];
  if (t <= 0.f || valid == 0) {
    if (threadIdx.x == 0) out[row] = valid ? si[0] : -1;
    return;
  }
  const int kk = top_k[row] > 0 ? min(top_k[row], valid) : valid;
  const float mx = sv[0];
  for (int j = threadIdx.x; j < kk; j += blockDim.x) sp[j] = __expf((sv[j] - mx) / t);
  __syncthreads();
  if (threadIdx.x == 0) {
    float Z = 0.f;
    for (int j = 0; j < kk; ++j) Z += sp[j];
    const float cap = top_p[row] * Z;
    float acc = 0.f;
    int keep = kk;
    for (int j = 0; j < kk; ++j) {
      acc += sp[j];
      if (acc >= cap) {
        keep = j + 1;
        break;
      }
    }
    s_keep = keep;
  }
  __syncthreads();
  const int keep = s_keep;
  float best = -INFINITY;
  int besti = 1 << 30;
  for (int j = threadIdx.x; j < keep; j += blockDim.x) {
    const float e = -__logf(rand_u01((uint64_t)seeds[row], 1, offset, (uint32_t)si[j]));
    const float score = sp[j] / e;
    if (score > best) {
      best = score;
      besti = j;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffff, best, o);
    const int oi = __shfl_xor_sync(0xffffffff, besti, o);
    if (ob > best || (ob == best && oi < besti)) {
      best = ob;
      besti = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    s_best[threadIdx.x / 32] = best;
    s_besti[threadIdx.x / 32] = besti;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)blockDim.x / 32; ++w)
      if (s_best[w] > best || (s_best[w] == best && s_besti[w] < besti)) {
        best = s_best[w];
        besti = s_besti[w];
      }
    out[row] = si[besti];
  }
}

}  // namespace

void gumbel_argmax_launch(const void* logits, bool bf16, int rows, int V, int ld,
                          const float* temperature, const int64_t* seeds, uint64_t offset,
                          const int64_t* row_offsets, int id_offset, int* ids, float* vals,
                          cudaStream_t stream) {
  if (rows <= 0) return;
  if (bf16)
    launch_pdl(gumbel_argmax_kernel<__nv_bfloat16>, dim3(rows), dim3(1024), 0, stream, nullptr,
               (const __nv_bfloat16*)logits, V, ld, temperature, seeds, offset, row_offsets,
               id_offset, ids, vals);
  else
    launch_pdl(gumbel_argmax_kernel<float>, dim3(rows), dim3(1024), 0, stream, nullptr,
               (const float*)logits, V, ld, temperature, seeds, offset, row_offsets, id_offset,
               ids, vals);
}

void topk_candidates_launch(const void* logits, bool bf16, int rows, int V, int ld, int K,
                            int id_offset, float* out_v, int* out_i, cudaStream_t stream) {
  if (rows <= 0) return;
  if (K < 1 || K > 64) throw std::runtime_error("topk_candidates: K must be in [1, 64]");
  if (bf16)
    launch_pdl(topk_candidates_kernel<__nv_bfloat16>, dim3(rows), dim3(512), 0, stream, nullptr,
               (const __nv_bfloat16*)logits, V, ld, K, id_offset, out_v, out_i);
  else
    launch_pdl(topk_candidates_kernel<float>, dim3(rows), dim3(512), 0, stream, nullptr,
               (const float*)logits, V, ld, K, id_offset, out_v, out_i);
}

void sample_candidates_launch(const float* cand_v, const int* cand_i, int rows, int C,
                              const float* temperature, const int* top_k, const float* top_p,
                              const int64_t* seeds, uint64_t offset, int* out,
                              cudaStream_t stream) {
  if (rows <= 0) return;
  if (C > 512) throw std::runtime_error("sample_candidates: at most 512 candidates");
  launch_pdl(sample_candidates_kernel, dim3(rows), dim3(256), 0, stream, nullptr, cand_v, cand_i,
             C, temperature, top_k, top_p, seeds, offset, out);
}

}  // namespace b200
