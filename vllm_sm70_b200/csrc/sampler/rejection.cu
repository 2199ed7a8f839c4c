// Speculative-decoding rejection sampler (Leviathan et al. / Chen et al. 2023).
//
// Per row (request) with k draft tokens d_0..d_{k-1}:
//   p_i = softmax(target_logits[i] / T), q_i = softmax(draft_logits[i] / T)
//   for i in 0..k-1: accept d_i iff u_i * q_i(d_i) <= p_i(d_i)     (u_i ~ U(0,1))
//   first rejection at i: emit a sample of normalise(max(p_i - q_i, 0)), stop
//   all accepted:         emit a bonus sample of p_k
// T <= 0 degenerates to greedy verification (accept iff d_i == argmax p_i;
// the emitted token is argmax p_i). Outputs: out_tokens [rows, k+1] (unused
// slots = -1) and num_out [rows] (accepted + 1).
//
// Randomness: Philox4x32-10 keyed by (seed, row) at counter (offset, stream, i)
// (see sample.cu). Sampling from a distribution r uses the exponential race
// argmax_j r_j / E_j, E_j ~ Exp(1), which needs no normalisation.
//
// Reference parity: upstream vLLM's RejectionSampler used by the reference's
// spec-decode path, and the sparse rejection of the fork bundle
// (sm70/reference/fork-cf9492a/qwen-dflash2/sparse_rejection.py), here as one
// CUDA kernel per verify step.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>

#include "sampler/sampler_api.h"

namespace b200 {
namespace {

__device__ __forceinline__ void mulhilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  const unsigned long long p = (unsigned long long)a * b;
  hi = (uint32_t)(p >> 32);
  lo = (uint32_t)p;
}
__device__ __forceinline__ uint32_t philox_x(uint4 c, uint2 k) {
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
  return c.x;
}
__device__ __forceinline__ float urand(uint64_t seed, uint32_t row, uint64_t offset, uint32_t stream,
                                       uint32_t i) {
  const uint32_t x = philox_x(make_uint4(i, stream, (uint32_t)offset, row ^ (uint32_t)(offset >> 32)),
                              make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
  return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

constexpr int kThreads = 512;

__device__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = -INFINITY;
  for (int w = 0; w < kThreads / 32; ++w) r = fmaxf(r, red[w]);
  __syncthreads();
  return r;
}
__device__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
  for (int w = 0; w < kThreads / 32; ++w) r += red[w];
  __syncthreads();
  return r;
}
// argmax of score over the block; ties to the lower index.
__device__ int block_argmax(float s, int i, float* redv, int* redi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float os = __shfl_xor_sync(0xffffffff, s, o);
    const int oi = __shfl_xor_sync(0xffffffff, i, o);
    if (os > s || (os == s && oi < i)) {
      s = os;
      i = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    redv[threadIdx.x >> 5] = s;
    redi[threadIdx.x >> 5] = i;
  }
  __syncthreads();
  float bs = redv[0];
  int bi = redi[0];
  for (int w = 1; w < kThreads / 32; ++w)
    if (redv[w] > bs || (redv[w] == bs && redi[w] < bi)) {
      bs = redv[w];
      bi = redi[w];
    }
  __syncthreads();
  return bi;
}

__global__ void __launch_bounds__(kThreads)
rejection_kernel(const __nv_bfloat16* __restrict__ tgt, const __nv_bfloat16* __restrict__ drf,
                 const int* __restrict__ draft_ids, int k, int V, const float* __restrict__ temp,
                 const int64_t* __restrict__ seeds, uint64_t offset, int* __restrict__ out_tokens,
                 int* __restrict__ num_out) {
  __shared__ float red[kThreads / 32];
  __shared__ int redi[kThreads / 32];
  const int row = blockIdx.x;
  const float T = temp[row];
  const uint64_t seed = (uint64_t)seeds[row];
  int emitted = 0;
  for (int i = 0; i <= k; ++i) {
    const __nv_bfloat16* tl = tgt + ((size_t)row * (k + 1) + i) * V;
    const bool bonus = i == k;
    if (T <= 0.f) {
      // greedy verification
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int j = threadIdx.x; j < V; j += kThreads) {
        const float v = __bfloat162float(tl[j]);
        if (v > best || (v == best && j < bi)) {
          best = v;
          bi = j;
        }
      }
      const int am = block_argmax(best, bi, red, redi);
      if (threadIdx.x == 0) out_tokens[(size_t)row * (k + 1) + emitted] = am;
      ++emitted;
      if (bonus || am != draft_ids[(size_t)row * k + i]) break;
      continue;
    }
    // target distribution p_i
    float mt = -INFINITY;
    for (int j = threadIdx.x; j < V; j += kThreads) mt = fmaxf(mt, __bfloat162float(tl[j]) / T);
    mt = block_max(mt, red);
    float zt = 0.f;
    for (int j = threadIdx.x; j < V; j += kThreads) zt += __expf(__bfloat162float(tl[j]) / T - mt);
    zt = block_sum(zt, red);
    if (bonus) {
      float bs = -INFINITY;
      int bi = 0x7fffffff;
      for (int j = threadIdx.x; j < V; j += kThreads) {
        const float pj = __expf(__bfloat162float(tl[j]) / T - mt);
        const float s = pj / -__logf(urand(seed, row, offset, 2u + 2u * i, j));
        if (s > bs) { bs = s; bi = j; }
      }
      const int tok = block_argmax(bs, bi, red, redi);
      if (threadIdx.x == 0) out_tokens[(size_t)row * (k + 1) + emitted] = tok;
      ++emitted;
      break;
    }
    const __nv_bfloat16* dl = drf + ((size_t)row * k + i) * V;
    float md = -INFINITY;
    for (int j = threadIdx.x; j < V; j += kThreads) md = fmaxf(md, __bfloat162float(dl[j]) / T);
    md = block_max(md, red);
    float zd = 0.f;
    for (int j = threadIdx.x; j < V; j += kThreads) zd += __expf(__bfloat162float(dl[j]) / T - md);
    zd = block_sum(zd, red);
    const int d = draft_ids[(size_t)row * k + i];
    const float pd = __expf(__bfloat162float(tl[d]) / T - mt) / zt;
    const float qd = __expf(__bfloat162float(dl[d]) / T - md) / zd;
    const float u = urand(seed, row, offset, 1u, (uint32_t)i);
    if (u * qd <= pd) {
      if (threadIdx.x == 0) out_tokens[(size_t)row * (k + 1) + emitted] = d;
      ++emitted;
      continue;
    }
    // residual distribution max(p - q, 0)
    float bs = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = threadIdx.x; j < V; j += kThreads) {
      const float pj = __expf(__bfloat162float(tl[j]) / T - mt) / zt;
      const float qj = __expf(__bfloat162float(dl[j]) / T - md) / zd;
      const float r = fmaxf(pj - qj, 0.f);
      if (r > 0.f) {
        const float s = r / -__logf(urand(seed, row, offset, 3u + 2u * i, j));
        if (s > bs) { bs = s; bi = j; }
      }
    }
    int tok = block_argmax(bs, bi, red, redi);
    if (tok == 0x7fffffff) tok = d;  // p == q exactly: the draft was fine
    if (threadIdx.x == 0) out_tokens[(size_t)row * (k + 1) + emitted] = tok;
    ++emitted;
    break;
  }
  if (threadIdx.x == 0) {
    num_out[row] = emitted;
    for (int i = emitted; i <= k; ++i) out_tokens[(size_t)row * (k + 1) + i] = -1;
  }
}

}  // namespace

void rejection_sample_launch(const void* target_logits, const void* draft_logits,
                             const int* draft_ids, int rows, int k, int V, const float* temperature,
                             const int64_t* seeds, uint64_t offset, int* out_tokens, int* num_out,
                             cudaStream_t stream) {
  if (rows <= 0) return;
  if (k < 1 || k > 16) throw std::runtime_error("rejection_sample: 1 <= k <= 16");
  rejection_kernel<<<rows, kThreads, 0, stream>>>((const __nv_bfloat16*)target_logits,
                                                 (const __nv_bfloat16*)draft_logits, draft_ids, k,
                                                 V, temperature, seeds, offset, out_tokens,
                                                 num_out);
}

}  // namespace b200
