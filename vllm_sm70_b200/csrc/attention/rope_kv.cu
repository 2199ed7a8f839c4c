// Fused (optional per-head q/k RMSNorm) + NeoX RoPE + paged KV-cache write.
//
// qkv [T, (Hq + 2 Hkv) * D] bf16 is the QKV projection output. In place, q and
// k are normalised (when q_norm / k_norm are given) and rotated; k and v are
// then written to k_cache / v_cache [num_blocks, Hkv, BS, D] at
// slot_mapping[t] = block * BS + offset (negative slot: token not cached).
// The attention kernel reads q straight from qkv with a token stride of
// (Hq + 2 Hkv) * D, so no separate q buffer is written.
//
// One warp per (token, head), D/64 rotation pairs per lane (any rotary
// width); full-width rotation takes the 16-byte-access variant below.
//
// Reference parity: the Triton q/k-norm + RoPE + KV writer
// (sm70/vllm_sm70/flint/qk_norm_rope_kv.py:55-148), here as a CUDA kernel.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>

#include "ops_api.h"
#include "common/launch.h"

namespace b200 {
namespace {

template <int D>
__global__ void rope_kv_kernel(__nv_bfloat16* __restrict__ qkv, const int64_t* __restrict__ pos,
                               const float* __restrict__ cos_sin, __nv_bfloat16* __restrict__ kc,
                               __nv_bfloat16* __restrict__ vc, const int64_t* __restrict__ slots,
                               const __nv_bfloat16* __restrict__ q_norm,
                               const __nv_bfloat16* __restrict__ k_norm, int T, int Hq, int Hkv,
                               int BS, float eps, int rot_dim, long long blk_stride) {
  pdl_wait();
  pdl_trigger();
  constexpr int P = D / 64;  // pairs per lane (first-half index i, second-half i + D/2)
  const int warps_per_block = blockDim.x / 32;
  const int gw = blockIdx.x * warps_per_block + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int heads = Hq + 2 * Hkv;
  const int t = gw / heads;
  const int h = gw % heads;
  if (t >= T) return;
  const size_t row = (size_t)t * heads * D;
  __nv_bfloat16* hp = qkv + row + (size_t)h * D;
  const bool is_q = h < Hq;
  const bool is_k = !is_q && h < Hq + Hkv;
  const bool is_v = h >= Hq + Hkv;
  const int64_t slot = slots ? slots[t] : -1;

  float a[P], b[P];
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const int i = lane + 32 * j;
    a[j] = __bfloat162float(hp[i]);
    b[j] = __bfloat162float(hp[i + D / 2]);
  }
  if (!is_v) {
    const __nv_bfloat16* nw = is_q ? q_norm : k_norm;
    if (nw != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < P; ++j) ss += a[j] * a[j] + b[j] * b[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
      const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
      for (int j = 0; j < P; ++j) {
        const int i = lane + 32 * j;
        a[j] = __bfloat162float(__float2bfloat16_rn(a[j] * inv)) * __bfloat162float(nw[i]);
        b[j] = __bfloat162float(__float2bfloat16_rn(b[j] * inv)) * __bfloat162float(nw[i + D / 2]);
      }
    }
    // NeoX rotation over the first rot_dim dims (pairs i, i + rot_dim/2).
    const int half = rot_dim / 2;
    const float* cs = cos_sin + (size_t)pos[t] * rot_dim;
    if (rot_dim == D) {
#pragma unroll
      for (int j = 0; j < P; ++j) {
        const int i = lane + 32 * j;
        const float c = cs[i], s = cs[half + i];
        const float x1 = a[j], x2 = b[j];
        a[j] = x1 * c - x2 * s;
        b[j] = x2 * c + x1 * s;
      }
    }
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int i = lane + 32 * j;
      hp[i] = __float2bfloat16_rn(a[j]);
      hp[i + D / 2] = __float2bfloat16_rn(b[j]);
    }
    if (rot_dim != D) {
      // Partial rotary (rot_dim < D): rotate pairs (i, i + half) for i < half.
      __syncwarp();
      for (int i = lane; i < half; i += 32) {
        const float c = cs[i], s = cs[half + i];
        const float x1 = __bfloat162float(hp[i]), x2 = __bfloat162float(hp[i + half]);
        hp[i] = __float2bfloat16_rn(x1 * c - x2 * s);
        hp[i + half] = __float2bfloat16_rn(x2 * c + x1 * s);
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < P; ++j) {
        const int i = lane + 32 * j;
        a[j] = __bfloat162float(hp[i]);
        b[j] = __bfloat162float(hp[i + D / 2]);
      }
    }
  }
  if ((is_k || is_v) && slot >= 0) {
    const int kvh = is_k ? h - Hq : h - Hq - Hkv;
    const int64_t blk = slot / BS, off = slot % BS;
    __nv_bfloat16* dst = (is_k ? kc : vc) + blk * blk_stride + ((long long)kvh * BS + off) * D;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int i = lane + 32 * j;
      dst[i] = __float2bfloat16_rn(a[j]);
      dst[i + D / 2] = __float2bfloat16_rn(b[j]);
    }
  }
}

// Full-rotary variant with 16-byte accesses: D/16 threads per (token, head),
// each holding 8 elements of the first half and the matching 8 of the second
// half (the NeoX pairs), so every load and store of the row is one uint4. The
// rotation and normalisation arithmetic is the same fp32 expression as in
// rope_kv_kernel; the q/k-norm sum of squares is reduced over the head's
// D/16 lanes.
__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 x = __bfloat1622float2(h[k]);
    f[2 * k] = x.x;
    f[2 * k + 1] = x.y;
  }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
  return u;
}

template <int D>
__global__ void __launch_bounds__(256) rope_kv_vec_kernel(
    __nv_bfloat16* __restrict__ qkv, const int64_t* __restrict__ pos,
    const float* __restrict__ cos_sin, __nv_bfloat16* __restrict__ kc,
    __nv_bfloat16* __restrict__ vc, const int64_t* __restrict__ slots,
    const __nv_bfloat16* __restrict__ q_norm, const __nv_bfloat16* __restrict__ k_norm, int T,
    int Hq, int Hkv, int BS, float eps, long long blk_stride) {
  constexpr int TPH = D / 16;  // threads per head
  pdl_wait();
  pdl_trigger();
  const int heads = Hq + 2 * Hkv;
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long gh = g / TPH;
  const int sub = (int)(g % TPH);
  // Heads occupy aligned groups of TPH lanes (TPH divides 32).
  if (gh >= (long long)T * heads) return;
  const int t = (int)(gh / heads);
  const int h = (int)(gh % heads);
  const int i0 = sub * 8;
  __nv_bfloat16* hp = qkv + ((size_t)t * heads + h) * D;
  const bool is_q = h < Hq;
  const bool is_k = !is_q && h < Hq + Hkv;
  float a[8], b[8];
  bf16x8_to_f32(*reinterpret_cast<const uint4*>(hp + i0), a);
  bf16x8_to_f32(*reinterpret_cast<const uint4*>(hp + D / 2 + i0), b);
  if (is_q || is_k) {
    const __nv_bfloat16* nw = is_q ? q_norm : k_norm;
    if (nw != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += a[j] * a[j] + b[j] * b[j];
      // The head's lanes: an aligned group of TPH lanes that run (or exit) together.
      const int lane = threadIdx.x & 31;
      const unsigned gmask =
          TPH == 32 ? 0xffffffffu : ((1u << TPH) - 1u) << (lane & ~(TPH - 1));
#pragma unroll
      for (int o = TPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(gmask, ss, o);
      const float inv = rsqrtf(ss / (float)D + eps);
      float wa[8], wb[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(nw + i0), wa);
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(nw + D / 2 + i0), wb);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        a[j] = __bfloat162float(__float2bfloat16_rn(a[j] * inv)) * wa[j];
        b[j] = __bfloat162float(__float2bfloat16_rn(b[j] * inv)) * wb[j];
      }
    }
    const float* cs = cos_sin + (size_t)pos[t] * D;
    const float4 c0 = *reinterpret_cast<const float4*>(cs + i0);
    const float4 c1 = *reinterpret_cast<const float4*>(cs + i0 + 4);
    const float4 s0 = *reinterpret_cast<const float4*>(cs + D / 2 + i0);
    const float4 s1 = *reinterpret_cast<const float4*>(cs + D / 2 + i0 + 4);
    const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x1 = a[j], x2 = b[j];
      a[j] = x1 * c[j] - x2 * sn[j];
      b[j] = x2 * c[j] + x1 * sn[j];
    }
  }
  const uint4 ua = f32_to_bf16x8(a), ub = f32_to_bf16x8(b);
  if (is_q || is_k) {
    *reinterpret_cast<uint4*>(hp + i0) = ua;
    *reinterpret_cast<uint4*>(hp + D / 2 + i0) = ub;
  }
  if (is_q) return;
  const int64_t slot = slots ? slots[t] : -1;
  if (slot < 0) return;
  const int kvh = is_k ? h - Hq : h - Hq - Hkv;
  const int64_t blk = slot / BS, off = slot % BS;
  __nv_bfloat16* dst = (is_k ? kc : vc) + blk * blk_stride + ((long long)kvh * BS + off) * D;
  *reinterpret_cast<uint4*>(dst + i0) = ua;
  *reinterpret_cast<uint4*>(dst + D / 2 + i0) = ub;
}

// Plain K/V scatter into the paged cache (RoPE applied by the caller):
// one thread per 16-byte chunk of one token's K or V head.
__global__ void kv_write_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                                long long ldk, long long ldv, __nv_bfloat16* __restrict__ kc,
                                __nv_bfloat16* __restrict__ vc, const int64_t* __restrict__ slots,
                                int T, int Hkv, int D, int BS, long long blk_stride) {
  pdl_wait();
  pdl_trigger();
  const long long chunks_per_tok = (long long)Hkv * (D / 8);
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)T * chunks_per_tok * 2;
  if (idx >= total) return;
  const bool is_v = idx >= total / 2;
  const long long j = is_v ? idx - total / 2 : idx;
  const int t = (int)(j / chunks_per_tok);
  const int rem = (int)(j % chunks_per_tok);
  const int h = rem / (D / 8), c = rem % (D / 8);
  const int64_t slot = slots[t];
  if (slot < 0) return;
  const __nv_bfloat16* src = (is_v ? v + t * ldv : k + t * ldk) + (long long)h * D + c * 8;
  __nv_bfloat16* dst = (is_v ? vc : kc) + (slot / BS) * blk_stride +
                       ((long long)h * BS + slot % BS) * D + c * 8;
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
}

}  // namespace

void kv_cache_write_launch(const void* k, const void* v, long long ldk, long long ldv,
                           void* k_cache, void* v_cache, const int64_t* slots, int T, int Hkv,
                           int D, int BS, long long blk_stride, cudaStream_t stream) {
  if (T <= 0) return;
  const long long total = (long long)T * Hkv * (D / 8) * 2;
  const int thr = 256;
  launch_pdl(kv_write_kernel, dim3((unsigned)((total + thr - 1) / thr)), dim3(thr), 0, stream,
             nullptr, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, ldk, ldv,
             (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, slots, T, Hkv, D, BS, blk_stride);
}

void rope_kv_write_launch(void* qkv, const int64_t* pos, const float* cos_sin, void* k_cache,
                          void* v_cache, const int64_t* slots, const void* q_norm,
                          const void* k_norm, int T, int Hq, int Hkv, int D, int BS, float eps,
                          int rot_dim, long long blk_stride, cudaStream_t stream) {
  if (blk_stride <= 0) blk_stride = (long long)Hkv * BS * D;
  if (T <= 0) return;
  if (rot_dim == D && (D == 64 || D == 128 || D == 256)) {
    const long long threads = (long long)T * (Hq + 2 * Hkv) * (D / 16);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
#define B200_ROPE_VEC(DD)                                                                       \
  launch_pdl(rope_kv_vec_kernel<DD>, dim3(blocks), dim3(256), 0, stream, nullptr,              \
             (__nv_bfloat16*)qkv, pos, cos_sin, (__nv_bfloat16*)k_cache,                      \
             (__nv_bfloat16*)v_cache, slots, (const __nv_bfloat16*)q_norm,                     \
             (const __nv_bfloat16*)k_norm, T, Hq, Hkv, BS, eps, blk_stride)
    if (D == 128) B200_ROPE_VEC(128);
    else if (D == 256) B200_ROPE_VEC(256);
    else B200_ROPE_VEC(64);
#undef B200_ROPE_VEC
    return;
  }
  const long warps = (long)T * (Hq + 2 * Hkv);
  const int wpb = 8;
  const long blocks = (warps + wpb - 1) / wpb;
#define B200_ROPE(DD)                                                                           \
  launch_pdl(rope_kv_kernel<DD>, dim3((unsigned)blocks), dim3(wpb * 32), 0, stream, nullptr,    \
             (__nv_bfloat16*)qkv, pos, cos_sin, (__nv_bfloat16*)k_cache,                      \
             (__nv_bfloat16*)v_cache, slots, (const __nv_bfloat16*)q_norm,                     \
             (const __nv_bfloat16*)k_norm, T, Hq, Hkv, BS, eps, rot_dim, blk_stride)
  if (D == 128) B200_ROPE(128);
  else if (D == 256) B200_ROPE(256);
  else if (D == 64) B200_ROPE(64);
  else throw std::runtime_error("rope_kv_write: head_dim must be 64, 128 or 256");
#undef B200_ROPE
}

}  // namespace b200
