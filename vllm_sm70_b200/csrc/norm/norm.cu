// RMSNorm and fused residual-add + RMSNorm, one CTA per row, 16-byte vectors.
//
// fused_add_rms_norm: s = bf16(x + residual) ; residual <- s ;
//                     x <- bf16(s * rsqrt(mean(s^2) + eps) * w)
// The variance is taken from the rounded bf16 sum, reduced in a block-size-
// independent order (common/rowsum.cuh), so the fused collective variants
// (comm/ar_rmsnorm.cu, and the GEMM that runs it as its last phase) that
// perform the same rounding match this kernel bit for bit.
//
// Reference parity: upstream vLLM fused_add_rms_norm as pinned by the reference
// (sm70/vllm_sm70/_cuda_platform.py:276-302) and the TP2 AR+RMSNorm kernel's
// epilogue (sm70/csrc/custom_ar/tp2_ar_fused_add_rms_norm.cu:67-174).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "ops_api.h"
#include "common/launch.h"
#include "common/rowsum.cuh"

namespace b200 {
namespace {

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

constexpr int kMaxVec = 4;  // up to 4 x 8 elements per thread kept in registers

template <bool ADD>
__global__ void rms_norm_kernel(__nv_bfloat16* __restrict__ out, int ld_out,
                                __nv_bfloat16* __restrict__ x, int ld_x,
                                __nv_bfloat16* __restrict__ residual, int ld_r,
                                const __nv_bfloat16* __restrict__ w, int H, float eps) {
  pdl_wait();
  pdl_trigger();
  __shared__ float part[kMaxVec * 1024];  // one partial per 8-element vector
  __shared__ float bcast;
  const int row = blockIdx.x;
  const int nvec = H / 8;
  uint4* xr = reinterpret_cast<uint4*>(x + (size_t)row * ld_x);
  uint4* rr = ADD ? reinterpret_cast<uint4*>(residual + (size_t)row * ld_r) : nullptr;
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * ld_out);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  float v[kMaxVec][8];
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      unpack8(xr[i], v[k]);
      if (ADD) {
        float r[8];
        unpack8(rr[i], r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k][e] += r[e];
        const uint4 s = pack8(v[k]);
        rr[i] = s;
        unpack8(s, v[k]);  // continue with the rounded sum
      }
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
      part[i] = ss;
    }
  }
  const float tot = canonical_block_sum(part, nvec, &bcast);
  const float inv = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float wf[8];
      unpack8(wr[i], wf);
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        // Round the normalised value to bf16 before the weight multiply
        // (same order as the HF / vLLM reference implementations).
        const float n = __bfloat162float(__float2bfloat16_rn(v[k][e] * inv));
        o[e] = n * wf[e];
      }
      orow[i] = pack8(o);
    }
  }
}

int norm_threads(int H) {
  const int nvec = H / 8;
  int t = (nvec + kMaxVec - 1) / kMaxVec;
  t = ((t + 31) / 32) * 32;
  if (t < 32) t = 32;
  if (t > 1024) throw std::runtime_error("rms_norm: hidden size too large");
  return t;
}

}  // namespace

void rms_norm_launch(void* out, int ld_out, const void* x, int ld_x, const void* w, int rows,
                     int H, float eps, cudaStream_t stream) {
  if (H % 8) throw std::runtime_error("rms_norm: H % 8 != 0");
  if (rows <= 0) return;
  launch_pdl(rms_norm_kernel<false>, dim3(rows), dim3(norm_threads(H)), 0, stream, nullptr,
             (__nv_bfloat16*)out, ld_out, (__nv_bfloat16*)x, ld_x, (__nv_bfloat16*)nullptr, 0,
             (const __nv_bfloat16*)w, H, eps);
}

void fused_add_rms_norm_launch(void* x, int ld_x, void* residual, int ld_r, const void* w,
                               int rows, int H, float eps, cudaStream_t stream) {
  if (H % 8) throw std::runtime_error("fused_add_rms_norm: H % 8 != 0");
  if (rows <= 0) return;
  launch_pdl(rms_norm_kernel<true>, dim3(rows), dim3(norm_threads(H)), 0, stream, nullptr,
             (__nv_bfloat16*)x, ld_x, (__nv_bfloat16*)x, ld_x, (__nv_bfloat16*)residual, ld_r,
             (const __nv_bfloat16*)w, H, eps);
}

}  // namespace b200
