// Per-format weight dequantisation shared by the fused dequant-in-producer
// GEMM (gemm_bf16_tc.cu) and the standalone dequantiser (quant/dequant.cu),
// so both produce bit-identical bf16 weights.
//
// Formats (see gemm_api.h): FP8 e4m3 with fp32 128x128 block scales; AWQ
// int4 (low nibble = even k) with per-(row, 128-group) bf16x2 (s, -z*s);
// NVFP4 e2m1 (low nibble = even k) with an e4m3 scale per (row, 16 k).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "common/ptx.cuh"
#include "gemm/gemm_api.h"

namespace b200 {

__device__ __forceinline__ float e2m1_to_float(uint32_t x) {
  // magnitudes {0, 0.5, 1, 1.5, 2, 3, 4, 6}; bit 3 is the sign
  const uint32_t m = x & 7u;
  const float mag = m < 4u ? 0.5f * (float)m : (float)(m == 4u ? 2 : m == 5u ? 3 : m == 6u ? 4 : 6);
  return (x & 8u) ? -mag : mag;
}

__device__ __forceinline__ float e4m3_to_float(uint8_t b) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)b));
  return __low2float(*reinterpret_cast<const __half2*>(&h));
}

// The scale a thread needs for its 8 consecutive k of weight row n in
// k-block kb (64 k) at 16-byte output chunk c: fetched apart from the
// conversion so that a caller can issue every row's scale load before it
// waits for the weight bytes (the loads are independent of the TMA copy).
template <int WF>
struct DqScale {
  using type = float;  // FP8: 128x128 block scale; NVFP4: e4m3 block-16 scale as fp32
};
template <>
struct DqScale<kWAwq> {
  using type = __nv_bfloat162;  // (s, -z*s)
};

template <int WF>
__device__ __forceinline__ typename DqScale<WF>::type dq_scale(const WQParams& q, int n, int kb,
                                                               int c) {
  if constexpr (WF == kWFp8) {
    return q.scales_f32[(size_t)(n >> 7) * q.scale_ld + (kb >> 1)];
  } else if constexpr (WF == kWAwq) {
    return q.scale_zero[(size_t)n * q.scale_ld + (kb >> 1)];
  } else {
    return e4m3_to_float(q.scales_u8[(size_t)n * q.scale_ld + kb * 4 + (c >> 1)]);
  }
}

// Dequantise 8 consecutive k of one weight row into 8 bf16 (one 16 B chunk)
// with the scale from dq_scale.
template <int WF>
__device__ __forceinline__ uint4 dequant8_s(const uint8_t* raw_row, int c,
                                            typename DqScale<WF>::type sc) {
  uint32_t out[4];
  if constexpr (WF == kWFp8) {
    const uint2 v = *reinterpret_cast<const uint2*>(raw_row + c * 8);
    const uint32_t w[2] = {v.x, v.y};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t lo, hi;
      const uint16_t b0 = (uint16_t)(w[h] & 0xffffu), b1 = (uint16_t)(w[h] >> 16);
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"(b0));
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"(b1));
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&lo));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&hi));
      out[2 * h] = pack_bf16x2(f0.x * sc, f0.y * sc);
      out[2 * h + 1] = pack_bf16x2(f1.x * sc, f1.y * sc);
    }
  } else if constexpr (WF == kWAwq) {
    // int4 with a per-(row, 128-group) (scale, -zero*scale) pair: w = q*s + zs.
    const float s_ = __low2float(sc), zs = __high2float(sc);
    const uint32_t v = *reinterpret_cast<const uint32_t*>(raw_row + c * 4);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float a = (float)((v >> (8 * h)) & 0xfu), b = (float)((v >> (8 * h + 4)) & 0xfu);
      out[h] = pack_bf16x2(fmaf(a, s_, zs), fmaf(b, s_, zs));
    }
  } else {  // kWNvfp4: e2m1 pairs (low nibble first) -> exact f16 pairs, then x scale in fp32
    const uint32_t v = *reinterpret_cast<const uint32_t*>(raw_row + c * 4);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      uint32_t hv;
      const uint16_t byte = (uint16_t)((v >> (8 * h)) & 0xffu);
      asm("{\n\t.reg .b8 t;\n\tcvt.u8.u16 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
          : "=r"(hv)
          : "h"(byte));
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hv));
      out[h] = pack_bf16x2(f.x * sc, f.y * sc);
    }
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

template <int WF>
__device__ __forceinline__ uint4 dequant8(const uint8_t* raw_row, int c, const WQParams& q,
                                          int n, int kb) {
  return dequant8_s<WF>(raw_row, c, dq_scale<WF>(q, n, kb, c));
}

}  // namespace b200
