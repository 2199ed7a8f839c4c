// Standalone weight dequantiser: raw quantised rows -> bf16 [N, K] (prefill
// path: dequantise once, then the bf16 tcgen05 GEMM; the decode path fuses the
// same per-chunk math into the GEMM producer, gemm/dequant.cuh).
//
// Reference parity: fp8_sm70_dequantize_out / awq_sm70_dequantize_out /
// nvfp4 dequant (sm70/csrc/turbomind/ops/tm_fp8_sm70.cu:570,
// tm_awq_sm70.cu:718).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>

#include "gemm/dequant.cuh"

namespace b200 {
namespace {

// One thread per 16-byte output chunk (8 k of one row).
template <int WF>
__global__ void dequant_kernel(const uint8_t* __restrict__ raw, long long ld_raw,
                               __nv_bfloat16* __restrict__ out, int N, int K, const WQParams q) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int chunks_per_row = K / 8;
  if (idx >= (long long)N * chunks_per_row) return;
  const int n = (int)(idx / chunks_per_row);
  const int ck = (int)(idx % chunks_per_row);  // chunk index along k
  const int kb = ck / 8, c = ck % 8;            // 64-wide k-block, chunk within it
  const uint8_t* row = raw + (size_t)n * ld_raw + (size_t)kb * raw_row_bytes(WF);
  const uint4 v = dequant8<WF>(row, c, q, n, kb);
  *reinterpret_cast<uint4*>(out + (size_t)n * K + (size_t)ck * 8) = v;
}

}  // namespace

void dequant_weight_launch(const void* raw, long long ld_raw, void* out, int N, int K, int wf,
                           const WQParams& q, cudaStream_t stream) {
  if (K % 64 != 0) throw std::runtime_error("dequant_weight: K must be a multiple of 64");
  const long long total = (long long)N * (K / 8);
  const int thr = 256;
  const unsigned grid = (unsigned)((total + thr - 1) / thr);
  switch (wf) {
    case kWFp8:
      dequant_kernel<kWFp8><<<grid, thr, 0, stream>>>((const uint8_t*)raw, ld_raw,
                                                      (__nv_bfloat16*)out, N, K, q);
      break;
    case kWAwq:
      dequant_kernel<kWAwq><<<grid, thr, 0, stream>>>((const uint8_t*)raw, ld_raw,
                                                      (__nv_bfloat16*)out, N, K, q);
      break;
    case kWNvfp4:
      dequant_kernel<kWNvfp4><<<grid, thr, 0, stream>>>((const uint8_t*)raw, ld_raw,
                                                        (__nv_bfloat16*)out, N, K, q);
      break;
    default:
      throw std::runtime_error("dequant_weight: unknown format");
  }
}

}  // namespace b200
