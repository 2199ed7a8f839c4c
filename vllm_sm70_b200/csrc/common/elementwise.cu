// Small memory-bound kernels: SiLU(gate) * up, embedding gather.
//
// Reference parity: sm70_silu_and_mul{,_interleaved}_fp16_kernel
// (sm70/csrc/turbomind/ops/tm_ops_common_sm70.cuh:50-110). The GEMM epilogue
// (gemm/gemm_bf16_tc.cu, kEpiSiluMul) fuses this op on the main path; this
// standalone kernel serves layouts the epilogue does not cover.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>

#include "ops_api.h"
#include "common/launch.h"

namespace b200 {
namespace {

// x [T, 2I] = [gate | up] (block = 0), or gate/up interleaved in blocks of
// `block` columns ([g0..g_b-1, u0..u_b-1, g_b.., ...], the layout of the
// fused-epilogue gate_up weights); out [T, I]
__global__ void silu_mul_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
                                int I, int ld_x, int ld_o, int block, const int* __restrict__ n_rows) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;  // rows on x: grid.y is limited to 65535
  if (n_rows != nullptr && t >= *n_rows) return;  // rows past the device-side count
  const int i8 = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (i8 >= I) return;
  const __nv_bfloat16* g =
      x + (size_t)t * ld_x + (block > 0 ? (i8 / block) * 2 * block + i8 % block : i8);
  const __nv_bfloat16* u = g + (block > 0 ? block : I);
  const uint4 gv = *reinterpret_cast<const uint4*>(g);
  const uint4 uv = *reinterpret_cast<const uint4*>(u);
  const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
  const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
  uint32_t ow[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float g0 = __uint_as_float(gw[k] << 16), g1 = __uint_as_float(gw[k] & 0xffff0000u);
    const float u0 = __uint_as_float(uw[k] << 16), u1 = __uint_as_float(uw[k] & 0xffff0000u);
    const float o0 = __fdividef(g0, 1.f + __expf(-g0)) * u0;
    const float o1 = __fdividef(g1, 1.f + __expf(-g1)) * u1;
    __nv_bfloat162 h = __floats2bfloat162_rn(o0, o1);
    ow[k] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(out + (size_t)t * ld_o + i8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

__global__ void embedding_kernel(__nv_bfloat16* __restrict__ out, const int64_t* __restrict__ ids,
                                 const __nv_bfloat16* __restrict__ table, int H, int64_t vocab_start,
                                 int64_t vocab_end) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int64_t id = ids[t];
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H);
  const bool in = id >= vocab_start && id < vocab_end;
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)(in ? id - vocab_start : 0) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = in ? src[i] : make_uint4(0, 0, 0, 0);
}

}  // namespace

void silu_mul_launch(void* out, const void* x, int T, int I, int ld_x, int ld_o,
                     cudaStream_t stream, int block, const int* n_rows) {
  if (T <= 0) return;
  if (I % 8) throw std::runtime_error("silu_mul: I % 8 != 0");
  if (block < 0 || block % 8 || (block > 0 && I % block))
    throw std::runtime_error("silu_mul: interleave block must be a multiple of 8 dividing I");
  dim3 grid(T, (I / 8 + 127) / 128);
  launch_pdl(silu_mul_kernel, grid, dim3(128), 0, stream, nullptr, (__nv_bfloat16*)out,
             (const __nv_bfloat16*)x, I, ld_x, ld_o, block, n_rows);
}

void embedding_launch(void* out, const int64_t* ids, const void* table, int T, int H,
                      int64_t vocab_start, int64_t vocab_end, cudaStream_t stream) {
  if (T <= 0) return;
  if (H % 8) throw std::runtime_error("embedding: H % 8 != 0");
  launch_pdl(embedding_kernel, dim3(T), dim3(256), 0, stream, nullptr, (__nv_bfloat16*)out, ids,
             (const __nv_bfloat16*)table, H, vocab_start, vocab_end);
}

}  // namespace b200
