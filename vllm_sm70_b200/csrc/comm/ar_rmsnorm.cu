// Fused tensor-parallel all-reduce + residual add + RMSNorm over NVLink peer
// memory (one process per GPU, symmetric buffers exchanged at start-up).
//
//   stage_r  [T, H] bf16   rank r's partial sums (written by the row-parallel
//                          GEMM directly: the GEMM's output buffer IS the stage)
//   res      [T, H] bf16   residual (identical on every rank), updated in place
//   out_x    [T, H] bf16   normalised output, written on every rank
//
// Two-shot, row-partitioned: rank r owns rows [r*T/W, (r+1)*T/W). For each of
// its rows it loads the W partial rows from the peers' stages (NVLink P2P
// loads, summed in rank order in fp32 -- deterministic and identical on every
// rank), rounds the sum to bf16, adds the residual (bf16 round, as the unfused
// fused_add_rms_norm does), RMS-normalises, and stores the new residual row and
// the normalised row into EVERY rank's res / out_x (P2P stores). Traffic per
// rank: (W-1)/W of the tensor in, (W-1)/W * 2 out.
//
// Synchronisation (epoch flags in each rank's signal pad, .sys scope):
//   start : CTA 0 of rank r release-stores ready[r] = epoch on every peer;
//           every CTA acquire-spins until ready[p] >= epoch for all p.
//   end   : every CTA release-adds 1 to done[r] on every peer after its stores;
//           CTA 0 acquire-spins until done[p] reaches the cumulative CTA count
//           of all launches so far (the grid is rank-uniform), then bumps the
//           local epoch. The kernel therefore ends only after every
//           peer has finished reading this rank's stage and writing its rows
//           here, so the next launch may overwrite the stage and the next
//           kernel on the stream may read res / out_x.
// Every spin is bounded (%globaltimer); on timeout the kernel records
// kErrPeerTimeout in the status word and returns -- it never traps.
//
// Reference parity: the TP2 AR + add + RMSNorm kernel
// (sm70/csrc/custom_ar/tp2_ar_fused_add_rms_norm.cu:67-174: stage -> membar.sys
// flag barrier -> peer read -> fp32 sum -> one rounding -> +residual -> RMSNorm
// -> end-flag barrier). Differences: W in {2,4,8}, two-shot row partition
// instead of every rank reducing every row, release/acquire flags with
// bounded waits, and no extra staging copy.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "common/ptx.cuh"
#include "comm/comm_api.h"
#include "common/launch.h"

namespace b200 {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded acquire-spin until *p >= target (wrap-safe compare).
__device__ __forceinline__ bool wait_geq(const uint32_t* p, uint32_t target, unsigned int* err,
                                         unsigned long long timeout_ns) {
  const unsigned long long t0 = globaltimer();
  uint32_t n = 0;
  while ((int32_t)(ld_acquire_sys(p) - target) < 0) {
    if ((++n & 255u) == 0) {
      if (globaltimer() - t0 > timeout_ns) {
        atomicCAS(err, kErrNone, kErrPeerTimeout);
        return false;
      }
      if (*(volatile unsigned int*)err != kErrNone) return false;
    }
  }
  return true;
}

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
  for (int i = 0; i < 4; ++i) w[i] = pack_bf16x2(f[2 * i], f[2 * i + 1]);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

constexpr int kMaxVec = 4;  // 16-byte vectors per thread kept in registers (H <= 8*4*threads)

template <int W>
__global__ void __launch_bounds__(512) ar_rmsnorm_kernel(ArRmsNormParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ int s_ok;
  const int tid = threadIdx.x;
  uint32_t* ready = p.flags_local;          // [W]
  uint32_t* done = p.flags_local + W;       // [W]
  uint32_t* epoch_p = p.flags_local + 2 * W;
  uint32_t* target_p = p.flags_local + 2 * W + 1;  // cumulative CTAs per peer
  const uint32_t epoch = *(volatile uint32_t*)epoch_p + 1;

  // ---- start barrier: every peer's stage is complete
  if (tid == 0) {
    if (blockIdx.x == 0) {
      __threadfence_system();
#pragma unroll
      for (int q = 0; q < W; ++q) st_release_sys(p.flags_peer[q] + p.rank, epoch);
    }
    int ok = 1;
#pragma unroll
    for (int q = 0; q < W; ++q) ok &= wait_geq(ready + q, epoch, p.err, p.timeout_ns);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;

  const int H = p.H;
  const int nvec = H / 8;
  const int rows_per_rank = (p.T + W - 1) / W;
  const int r0 = p.rank * rows_per_rank;
  const int r1 = min(p.T, r0 + rows_per_rank);
  for (int row = r0 + blockIdx.x; row < r1; row += gridDim.x) {
    float v[kMaxVec][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
      const int i = tid + k * blockDim.x;
      if (i < nvec) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        uint4 parts[W];
#pragma unroll
        for (int q = 0; q < W; ++q)
          parts[q] = __ldcv(reinterpret_cast<const uint4*>(p.stage_peer[q] + (size_t)row * H) + i);
#pragma unroll
        for (int q = 0; q < W; ++q) {  // rank order
          float f[8];
          unpack8(parts[q], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += f[e];
        }
        float res[8];
        unpack8(*(reinterpret_cast<const uint4*>(p.res_local + (size_t)row * H) + i), res);
        // bf16(allreduce) + residual, rounded: matches fused_add_rms_norm(x, res).
        const uint4 xs = pack8(acc);
        unpack8(xs, acc);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += res[e];
        const uint4 rs = pack8(acc);
        unpack8(rs, v[k]);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
#pragma unroll
        for (int q = 0; q < W; ++q)
          *(reinterpret_cast<uint4*>(p.res_peer[q] + (size_t)row * H) + i) = rs;
      }
    }
    // block reduction (fixed order)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    __syncthreads();
    const float inv = rsqrtf(tot / (float)H + p.eps);
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
      const int i = tid + k * blockDim.x;
      if (i < nvec) {
        float wf[8], o[8];
        unpack8(*(reinterpret_cast<const uint4*>(p.w) + i), wf);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          o[e] = __bfloat162float(__float2bfloat16_rn(v[k][e] * inv)) * wf[e];
        const uint4 ov = pack8(o);
#pragma unroll
        for (int q = 0; q < W; ++q)
          *(reinterpret_cast<uint4*>(p.out_peer[q] + (size_t)row * H) + i) = ov;
      }
    }
  }

  // ---- end barrier: all peers finished with our stage / wrote our rows
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
#pragma unroll
    for (int q = 0; q < W; ++q) red_release_sys_add(p.flags_peer[q] + W + p.rank, 1u);
    if (blockIdx.x == 0) {
      const uint32_t target = *(volatile uint32_t*)target_p + gridDim.x;
      bool ok = true;
#pragma unroll
      for (int q = 0; q < W; ++q) ok &= wait_geq(done + q, target, p.err, p.timeout_ns);
      (void)ok;
      *(volatile uint32_t*)target_p = target;
      *(volatile uint32_t*)epoch_p = epoch;
      __threadfence();
    }
  }
}

}  // namespace

void ar_rmsnorm_launch(const ArRmsNormParams& p, int grid, cudaStream_t stream) {
  if (p.H % 8 != 0) throw std::runtime_error("ar_rmsnorm: H % 8 != 0");
  int threads = ((p.H / 8 + kMaxVec - 1) / kMaxVec + 31) / 32 * 32;
  if (threads < 64) threads = 64;
  if (threads > 512) throw std::runtime_error("ar_rmsnorm: H too large");
  switch (p.world) {
    case 2: launch_pdl(ar_rmsnorm_kernel<2>, dim3(grid), dim3(threads), 0, stream, nullptr, p); break;
    case 4: launch_pdl(ar_rmsnorm_kernel<4>, dim3(grid), dim3(threads), 0, stream, nullptr, p); break;
    case 8: launch_pdl(ar_rmsnorm_kernel<8>, dim3(grid), dim3(threads), 0, stream, nullptr, p); break;
    default: throw std::runtime_error("ar_rmsnorm: world size must be 2, 4 or 8");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("ar_rmsnorm: ") + cudaGetErrorString(e));
}

}  // namespace b200
