// Device side of the fused tensor-parallel all-reduce + residual add +
// RMSNorm, shared by the standalone collective kernel (ar_rmsnorm.cu) and
// the row-parallel GEMM that runs it as its last phase (gemm_bf16_tc.cu,
// epilogue kEpiArNorm).
//
// Protocol (signal pad of each rank, uint32 words): ready[W], done[W],
// epoch, done_target, arrive.
//   start : the rank's stage is complete -> release-store ready[rank] = epoch
//           on every peer; every CTA acquire-spins until ready[p] >= epoch.
//           Standalone kernel: CTA 0 publishes at once (the stage was written
//           by an earlier kernel). GEMM phase: every CTA adds 1 to `arrive`
//           after its tiles are stored; the last one publishes.
//   rows  : rank r owns rows [r*T/W, (r+1)*T/W); per row: the W partial rows
//           from the peers' stages (NVLink loads) summed in rank order in
//           fp32, one bf16 round, + residual (bf16 round), RMSNorm (sum of
//           squares in the block-size-independent order of rowsum.cuh), and the
//           new residual / normalised rows stored into EVERY rank's buffers.
//           NVLS variant (multicast addresses given): the switch sums the W
//           partials (fp32 accumulation in the switch, order unspecified, one
//           bf16 result) and one multimem.st writes every rank's copy.
//   end   : every CTA release-adds 1 to done[rank] on every peer; CTA 0 waits
//           until done[p] reaches the cumulative CTA count of all launches
//           (rank-uniform grids), then bumps the epoch -- so no rank reuses
//           its stage while a peer still reads it.
// Every spin is bounded (%globaltimer); a timeout records kErrPeerTimeout in
// the status word and the CTA returns. Nothing traps.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "comm/comm_api.h"
#include "common/ptx.cuh"
#include "common/rowsum.cuh"
#include "ops_api.h"

namespace b200 {
namespace ardev {

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

// NVLS (NVLink SHARP) accesses through a multicast address: the switch sums
// the 16 bytes of every rank's copy (fp32 accumulation, bf16 result), or
// writes 16 bytes to every rank's copy.
__device__ __forceinline__ uint4 multimem_ld_add_bf16x8(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}
__device__ __forceinline__ void multimem_st_16(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
// Orders this thread's accesses through the unicast and multicast aliases of
// the same memory.
__device__ __forceinline__ void fence_proxy_alias() {
  asm volatile("fence.proxy.alias;" ::: "memory");
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

constexpr int kMaxVec = 4;  // 16-byte vectors per thread held in registers (H <= 32 * threads)

// Pad word indices.
template <int W> struct Pad {
  static constexpr int kReady = 0, kDone = W, kEpoch = 2 * W, kTarget = 2 * W + 1,
                       kArrive = 2 * W + 2;
};

// Start barrier. `gated`: publish only once every CTA of the grid has
// arrived (the stage is written by this grid). Returns false on timeout.
template <int W>
__device__ bool start_barrier(const ArRmsNormParams& p, uint32_t epoch, bool gated, int* s_ok) {
  uint32_t* pad = p.flags_local;
  if (threadIdx.x == 0) {
    bool publish = !gated && blockIdx.x == 0;
    if (gated) {
      __threadfence_system();  // this CTA's stage stores, visible system-wide
      const uint32_t n = atomicAdd(pad + Pad<W>::kArrive, 1u) + 1u;
      if (n == gridDim.x) {
        atomicExch(pad + Pad<W>::kArrive, 0u);  // re-arm for the next launch
        publish = true;
      }
    }
    if (publish) {
      __threadfence_system();
#pragma unroll
      for (int q = 0; q < W; ++q) st_release_sys(p.flags_peer[q] + Pad<W>::kReady + p.rank, epoch);
    }
    int ok = 1;
#pragma unroll
    for (int q = 0; q < W; ++q)
      ok &= wait_geq(pad + Pad<W>::kReady + q, epoch, p.err, p.timeout_ns) ? 1 : 0;
    *s_ok = ok;
  }
  __syncthreads();
  if (p.mc_stage != nullptr) fence_proxy_alias();  // stages were written through unicast
  return *s_ok != 0;
}

// The rows this rank owns, CTA-strided; every thread of the CTA takes part.
template <int W>
__device__ void rows_phase(const ArRmsNormParams& p, float* part, float* bcast) {
  const int tid = threadIdx.x;
  const int H = p.H;
  const int nvec = H / 8;
  const int rows_per_rank = (p.T + W - 1) / W;
  const int r0 = p.rank * rows_per_rank;
  const int r1 = min(p.T, r0 + rows_per_rank);
  for (int row = r0 + blockIdx.x; row < r1; row += gridDim.x) {
    float v[kMaxVec][8];
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
      const int i = tid + k * blockDim.x;
      if (i < nvec) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (p.mc_stage != nullptr) {
          // In-switch sum of every rank's partial (bf16 result of an fp32 sum).
          unpack8(multimem_ld_add_bf16x8(reinterpret_cast<const uint4*>(
                      p.mc_stage + (size_t)row * H) + i), acc);
        } else {
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
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
        part[i] = ss;
        if (p.mc_res != nullptr) {
          multimem_st_16(reinterpret_cast<uint4*>(p.mc_res + (size_t)row * H) + i, rs);
        } else {
#pragma unroll
          for (int q = 0; q < W; ++q)
            *(reinterpret_cast<uint4*>(p.res_peer[q] + (size_t)row * H) + i) = rs;
        }
      }
    }
    // Row sum of squares in the block-size-independent order.
    const float tot = canonical_block_sum(part, nvec, bcast);
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
        if (p.mc_out != nullptr) {
          multimem_st_16(reinterpret_cast<uint4*>(p.mc_out + (size_t)row * H) + i, ov);
        } else {
#pragma unroll
          for (int q = 0; q < W; ++q)
            *(reinterpret_cast<uint4*>(p.out_peer[q] + (size_t)row * H) + i) = ov;
        }
      }
    }
  }
}

template <int W>
__device__ void end_barrier(const ArRmsNormParams& p, uint32_t epoch) {
  uint32_t* pad = p.flags_local;
  if (p.mc_out != nullptr) fence_proxy_alias();  // multicast stores before the release below
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
#pragma unroll
    for (int q = 0; q < W; ++q) red_release_sys_add(p.flags_peer[q] + Pad<W>::kDone + p.rank, 1u);
    if (blockIdx.x == 0) {
      const uint32_t target = *(volatile uint32_t*)(pad + Pad<W>::kTarget) + gridDim.x;
      bool ok = true;
#pragma unroll
      for (int q = 0; q < W; ++q)
        ok &= wait_geq(pad + Pad<W>::kDone + q, target, p.err, p.timeout_ns);
      (void)ok;
      *(volatile uint32_t*)(pad + Pad<W>::kTarget) = target;
      *(volatile uint32_t*)(pad + Pad<W>::kEpoch) = epoch;
      __threadfence();
    }
  }
}

// Whole collective for W ranks. `gated`: see start_barrier.
// `part`: shared scratch of at least kMaxVec * blockDim.x floats.
template <int W>
__device__ void run(const ArRmsNormParams& p, bool gated, float* part, float* bcast, int* s_ok) {
  const uint32_t epoch = *(volatile uint32_t*)(p.flags_local + Pad<W>::kEpoch) + 1;
  if (!start_barrier<W>(p, epoch, gated, s_ok)) return;
  rows_phase<W>(p, part, bcast);
  end_barrier<W>(p, epoch);
}

// Runtime world size -> instantiation.
__device__ __forceinline__ void run_any(const ArRmsNormParams& p, bool gated, float* part,
                                        float* bcast, int* s_ok) {
  switch (p.world) {
    case 1: run<1>(p, gated, part, bcast, s_ok); break;  // residual add + RMSNorm after a GEMM (TP1)
    case 2: run<2>(p, gated, part, bcast, s_ok); break;
    case 4: run<4>(p, gated, part, bcast, s_ok); break;
    case 8: run<8>(p, gated, part, bcast, s_ok); break;
    default: break;
  }
}

}  // namespace ardev
}  // namespace b200
