// Small-message tensor-parallel exchanges of the vocab-parallel sampler over
// NVLink peer memory, one kernel per exchange.
//
// Each rank holds the sampler's result for its vocab shard: per row either
// one (value, id) pair (greedy / Gumbel-max sampling) or its top-C candidate
// (value, id) lists (top-k / top-p sampling). Instead of an NCCL all-gather
// followed by a merge kernel, one kernel stores this rank's message straight
// into every rank's symmetric receive buffer, raises an epoch flag on every
// rank, waits for all ranks' flags and then finishes locally:
//   mode kTop1:  ids[row] = the global top-1 over the ranks' pairs in rank
//                order -- NaN values first (lowest id), else the largest
//                value, ties to the lowest id (the same rule as the
//                single-shard argmax kernel, so TP and TP1 pick the same id);
//   mode kGather: out_v / out_i [rows, W * C] = the ranks' candidate lists
//                concatenated in rank order (what an all-gather along the
//                candidate dimension gives).
//
// Protocol (pad words per rank: ready[W], arrive, done, epoch):
//   e = epoch + 1, read after the PDL wait (the previous launch is complete);
//   phase 1: every CTA stores its slice of the message into half (e & 1),
//            slot `rank`, of every rank's receive buffer (4-byte P2P stores);
//   phase 2: fence; the last CTA to arrive re-arms `arrive` and release-stores
//            ready[rank] = e into every rank's pad;
//   phase 3: every CTA acquire-waits (bounded) until ready[q] >= e for all q,
//            then merges / copies out its rows;
//   end:     the last CTA to finish re-arms `done` and bumps the epoch.
// The receive buffer has two halves used by alternate epochs. A rank writes
// half (e + 1) & 1 only after it saw every peer's ready flag for e, which
// each peer raised after its launch e - 1 (the previous reader of that half)
// had completed -- so no end-of-launch barrier is needed. Every wait is
// bounded (%globaltimer); a timeout records kErrPeerTimeout and returns.
//
// Reference parity: the staged P2P top-1 exchange and the candidate gather
// of the vocab-parallel sampler (sm70/csrc/custom_ar/top1_custom_ar.cu:52-101,
// sm70/vllm_sm70/sample.py:308-309).
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "comm/comm_api.h"
#include "common/launch.h"
#include "common/ptx.cuh"
#include "ops_api.h"

namespace b200 {
namespace {

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool wait_ready(const uint32_t* p, uint32_t target, unsigned int* err,
                           unsigned long long timeout_ns) {
  const unsigned long long t0 = globaltimer();
  uint32_t n = 0;
  while ((int32_t)(ld_acquire_sys_u32(p) - target) < 0) {
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

// The ordering of the merge: is (v, id) ahead of (bv, bid)?
__device__ __forceinline__ bool top1_better(float v, int id, float bv, int bid) {
  const bool n = v != v, bn = bv != bv;
  if (n != bn) return n;        // NaN first
  if (n) return id < bid;       // both NaN: lowest id
  if (v != bv) return v > bv;   // largest value
  return id < bid;              // tie: lowest id
}

template <int W>
__global__ void __launch_bounds__(256) tp_exchange_kernel(TpExchangeParams p) {
  pdl_wait();
  uint32_t* pad = p.pad_local;
  constexpr int kReady = 0, kArrive = W, kDone = W + 1, kEpoch = W + 2;
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_epoch = *(volatile uint32_t*)(pad + kEpoch) + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;
  const long long half = (long long)(e & 1u) * W * p.cap;
  const long long slot = half + (long long)p.rank * p.cap;
  // Phase 1: this rank's message (src0 then src1, 4-byte words) into every rank.
  const long long w0 = p.n0 / 4, w1 = p.n1 / 4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const uint32_t* s0 = reinterpret_cast<const uint32_t*>(p.src0);
  const uint32_t* s1 = reinterpret_cast<const uint32_t*>(p.src1);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < w0 + w1; i += stride) {
    const uint32_t v = i < w0 ? __ldg(s0 + i) : __ldg(s1 + (i - w0));
#pragma unroll
    for (int q = 0; q < W; ++q)
      reinterpret_cast<uint32_t*>(p.recv_peer[q] + slot)[i] = v;
  }
  // Phase 2: the last CTA publishes this rank's ready flag on every rank.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t n = atomicAdd(pad + kArrive, 1u) + 1u;
    if (n == gridDim.x) {
      atomicExch(pad + kArrive, 0u);
      __threadfence_system();
#pragma unroll
      for (int q = 0; q < W; ++q) st_release_sys_u32(p.pad_peer[q] + kReady + p.rank, e);
    }
    int ok = 1;
#pragma unroll
    for (int q = 0; q < W; ++q)
      ok &= wait_ready(pad + kReady + q, e, p.err, p.timeout_ns) ? 1 : 0;
    s_ok = ok;
  }
  __syncthreads();
  pdl_trigger();
  if (s_ok) {
    // Phase 3: finish locally from this rank's receive buffer.
    const uint8_t* rb = p.recv_local + half;
    if (p.mode == kTpXchgTop1) {
      for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < p.rows; r += (int)stride) {
        float bv = 0.f;
        int bid = 0x7fffffff;
        bool have = false;
#pragma unroll
        for (int q = 0; q < W; ++q) {
          const float* vq = reinterpret_cast<const float*>(rb + (long long)q * p.cap);
          const int* iq = reinterpret_cast<const int*>(rb + (long long)q * p.cap + p.n0);
          const float v = vq[r];
          const int id = iq[r];
          if (!have || top1_better(v, id, bv, bid)) {
            bv = v;
            bid = id;
            have = true;
          }
        }
        p.out_ids[r] = bid;
      }
    } else {
      const long long per_rank = (long long)p.rows * p.C;
      const long long total = per_rank * W;
      for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < total;
           j += stride) {
        const long long r = j / ((long long)W * p.C);
        const int rem = (int)(j - r * W * p.C);
        const int q = rem / p.C, c = rem - q * p.C;
        const uint8_t* base = rb + (long long)q * p.cap;
        p.out_v[j] = reinterpret_cast<const float*>(base)[r * p.C + c];
        p.out_i[j] = reinterpret_cast<const int*>(base + p.n0)[r * p.C + c];
      }
    }
  }
  // End: the last CTA to finish bumps the epoch for the next launch.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t n = atomicAdd(pad + kDone, 1u) + 1u;
    if (n == gridDim.x) {
      atomicExch(pad + kDone, 0u);
      atomicExch(pad + kEpoch, e);
    }
  }
}

}  // namespace

void tp_exchange_launch(const TpExchangeParams& p, cudaStream_t stream) {
  if (p.n0 % 4 || p.n1 % 4) throw std::runtime_error("tp_exchange: message parts must be 4-byte words");
  if (p.n0 + p.n1 > p.cap) throw std::runtime_error("tp_exchange: message exceeds the slot");
  const long long words = (p.n0 + p.n1) / 4;
  const long long out_items = p.mode == kTpXchgTop1 ? p.rows : (long long)p.rows * p.C * p.world;
  long long need = words > out_items ? words : out_items;
  int grid = (int)((need + 255) / 256);
  if (grid < 1) grid = 1;
  if (grid > 32) grid = 32;
  switch (p.world) {
    case 2: launch_pdl(tp_exchange_kernel<2>, dim3(grid), dim3(256), 0, stream, nullptr, p); break;
    case 4: launch_pdl(tp_exchange_kernel<4>, dim3(grid), dim3(256), 0, stream, nullptr, p); break;
    case 8: launch_pdl(tp_exchange_kernel<8>, dim3(grid), dim3(256), 0, stream, nullptr, p); break;
    default: throw std::runtime_error("tp_exchange: world size must be 2, 4 or 8");
  }
}

}  // namespace b200
