// Expert-parallel token exchange over NVLink peer memory (one process per
// GPU, symmetric buffers exchanged at start-up): the dispatch and combine of a
// data-parallel-attention MoE block without NCCL.
//
// Per rank, symmetric (peer-written) buffers, T_cap rows per source:
//   recv_x    [W][T_cap][H] bf16      rows other ranks send to this rank
//   recv_meta [W][T_cap][2k] int32    their routing: k expert ids, k weight bits
//   back_y    [W][T_cap][H] bf16      partial outputs this rank's rows got back
//   pad       [kPadWords] uint32      counts and epoch flags (below)
//
// One MoE block, on every rank of the EP group (all ranks run the same
// sequence of blocks -- idle ranks with zero tokens -- so epochs agree):
//   plan      slot[t][d] = rank of token t among this rank's tokens that route
//             to destination d (exclusive scan in token order; -1 = none)
//   dispatch  rows + routing stored into the destinations' recv buffers (P2P
//             stores); the last CTA bumps the local epoch e and release-stores
//             (count, e) into every destination's pad
//   receive   wait (bounded) for every source's flag >= e; compact the
//             received rows in (source, slot) order into local buffers -- the
//             same rows in the same order as the NCCL all-to-all delivers
//   (the local grouped expert GEMMs run on the compacted rows)
//   return    each partial row stored back into its source's back_y (P2P);
//             the last CTA release-stores e into every source's return flag
//   finish    wait (bounded) for every destination's return flag >= e; per
//             token, sum the partial rows over destinations in rank order in
//             fp32, add the shared-expert row, round once to bf16 -- the same
//             arithmetic as the NCCL path, so the two agree bit for bit.
// Buffer reuse is safe without extra barriers: a source writes a
// destination's recv region for block i+1 only after its finish of block i
// saw that destination's return flag, which the destination raises after it
// compacted block i's rows; back_y likewise.
// Every wait is bounded (%globaltimer): on timeout the status word records
// kErrPeerTimeout and the kernel returns. Plain loads / stores only (no
// multicast objects, no TMA on peer memory).
//
// Reference parity: the reference refuses expert parallelism
// (sm70/vllm_sm70/fused_moe/method.py:357-358); the exchange semantics are the
// NCCL all-to-all path of this library (parallel/ep.py), which this replaces.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "comm/ar_rmsnorm_dev.cuh"
#include "comm/comm_api.h"
#include "common/launch.h"
#include "ops_api.h"

namespace b200 {
namespace {

// Pad words: cnt[W] (rows source s sent here, written by s), dflag[W]
// (dispatch epoch of source s), rflag[W] (return epoch of destination d),
// then local words: epoch, arrive (dispatch), arrive (return).
constexpr int kPadCnt = 0, kPadDFlag = kMaxRanks, kPadRFlag = 2 * kMaxRanks,
              kPadEpoch = 3 * kMaxRanks, kPadArriveD = 3 * kMaxRanks + 1,
              kPadArriveR = 3 * kMaxRanks + 2;

// slot[t * W + d]: one CTA per destination, block-wide exclusive scan over tokens.
__global__ void __launch_bounds__(1024) ep_plan_kernel(const EpParams p, const int* __restrict__ ids,
                                                       int T, int* __restrict__ slot,
                                                       int* __restrict__ send_count) {
  pdl_wait();
  __shared__ int warp_sum[32];
  __shared__ int carry;
  const int d = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < T; base += blockDim.x) {
    const int t = base + threadIdx.x;
    int f = 0;
    if (t < T) {
      for (int j = 0; j < p.k; ++j) {
        const int e = ids[(size_t)t * p.k + j];
        if (e >= 0 && e / p.E_local == d) f = 1;
      }
    }
    int incl = f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sum[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      int w = lane < (int)(blockDim.x >> 5) ? warp_sum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += v;
      }
      warp_sum[lane] = w;  // inclusive prefix over warps
    }
    __syncthreads();
    const int before = carry + (wid > 0 ? warp_sum[wid - 1] : 0) + incl - f;
    if (t < T) slot[(size_t)t * p.world + d] = f ? before : -1;
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_sum[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) send_count[d] = carry;
}

// Row + routing of (token, destination) pairs to the destinations' recv buffers.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EpParams p,
                                                          const __nv_bfloat16* __restrict__ x,
                                                          const int* __restrict__ ids,
                                                          const float* __restrict__ w, int T,
                                                          const int* __restrict__ slot,
                                                          const int* __restrict__ send_count) {
  pdl_wait();
  const int W = p.world, H8 = p.H / 8;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * p.H);
    for (int d = 0; d < W; ++d) {
      const int s = slot[(size_t)t * W + d];
      if (s < 0) continue;
      const size_t row = (size_t)p.rank * p.T_cap + s;
      uint4* dst = reinterpret_cast<uint4*>(p.recv_x_peer[d] + row * p.H);
      for (int i = threadIdx.x; i < H8; i += blockDim.x) dst[i] = src[i];
      int* meta = p.recv_meta_peer[d] + row * 2 * p.k;
      if (threadIdx.x < p.k) {
        meta[threadIdx.x] = ids[(size_t)t * p.k + threadIdx.x];
        meta[p.k + threadIdx.x] = __float_as_int(w[(size_t)t * p.k + threadIdx.x]);
      }
    }
  }
  // The last CTA publishes: counts first, then the epoch flag (release).
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t n = atomicAdd(p.pad_local + kPadArriveD, 1u) + 1u;
    last = n == gridDim.x;
    if (last) atomicExch(p.pad_local + kPadArriveD, 0u);
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    const uint32_t e = p.pad_local[kPadEpoch] + 1u;
    p.pad_local[kPadEpoch] = e;
    for (int d = 0; d < W; ++d) {
      volatile uint32_t* c = p.pad_peer[d] + kPadCnt + p.rank;
      *c = (uint32_t)send_count[d];
    }
    __threadfence_system();
    for (int d = 0; d < W; ++d) ardev::st_release_sys(p.pad_peer[d] + kPadDFlag + p.rank, e);
  }
}

// Wait for every source, then compact the received rows (source, slot order).
// out_rows[0] = N (rows received); rows past N up to n_max get ids -1.
__global__ void __launch_bounds__(256) ep_receive_kernel(const EpParams p,
                                                         __nv_bfloat16* __restrict__ xc,
                                                         int* __restrict__ idc,
                                                         float* __restrict__ wc,
                                                         int* __restrict__ row_src,
                                                         int* __restrict__ n_rows, int n_max) {
  pdl_wait();
  __shared__ int off[kMaxRanks + 1];
  __shared__ int ok;
  const int W = p.world;
  if (threadIdx.x == 0) {
    const uint32_t e = p.pad_local[kPadEpoch];
    int good = 1;
    for (int s = 0; s < W; ++s)
      good &= ardev::wait_geq(p.pad_local + kPadDFlag + s, e, p.err, p.timeout_ns) ? 1 : 0;
    off[0] = 0;
    for (int s = 0; s < W; ++s) {
      const int c = good ? (int)((volatile uint32_t*)p.pad_local)[kPadCnt + s] : 0;
      off[s + 1] = off[s] + (c < p.T_cap ? c : p.T_cap);
    }
    ok = good;
    if (blockIdx.x == 0) *n_rows = off[W] < n_max ? off[W] : n_max;
  }
  __syncthreads();
  const int N = off[W] < n_max ? off[W] : n_max;
  const int H8 = p.H / 8;
  for (int i = blockIdx.x; i < n_max; i += gridDim.x) {
    if (i >= N || !ok) {
      if (threadIdx.x < p.k) {
        idc[(size_t)i * p.k + threadIdx.x] = -1;
        wc[(size_t)i * p.k + threadIdx.x] = 0.f;
      }
      if (threadIdx.x == 0) row_src[i] = -1;
      continue;
    }
    int s = 0;
    while (s + 1 < W && i >= off[s + 1]) ++s;
    const size_t row = (size_t)s * p.T_cap + (i - off[s]);
    const uint4* src = reinterpret_cast<const uint4*>(p.recv_x_local + row * p.H);
    uint4* dst = reinterpret_cast<uint4*>(xc + (size_t)i * p.H);
    for (int j = threadIdx.x; j < H8; j += blockDim.x) dst[j] = src[j];
    const int* meta = p.recv_meta_local + row * 2 * p.k;
    if (threadIdx.x < p.k) {
      idc[(size_t)i * p.k + threadIdx.x] = meta[threadIdx.x];
      wc[(size_t)i * p.k + threadIdx.x] = __int_as_float(meta[p.k + threadIdx.x]);
    }
    if (threadIdx.x == 0) row_src[i] = (int)row;
  }
}

// Partial rows back to their sources; the last CTA raises the return flags.
__global__ void __launch_bounds__(256) ep_return_kernel(const EpParams p,
                                                        const __nv_bfloat16* __restrict__ y,
                                                        const int* __restrict__ row_src,
                                                        const int* __restrict__ n_rows) {
  pdl_wait();
  const int N = *n_rows;
  const int H8 = p.H / 8;
  for (int i = blockIdx.x; i < N; i += gridDim.x) {
    const int row = row_src[i];
    const int s = row / p.T_cap, sl = row - s * p.T_cap;
    const uint4* src = reinterpret_cast<const uint4*>(y + (size_t)i * p.H);
    uint4* dst = reinterpret_cast<uint4*>(p.back_y_peer[s] + ((size_t)p.rank * p.T_cap + sl) * p.H);
    for (int j = threadIdx.x; j < H8; j += blockDim.x) dst[j] = src[j];
  }
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t n = atomicAdd(p.pad_local + kPadArriveR, 1u) + 1u;
    last = n == gridDim.x;
    if (last) atomicExch(p.pad_local + kPadArriveR, 0u);
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    const uint32_t e = p.pad_local[kPadEpoch];
    __threadfence_system();
    for (int s = 0; s < p.world; ++s) ardev::st_release_sys(p.pad_peer[s] + kPadRFlag + p.rank, e);
  }
}

// out[t] = bf16( sum over d in rank order of back_y[d][slot[t][d]] + shared[t] ).
__global__ void __launch_bounds__(256) ep_finish_kernel(const EpParams p,
                                                        const int* __restrict__ slot, int T,
                                                        const __nv_bfloat16* __restrict__ shared,
                                                        __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  __shared__ int ok;
  const int W = p.world;
  if (threadIdx.x == 0) {
    const uint32_t e = p.pad_local[kPadEpoch];
    int good = 1;
    for (int d = 0; d < W; ++d)
      good &= ardev::wait_geq(p.pad_local + kPadRFlag + d, e, p.err, p.timeout_ns) ? 1 : 0;
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const int H8 = p.H / 8;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    for (int j = threadIdx.x; j < H8; j += blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int d = 0; d < W; ++d) {
        const int s = slot[(size_t)t * W + d];
        if (s < 0) continue;
        const uint4 v = reinterpret_cast<const uint4*>(
            p.back_y_local + ((size_t)d * p.T_cap + s) * p.H)[j];
        float f[8];
        ardev::unpack8(v, f);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += f[q];
      }
      if (shared != nullptr) {
        float f[8];
        ardev::unpack8(reinterpret_cast<const uint4*>(shared + (size_t)t * p.H)[j], f);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += f[q];
      }
      reinterpret_cast<uint4*>(out + (size_t)t * p.H)[j] = ardev::pack8(acc);
    }
  }
}

int grid_for(long rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long g = rows < 4L * sms ? rows : 4L * sms;
  return g > 0 ? (int)g : 1;
}

void check(const EpParams& p) {
  if (p.world < 2 || p.world > kMaxRanks) throw std::runtime_error("ep_a2a: world must be 2..8");
  if (p.H % 8 != 0) throw std::runtime_error("ep_a2a: H % 8 != 0");
  if (p.k < 1 || p.k > 32) throw std::runtime_error("ep_a2a: top-k must be 1..32");
}

}  // namespace

void ep_dispatch_launch(const EpParams& p, const void* x, const int* ids, const float* w, int T,
                        int* slot, int* send_count, cudaStream_t stream) {
  check(p);
  if (T > p.T_cap) throw std::runtime_error("ep_dispatch: more tokens than the buffer capacity");
  launch_pdl(ep_plan_kernel, dim3(p.world), dim3(1024), 0, stream, nullptr, p, ids, T, slot,
             send_count);
  launch_pdl(ep_dispatch_kernel, dim3(grid_for(T)), dim3(256), 0, stream, nullptr, p,
             reinterpret_cast<const __nv_bfloat16*>(x), ids, w, T, (const int*)slot,
             (const int*)send_count);
}

void ep_receive_launch(const EpParams& p, void* xc, int* idc, float* wc, int* row_src,
                       int* n_rows, int n_max, cudaStream_t stream) {
  check(p);
  launch_pdl(ep_receive_kernel, dim3(grid_for(n_max)), dim3(256), 0, stream, nullptr, p,
             reinterpret_cast<__nv_bfloat16*>(xc), idc, wc, row_src, n_rows, n_max);
}

void ep_return_launch(const EpParams& p, const void* y, const int* row_src, const int* n_rows,
                      int n_max, cudaStream_t stream) {
  check(p);
  launch_pdl(ep_return_kernel, dim3(grid_for(n_max)), dim3(256), 0, stream, nullptr, p,
             reinterpret_cast<const __nv_bfloat16*>(y), row_src, n_rows);
}

void ep_finish_launch(const EpParams& p, const int* slot, int T, const void* shared, void* out,
                      cudaStream_t stream) {
  check(p);
  launch_pdl(ep_finish_kernel, dim3(grid_for(T)), dim3(256), 0, stream, nullptr, p, slot, T,
             reinterpret_cast<const __nv_bfloat16*>(shared), reinterpret_cast<__nv_bfloat16*>(out));
}

}  // namespace b200
