// Block-scaled FP8 GEMM on the 5th-generation tensor cores (tcgen05.mma
// kind::f8f6f4, e4m3 x e4m3 -> fp32), with exact fp32 scale promotion.
//
//   C[m, n] = sum_kb sa[kb][m] * sw[n / 128][kb] * sum_{k in block kb} Aq[m, k] * Wq[n, k]
//
// A (activations): e4m3 [M, K], quantised per token and 128-wide K group, fp32
// scales stored K-group major, sa[K/128][ld_sa] (quant_fp8_act_launch writes
// both). W: e4m3 [N, K] with one fp32 scale per 128 x 128 block,
// sw[N/128][ld_sw] (the block-FP8 checkpoint layout, "weight_scale_inv").
//
// Promotion: every 128-wide K block is accumulated by its own 4 MMAs (K = 32
// each) into one of 4 rotating TMEM buffers; the epilogue warps read the
// block's partial sums with tcgen05.ld and fold them into fp32 register
// accumulators times the product of the two scales, then hand the buffer back
// to the MMA issuer. The scales are applied in fp32 exactly as the block
// format defines them (no power-of-two rounding of the scales, as the
// hardware block-scaled kind::mxf8f6f4 would need), and the MMA issuer runs
// up to 4 K blocks ahead of the promotion.
//
// Modes: normal (P = A rows, Q = W rows; large M) and swap-AB (P = W rows,
// Q = A rows; small M, and the grouped MoE form whose tiles walk experts).
// Warp roles (320 threads, one CTA per SM, persistent over tiles):
//   warp 0       TMA producer: 128 x 128 B P tiles and BN x 128 B Q tiles,
//                128-byte swizzle, STAGES-deep ring
//   warp 1       TMEM allocator + single-thread MMA issuer
//   warps 2..9   scale staging (cp.async, double-buffered chunks of 16 K
//                blocks), promotion of BN/2 columns each (two warps per TMEM
//                lane quadrant), bf16 store
// All waits are bounded; on a timeout every role leaves its loop, outstanding
// MMAs and copies are drained and TMEM is freed before the CTA exits.
//
// Reference parity: the reference runs block-FP8 checkpoints weight-only on
// Volta (sm70/csrc/turbomind/ops/tm_fp8_sm70.cu:566-600, dequantise to f16 in
// the GEMM's operand load); the block-scale semantics (128 x 128 weight
// blocks, fp32 scale_inv) are the checkpoint format and are kept.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "common/launch.h"
#include "common/ptx.cuh"
#include "common/tmap.h"
#include "gemm/gemm_api.h"

namespace b200 {
namespace {

constexpr int kF8BM = 128;
constexpr int kF8BK = 128;      // e4m3 elements (= bytes) per K block: one 128-byte swizzle row
constexpr int kF8UmmaK = 32;    // K per kind::f8f6f4 MMA
constexpr int kF8Bufs = 4;      // rotating TMEM partial buffers
constexpr int kF8Chunk = 16;    // K blocks per staged scale chunk
constexpr int kF8Threads = 320;
constexpr int kF8EpiThreads = 256;

template <int BN, int STAGES>
struct F8Smem {
  static constexpr int kPBytes = kF8BM * kF8BK;
  static constexpr int kQBytes = BN * kF8BK;
  static constexpr int kStageBytes = kPBytes + kQBytes;
  static constexpr int kTileBytes = STAGES * kStageBytes;
  // Scale staging: vector [2][chunk][128] (per token) + tile scalar [2][chunk].
  static constexpr int kVecBytes = 2 * kF8Chunk * 128 * 4;
  static constexpr int kScalBytes = 2 * kF8Chunk * 4;
  static constexpr int kBarBytes = 256;
  static constexpr int kTotal = kTileBytes + kVecBytes + kScalBytes + kBarBytes + 1024;
};

struct F8Args {
  const float* sa;      // [num_kb][ld_sa] activation scales
  const float* sw;      // [rows / 128][ld_sw] weight block scales
  int ld_sa, ld_sw;
  int M;                // activation rows (tokens) = valid range of sa's vector index
};

__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_le1() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Tile -> operand rows and output bounds (same conventions as the bf16 kernel).
struct F8Unit {
  int p_row, q_row;   // TMA row coordinates of P / Q
  int out_i0;         // output index base along P
  int q_lim;          // exclusive bound of valid Q rows of this tile
  int p_lim;          // exclusive bound of valid output indices along P
};

template <int BN>
__device__ __forceinline__ F8Unit f8_unit(int t, int num_n, const GroupInfo& g, int p_rows,
                                          int q_rows) {
  F8Unit u;
  if (g.E > 0) {
    int lo = 0, hi = g.E;  // largest e with tile_off[e] <= t
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(g.tile_off + mid) <= t) lo = mid; else hi = mid;
    }
    const int e = lo;
    const int local = t - __ldg(g.tile_off + e);
    const int nbs = g.N / kF8BM;
    const int nb = local % nbs, qb = local / nbs;
    u.p_row = e * g.N + nb * kF8BM;
    u.q_row = __ldg(g.row_off + e) + qb * BN;
    u.out_i0 = nb * kF8BM;
    u.q_lim = __ldg(g.row_off + e + 1);
    u.p_lim = g.N;
    return u;
  }
  // Consecutive tiles share the P block (the Q blocks of one P block run
  // together, so the P tile stays hot in L2).
  const int pb = t / num_n, qb = t - pb * num_n;
  u.p_row = pb * kF8BM;
  u.q_row = qb * BN;
  u.out_i0 = pb * kF8BM;
  u.q_lim = q_rows;
  u.p_lim = p_rows;
  return u;
}

template <int BN, int STAGES, bool SWAP>
__global__ void __launch_bounds__(kF8Threads, 1)
gemm_fp8_tc_kernel(const __grid_constant__ CUtensorMap tmap_p,
                   const __grid_constant__ CUtensorMap tmap_q, __nv_bfloat16* __restrict__ C,
                   int ldc, int p_rows, int q_rows, int K, const F8Args fa, const GroupInfo grp,
                   unsigned int* err) {
  static_assert(BN >= 32 && BN <= 128 && BN % 32 == 0, "tile width");
  constexpr int EW = BN / 2;  // columns promoted per epilogue warp
  using S = F8Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  float* vbuf = reinterpret_cast<float*>(smem + S::kTileBytes);                 // [2][CH][128]
  float* tbuf = reinterpret_cast<float*>(smem + S::kTileBytes + S::kVecBytes);  // [2][CH]
  uint64_t* full_bar =
      reinterpret_cast<uint64_t*>(smem + S::kTileBytes + S::kVecBytes + S::kScalBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;    // [kF8Bufs]
  uint64_t* tempty_bar = tfull_bar + kF8Bufs;  // [kF8Bufs]
  uint64_t* done_bar = tempty_bar + kF8Bufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_n = (q_rows + BN - 1) / BN;
  const int num_p = (p_rows + kF8BM - 1) / kF8BM;
  const int num_kb = (K + kF8BK - 1) / kF8BK;
  constexpr uint32_t kCols = kF8Bufs * BN;
  constexpr uint32_t kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128
                                 : kCols <= 256 ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < kF8Bufs; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], kF8EpiThreads / 32);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_p);
    tma_prefetch_desc(&tmap_q);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Tile lists, scales and activations come from earlier kernels.
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const int num_units = grp.E > 0 ? __ldg(grp.tile_off + grp.E) : num_p * num_n;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x) {
        const F8Unit uc = f8_unit<BN>(u, num_n, grp, p_rows, q_rows);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* sp = smem + stage * S::kStageBytes;
          mbar_arrive_expect_tx(&full_bar[stage], (uint32_t)S::kStageBytes);
          tma_load_2d(sp, &tmap_p, &full_bar[stage], kb * kF8BK, uc.p_row);
          tma_load_2d(sp + S::kPBytes, &tmap_q, &full_bar[stage], kb * kF8BK, uc.q_row);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain the copies still in flight (bounded).
      const long n_drain = issued < STAGES ? issued : STAGES;
      for (long j = 0; j < n_drain; ++j) {
        const long it = issued - 1 - j;
        mbar_wait(&full_bar[it % STAGES], (uint32_t)((it / STAGES) & 1), err);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_e4m3(kF8BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      long g = 0;  // global K-block counter: TMEM buffer g % 4
      for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x) {
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int b = (int)(g % kF8Bufs);
          const uint32_t bphase = (uint32_t)((g / kF8Bufs) & 1);
          if (!mbar_wait(&tempty_bar[b], bphase ^ 1u, err) ||
              !mbar_wait(&full_bar[stage], phase, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t spa = smem_u32(smem + stage * S::kStageBytes);
          const uint64_t adesc = umma_desc_sw128(spa);
          const uint64_t bdesc = umma_desc_sw128(spa + S::kPBytes);
          const uint32_t d = tmem_base + (uint32_t)(b * BN);
#pragma unroll
          for (int k = 0; k < kF8BK / kF8UmmaK; ++k)  // +32 bytes per K = 32 step
            umma_f8(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                    k > 0 ? 1u : 0u);
          umma_commit(&empty_bar[stage]);
          umma_commit(&tfull_bar[b]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ promotion / epilogue
    const int et = threadIdx.x - 64;   // 0..255
    const int q = warp & 3;            // TMEM lane quadrant
    const int half = (warp - 2) >> 2;  // column half of the tile
    const int row = q * 32 + lane;     // P row within the tile
    const uint32_t vbase = smem_u32(vbuf);
    const uint32_t tbase = smem_u32(tbuf);
    const int n_chunks = (num_kb + kF8Chunk - 1) / kF8Chunk;
    // Stage the scales of (unit u, chunk c) into buffer `buf`: the per-token
    // vector (P rows in normal mode, Q rows in swap mode) and the tile scalar.
    auto stage_scales = [&](int u, int c, int buf) {
      const F8Unit uc = f8_unit<BN>(u, num_n, grp, p_rows, q_rows);
      const int v0 = SWAP ? uc.q_row : uc.p_row;    // first token of the vector
      const int wrow = SWAP ? uc.p_row : uc.q_row;  // first weight row of the tile
      const float* tsrc = fa.sw + (size_t)(wrow / kF8BM) * fa.ld_sw;
      for (int idx = et; idx < kF8Chunk * 128; idx += kF8EpiThreads) {
        const int kk = idx >> 7, v = idx & 127;
        const int kb = c * kF8Chunk + kk;
        const bool ok = kb < num_kb && v0 + v < fa.M && v < (SWAP ? BN : kF8BM);
        const float* src = ok ? fa.sa + (size_t)kb * fa.ld_sa + (v0 + v) : fa.sa;
        cp_async_4(vbase + (uint32_t)(((buf * kF8Chunk + kk) * 128 + v) * 4), src, ok);
      }
      if (et < kF8Chunk) {
        const int kb = c * kF8Chunk + et;
        const bool ok = kb < num_kb;
        cp_async_4(tbase + (uint32_t)((buf * kF8Chunk + et) * 4), ok ? tsrc + kb : fa.sw, ok);
      }
    };
    long g = 0;    // global K-block counter (TMEM buffer rotation)
    long seq = 0;  // global scale-chunk counter (staging buffer rotation)
    if ((int)blockIdx.x < num_units) stage_scales(blockIdx.x, 0, 0);
    cp_async_commit();
    for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x) {
      const F8Unit uc = f8_unit<BN>(u, num_n, grp, p_rows, q_rows);
      float acc[EW];
#pragma unroll
      for (int c = 0; c < EW; ++c) acc[c] = 0.f;
      bool ok = true;
      for (int c = 0; c < n_chunks && ok; ++c, ++seq) {
        // Prefetch the next chunk (this unit's next, or the next unit's first).
        const int nu = c + 1 < n_chunks ? u : u + (int)gridDim.x;
        const int nc = c + 1 < n_chunks ? c + 1 : 0;
        if (nu < num_units) stage_scales(nu, nc, (int)((seq + 1) & 1));
        cp_async_commit();
        cp_async_wait_le1();
        named_barrier_sync(1, kF8EpiThreads);
        const int buf = (int)(seq & 1);
        const float* vb = vbuf + buf * kF8Chunk * 128;
        const float* tb = tbuf + buf * kF8Chunk;
        const int kb_end = min(num_kb, (c + 1) * kF8Chunk);
        for (int kb = c * kF8Chunk; kb < kb_end; ++kb, ++g) {
          const int b = (int)(g % kF8Bufs);
          if (!mbar_wait(&tfull_bar[b], (uint32_t)((g / kF8Bufs) & 1), err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int kk = kb - c * kF8Chunk;
          const float ts = tb[kk];
          const uint32_t taddr =
              tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + half * EW);
          uint32_t r[EW];
          if constexpr (EW >= 32) {
#pragma unroll
            for (int j = 0; j < EW / 32; ++j)
              tmem_ld_32x32b_x32(taddr + j * 32, *reinterpret_cast<uint32_t(*)[32]>(r + j * 32));
          } else {
            tmem_ld_32x32b_x16(taddr, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tmem_wait_ld();
          // The partial is in registers: hand the TMEM buffer back.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[b]);
          if constexpr (!SWAP) {
            const float s = vb[kk * 128 + row] * ts;
#pragma unroll
            for (int cc = 0; cc < EW; ++cc) acc[cc] = fmaf(__uint_as_float(r[cc]), s, acc[cc]);
          } else {
            const float4* v4 = reinterpret_cast<const float4*>(vb + kk * 128 + half * EW);
#pragma unroll
            for (int c4 = 0; c4 < EW / 4; ++c4) {
              const float4 sv = v4[c4];
              acc[4 * c4] = fmaf(__uint_as_float(r[4 * c4]) * sv.x, ts, acc[4 * c4]);
              acc[4 * c4 + 1] = fmaf(__uint_as_float(r[4 * c4 + 1]) * sv.y, ts, acc[4 * c4 + 1]);
              acc[4 * c4 + 2] = fmaf(__uint_as_float(r[4 * c4 + 2]) * sv.z, ts, acc[4 * c4 + 2]);
              acc[4 * c4 + 3] = fmaf(__uint_as_float(r[4 * c4 + 3]) * sv.w, ts, acc[4 * c4 + 3]);
            }
          }
        }
        // Every thread is done with this staging buffer before it is refilled.
        named_barrier_sync(1, kF8EpiThreads);
      }
      if (!ok) {
        *abort_flag = 1;
        break;
      }
      // Store the finished tile (bf16).
      const int i = uc.out_i0 + row;  // output index along P
      const int j0 = uc.q_row + half * EW;
      if constexpr (!SWAP) {
        if (i < uc.p_lim) {
          __nv_bfloat16* dst = C + (size_t)i * ldc + j0;
#pragma unroll
          for (int v = 0; v < EW / 8; ++v) {
            if (j0 + v * 8 + 8 <= uc.q_lim) {
              uint4 pk;
              pk.x = pack_bf16x2(acc[8 * v + 0], acc[8 * v + 1]);
              pk.y = pack_bf16x2(acc[8 * v + 2], acc[8 * v + 3]);
              pk.z = pack_bf16x2(acc[8 * v + 4], acc[8 * v + 5]);
              pk.w = pack_bf16x2(acc[8 * v + 6], acc[8 * v + 7]);
              *reinterpret_cast<uint4*>(dst + v * 8) = pk;
            }
          }
        }
      } else {
        // Transposed: lane = weight row = output column; consecutive lanes
        // write consecutive bf16 of one output row.
        if (i < uc.p_lim) {
#pragma unroll
          for (int cc = 0; cc < EW; ++cc) {
            const int j = j0 + cc;
            if (j < uc.q_lim) C[(size_t)j * ldc + i] = __float2bfloat16_rn(acc[cc]);
          }
        }
      }
    }
    cp_async_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Per-expert tile prefix: tiles of expert e = (N / 128) x ceil(rows_e / bn).
__global__ void fp8_grouped_tiles_kernel(const int* __restrict__ row_off, int E, int nbs, int bn,
                                         int* __restrict__ tile_off) {
  pdl_wait();  // row_off comes from the routing kernels
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      tile_off[e] = acc;
      const int rows = row_off[e + 1] - row_off[e];
      acc += nbs * ((rows + bn - 1) / bn);
    }
    tile_off[E] = acc;
  }
}

// Activation quantisation: one warp per (row, 128-wide K group); amax over the
// group, scale = amax / 448 (the e4m3 maximum), q = x * (448 / amax) rounded
// to nearest e4m3 with saturation. Scales go K-group major: sa[g][row].
__global__ void quant_fp8_act_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int M, int K,
                                     uint8_t* __restrict__ xq, int ldq, float* __restrict__ sa,
                                     int ld_sa) {
  pdl_wait();
  const int groups = (K + 127) / 128;
  const long total = (long)M * groups;
  const int lane = threadIdx.x & 31;
  for (long w = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total;
       w += ((long)gridDim.x * blockDim.x) >> 5) {
    const int m = (int)(w / groups), g = (int)(w - (long)m * groups);
    const int k0 = g * 128 + lane * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    const __nv_bfloat16* src = x + (size_t)m * ldx + k0;
    if (k0 + 4 <= K) {
      const uint2 raw = *reinterpret_cast<const uint2*>(src);
      v[0] = bf16_bits_lo(raw.x);
      v[1] = bf16_bits_hi(raw.x);
      v[2] = bf16_bits_lo(raw.y);
      v[3] = bf16_bits_hi(raw.y);
    } else {
      for (int i = 0; i < 4; ++i)
        if (k0 + i < K) v[i] = __bfloat162float(src[i]);
    }
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = amax > 0.f ? amax / 448.f : 1.f;
    const float inv = amax > 0.f ? 448.f / amax : 1.f;
    const __nv_fp8x2_storage_t lo =
        __nv_cvt_float2_to_fp8x2(make_float2(v[0] * inv, v[1] * inv), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi =
        __nv_cvt_float2_to_fp8x2(make_float2(v[2] * inv, v[3] * inv), __NV_SATFINITE, __NV_E4M3);
    uint8_t* dst = xq + (size_t)m * ldq + k0;
    if (k0 + 4 <= K) {
      *reinterpret_cast<uint32_t*>(dst) = (uint32_t)lo | ((uint32_t)hi << 16);
    } else {
      const uint8_t b[4] = {(uint8_t)(lo & 0xff), (uint8_t)(lo >> 8), (uint8_t)(hi & 0xff),
                            (uint8_t)(hi >> 8)};
      for (int i = 0; i < 4; ++i)
        if (k0 + i < K) dst[i] = b[i];
    }
    if (lane == 0) sa[(size_t)g * ld_sa + m] = scale;
  }
}

template <int BN, int STAGES, bool SWAP>
void launch_fp8(const void* P, const void* Q, void* C, int p_rows, int q_rows, int K, int ldp,
                int ldq, int ldc, const F8Args& fa, const GroupInfo& grp, long units,
                unsigned int* err, cudaStream_t stream) {
  using S = F8Smem<BN, STAGES>;
  static_assert(S::kTotal <= 232448, "shared memory budget");
  auto kernel = gemm_fp8_tc_kernel<BN, STAGES, SWAP>;
  static bool attr_set[kMaxDevices] = {};
  set_smem_attr_once(kernel, S::kTotal, attr_set, "gemm_fp8_tc");
  const CUtensorMap tp = make_tmap_2d(P, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p_rows, K,
                                      (uint64_t)ldp, kF8BM, kF8BK);
  const CUtensorMap tq = make_tmap_2d(Q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q_rows, K,
                                      (uint64_t)ldq, BN, kF8BK);
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = units < num_sms(dev) ? (int)units : num_sms(dev);
  if (grid <= 0) return;
  launch_pdl(kernel, dim3(grid), dim3(kF8Threads), S::kTotal, stream, nullptr, tp, tq,
             reinterpret_cast<__nv_bfloat16*>(C), ldc, p_rows, q_rows, K, fa, grp, err);
}

void check_fp8_dims(int K, int lda, int ldw, int ldc) {
  if (K % 16 != 0 || lda % 16 != 0 || ldw % 16 != 0)
    throw std::runtime_error("gemm_fp8: K and the operand row strides must be multiples of 16");
  if (ldc % 8 != 0) throw std::runtime_error("gemm_fp8: ldc must be a multiple of 8");
}

}  // namespace

void quant_fp8_act_launch(const void* x, int ldx, int M, int K, void* xq, int ldq, float* sa,
                          int ld_sa, cudaStream_t stream) {
  if (M <= 0 || K <= 0) return;
  if (ldx % 4 != 0 || ldq % 4 != 0 || K % 4 != 0)
    throw std::runtime_error("quant_fp8_act: K and row strides must be multiples of 4");
  if (ld_sa < M) throw std::runtime_error("quant_fp8_act: ld_sa < M");
  int dev = 0;
  cudaGetDevice(&dev);
  const long warps = (long)M * ((K + 127) / 128);
  const long blocks = (warps + 7) / 8;
  const int grid = (int)(blocks < 8L * num_sms(dev) ? blocks : 8L * num_sms(dev));
  launch_pdl(quant_fp8_act_kernel, dim3(grid), dim3(256), 0, stream, nullptr,
             reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, K,
             reinterpret_cast<uint8_t*>(xq), ldq, sa, ld_sa);
}

void gemm_fp8_launch(const void* Aq, const float* sa, int ld_sa, const void* Wq, const float* sw,
                     int ld_sw, void* C, int M, int N, int K, int lda, int ldw, int ldc, int bn,
                     unsigned int* err, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return;
  check_fp8_dims(K, lda, ldw, ldc);
  if (N % 8 != 0) throw std::runtime_error("gemm_fp8: N must be a multiple of 8");
  const F8Args fa{sa, sw, ld_sa, ld_sw, M};
  const bool swap = bn > 0 ? bn < 128 : M <= 64;
  if (!swap) {
    // Normal: P = A (tokens), Q = W (weight rows), 128 x 128 tiles (one
    // weight block per tile: its scale is a scalar per K block).
    const long units = (long)((M + 127) / 128) * ((N + 127) / 128);
    return launch_fp8<128, 6, false>(Aq, Wq, C, M, N, K, lda, ldw, ldc, fa, GroupInfo{}, units,
                                     err, stream);
  }
  if (bn <= 0) bn = M <= 32 ? 32 : 64;
  const long units = (long)((N + 127) / 128) * ((M + bn - 1) / bn);
  switch (bn) {
    case 32:
      return launch_fp8<32, 10, true>(Wq, Aq, C, N, M, K, ldw, lda, ldc, fa, GroupInfo{}, units,
                                      err, stream);
    case 64:
      return launch_fp8<64, 8, true>(Wq, Aq, C, N, M, K, ldw, lda, ldc, fa, GroupInfo{}, units,
                                     err, stream);
    default:
      throw std::runtime_error("gemm_fp8: swap-AB tile width must be 32 or 64");
  }
}

void gemm_fp8_grouped_launch(const void* Xq, const float* sa, int ld_sa, const void* Wstk,
                             const float* sw, int ld_sw, void* C, int rows, int E, int N, int K,
                             int ldx, int ldw, int ldc, const int* row_off, int* tile_off, int bn,
                             unsigned int* err, cudaStream_t stream) {
  if (rows <= 0 || E <= 0) return;
  check_fp8_dims(K, ldx, ldw, ldc);
  if (N % 128 != 0)
    throw std::runtime_error("gemm_fp8_grouped: N per expert must be a multiple of 128");
  if (bn <= 0) {
    const int avg = rows / E;
    bn = avg <= 32 ? 32 : avg <= 64 ? 64 : 128;
  }
  launch_pdl(fp8_grouped_tiles_kernel, dim3(1), dim3(32), 0, stream, nullptr, row_off, E,
             N / 128, bn, tile_off);
  const GroupInfo g{tile_off, row_off, E, N};
  const long units = (long)(N / 128) * ((rows + bn - 1) / bn + E);
  const F8Args fa{sa, sw, ld_sa, ld_sw, rows};
  const int P = E * N;
  switch (bn) {
    case 32:
      return launch_fp8<32, 10, true>(Wstk, Xq, C, P, rows, K, ldw, ldx, ldc, fa, g, units, err,
                                      stream);
    case 64:
      return launch_fp8<64, 8, true>(Wstk, Xq, C, P, rows, K, ldw, ldx, ldc, fa, g, units, err,
                                     stream);
    case 128:
      return launch_fp8<128, 6, true>(Wstk, Xq, C, P, rows, K, ldw, ldx, ldc, fa, g, units, err,
                                      stream);
    default:
      throw std::runtime_error("gemm_fp8_grouped: tile width must be 32, 64 or 128");
  }
}

}  // namespace b200
