// Persistent warp-specialised BF16 GEMM on the 5th-generation tensor cores.
//
//   D[i, j] = sum_k P[i, k] * Q[j, k]        (both operands K-major, fp32 accumulate)
//
// Normal mode: P = activations A[M, K], Q = weights W[N, K]  -> C[M, N] = A W^T
// Swap-AB mode (small M): P = W, Q = A and the tile is written transposed,
// so the 128-row UMMA M side is filled by weight rows and the token count
// only has to cover the (>= 16) UMMA N side.
//
// Pipeline (one CTA per SM, 6 warps):
//   warp 0      TMA producer: one elected lane streams 128x64 P tiles and
//               BNx64 Q tiles (128-byte swizzle) into a STAGES-deep smem ring.
//   warp 1      TMEM allocator + MMA issuer: one lane issues tcgen05.mma
//               (M=128, N=BN, K=16) into a double-buffered TMEM accumulator and
//               tcgen05.commit's the smem slot back to the producer.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, convert, optional
//               fused SiLU(gate)*up, store bf16 to global. Runs concurrently
//               with the next tile's main loop (accumulator double buffer).
//
// Reference parity: replaces the TurboMind sm70 GEMM family
// (sm70/csrc/turbomind/lmdeploy/src/turbomind/kernels/gemm/gemm.h:14-50,
// kernel/sm70_884_*.cu) and its gated-SiLU epilogue (types.h:141); the
// reference computes the same contraction with mma.sync m8n8k4 on sm_70.
//
// All mbarrier waits are bounded (common/ptx.cuh); on a timeout every role
// leaves its loop, the MMA issuer drains its outstanding MMAs, the producer
// drains its outstanding TMA copies, and the CTA frees TMEM before exiting.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "common/ptx.cuh"
#include "common/tmap.h"
#include "gemm/gemm_api.h"

namespace b200 {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int UMMA_K = 16;
constexpr int kThreads = 192;
constexpr int kGroupM = 16;  // rasterisation group (M tiles) for L2 reuse

struct TileCoord {
  int mb, nb;
};

__device__ __forceinline__ TileCoord tile_coord(int t, int num_m, int num_n) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - g * per_group;
  return {first_m + r % gsize, r / gsize};
}

template <int BN, int STAGES>
struct Smem {
  static constexpr int kPBytes = BM * BK * 2;
  static constexpr int kQBytes = BN * BK * 2;
  static constexpr int kStageBytes = kPBytes + kQBytes;
  static constexpr int kTileBytes = STAGES * kStageBytes;
  static constexpr int kBarBytes = 256;
  static constexpr int kTotal = kTileBytes + kBarBytes + 1024;  // +1024 for manual alignment
};

template <int BN, int STAGES, bool SWAP, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmap_p,
                    const __grid_constant__ CUtensorMap tmap_q, __nv_bfloat16* __restrict__ C,
                    int ldc, int p_rows, int q_rows, int K, unsigned int* err) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S::kTileBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;      // [2]
  uint64_t* done_bar = tempty_bar + 2;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (p_rows + BM - 1) / BM;
  const int num_n = (q_rows + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  constexpr uint32_t kTmemCols = 2 * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 4);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        const TileCoord tc = tile_coord(t, num_m, num_n);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* sp = smem + stage * S::kStageBytes;
          mbar_arrive_expect_tx(&full_bar[stage], S::kStageBytes);
          tma_load_2d(sp, &tmap_p, &full_bar[stage], kb * BK, tc.mb * BM);
          tma_load_2d(sp + S::kPBytes, &tmap_q, &full_bar[stage], kb * BK, tc.nb * BN);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: wait for the copies this thread issued into each slot (bounded).
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
      constexpr uint32_t idesc = umma_idesc_f16(BM, BN, true);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sp = smem_u32(smem + stage * S::kStageBytes);
          const uint64_t adesc = umma_desc_sw128(sp);
          const uint64_t bdesc = umma_desc_sw128(sp + S::kPBytes);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // +32 bytes per K=16 step inside the 128-byte swizzle row.
            umma_f16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                     (kb | k) != 0);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit(&tfull_bar[acc]);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
      // Make sure no MMA is still writing TMEM before it is freed.
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = q * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++local) {
      const TileCoord tc = tile_coord(t, num_m, num_n);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      const int i = tc.mb * BM + row_in_tile;  // P row
      if constexpr (EPI == kEpiSiluMul) {
        // Tile columns hold [gate 64 | up 64] blocks; output has BN/2 columns.
#pragma unroll 1
        for (int blk = 0; blk < BN / 128; ++blk) {
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {
            uint32_t g[32], u[32];
            tmem_ld_32x32b_x32(t_row + blk * 128 + half * 32, g);
            tmem_ld_32x32b_x32(t_row + blk * 128 + 64 + half * 32, u);
            tmem_wait_ld();
            const int j0 = tc.nb * (BN / 2) + blk * 64 + half * 32;
            if (i < p_rows) {
              uint32_t packed[16];
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                float g0 = __uint_as_float(g[2 * c]), g1 = __uint_as_float(g[2 * c + 1]);
                float u0 = __uint_as_float(u[2 * c]), u1 = __uint_as_float(u[2 * c + 1]);
                float o0 = g0 / (1.0f + __expf(-g0)) * u0;
                float o1 = g1 / (1.0f + __expf(-g1)) * u1;
                packed[c] = pack_bf16x2(o0, o1);
              }
              __nv_bfloat16* dst = C + (size_t)i * ldc + j0;
              const int out_cols = q_rows / 2;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                if (j0 + v * 8 + 8 <= out_cols)
                  *reinterpret_cast<uint4*>(dst + v * 8) =
                      make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2],
                                 packed[4 * v + 3]);
              }
            }
          }
        }
      } else {
        constexpr int CW = BN >= 32 ? 32 : 16;  // columns per tcgen05.ld
#pragma unroll 1
        for (int ch = 0; ch < BN / CW; ++ch) {
          uint32_t r[32];
          if constexpr (CW == 32) {
            tmem_ld_32x32b_x32(t_row + ch * CW, r);
          } else {
            uint32_t (&r16)[16] = *reinterpret_cast<uint32_t(*)[16]>(r);
            tmem_ld_32x32b_x16(t_row + ch * CW, r16);
          }
          tmem_wait_ld();
          const int j0 = tc.nb * BN + ch * CW;
          if constexpr (!SWAP) {
            if (i < p_rows) {
              __nv_bfloat16* dst = C + (size_t)i * ldc + j0;
#pragma unroll
              for (int v = 0; v < CW / 8; ++v) {
                if (j0 + v * 8 + 8 <= q_rows) {
                  uint4 pk;
                  pk.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
                  pk.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
                  pk.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
                  pk.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
                  *reinterpret_cast<uint4*>(dst + v * 8) = pk;
                }
              }
            }
          } else {
            // Transposed store: lane i holds P row i (an output column);
            // consecutive lanes write consecutive bf16 of one output row.
            if (i < p_rows) {
#pragma unroll
              for (int c = 0; c < CW; ++c) {
                const int j = j0 + c;
                if (j < q_rows) C[(size_t)j * ldc + i] = __float2bfloat16_rn(__uint_as_float(r[c]));
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int BN, int STAGES, bool SWAP, int EPI>
void launch_cfg(const void* P, const void* Q, void* C, int p_rows, int q_rows, int K, int ldp,
                int ldq, int ldc, unsigned int* err, cudaStream_t stream) {
  using S = Smem<BN, STAGES>;
  auto kernel = gemm_bf16_tc_kernel<BN, STAGES, SWAP, EPI>;
  static bool attr_set = false;  // per instantiation; idempotent if raced
  if (!attr_set) {
    cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    if (e != cudaSuccess)
      throw std::runtime_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    attr_set = true;
  }
  CUtensorMap tp = make_tmap_2d(P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p_rows, K,
                                (uint64_t)ldp * 2, BM, BK);
  CUtensorMap tq = make_tmap_2d(Q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q_rows, K,
                                (uint64_t)ldq * 2, BN, BK);
  int dev = 0;
  cudaGetDevice(&dev);
  const int tiles = ((p_rows + BM - 1) / BM) * ((q_rows + BN - 1) / BN);
  const int grid = tiles < num_sms(dev) ? tiles : num_sms(dev);
  kernel<<<grid, kThreads, S::kTotal, stream>>>(tp, tq, reinterpret_cast<__nv_bfloat16*>(C), ldc,
                                                p_rows, q_rows, K, err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("gemm_bf16_tc launch: ") + cudaGetErrorString(e));
}

}  // namespace

int gemm_bf16_pick_config(int M, int N, int K, int epi, int num_sm) {
  // Swap-AB for small token counts: the weight fills the 128-row M side.
  if (epi == kEpiNone && M <= 64) {
    if (M <= 16) return kCfgSwap16;
    if (M <= 32) return kCfgSwap32;
    return kCfgSwap64;
  }
  const long tiles256 = (long)((M + 127) / 128) * ((N + 255) / 256);
  const long tiles128 = (long)((M + 127) / 128) * ((N + 127) / 128);
  if (tiles256 >= 2L * num_sm) return kCfgN256;
  if (tiles128 >= num_sm || epi == kEpiSiluMul) return tiles256 >= num_sm ? kCfgN256 : kCfgN128;
  return kCfgN128;
}

void gemm_bf16_launch(const void* A, const void* W, void* C, int M, int N, int K, int lda, int ldw,
                      int ldc, int epi, int cfg, unsigned int* err, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return;
  if (K % 8 != 0 || lda % 8 != 0 || ldw % 8 != 0)
    throw std::runtime_error("gemm_bf16: K and leading dims must be multiples of 8");
  if (N % 8 != 0 || ldc % 8 != 0) throw std::runtime_error("gemm_bf16: N, ldc must be multiples of 8");
  int dev = 0;
  cudaGetDevice(&dev);
  if (cfg < 0) cfg = gemm_bf16_pick_config(M, N, K, epi, num_sms(dev));
  if (epi == kEpiSiluMul) {
    if (N % 128 != 0) throw std::runtime_error("gemm_bf16 silu_mul: N must be a multiple of 128");
    if (cfg == kCfgN256)
      return launch_cfg<256, 4, false, kEpiSiluMul>(A, W, C, M, N, K, lda, ldw, ldc, err, stream);
    return launch_cfg<128, 6, false, kEpiSiluMul>(A, W, C, M, N, K, lda, ldw, ldc, err, stream);
  }
  switch (cfg) {
    case kCfgN256:
      return launch_cfg<256, 4, false, kEpiNone>(A, W, C, M, N, K, lda, ldw, ldc, err, stream);
    case kCfgN128:
      return launch_cfg<128, 6, false, kEpiNone>(A, W, C, M, N, K, lda, ldw, ldc, err, stream);
    case kCfgSwap16:
      return launch_cfg<16, 8, true, kEpiNone>(W, A, C, N, M, K, ldw, lda, ldc, err, stream);
    case kCfgSwap32:
      return launch_cfg<32, 8, true, kEpiNone>(W, A, C, N, M, K, ldw, lda, ldc, err, stream);
    case kCfgSwap64:
      return launch_cfg<64, 8, true, kEpiNone>(W, A, C, N, M, K, ldw, lda, ldc, err, stream);
    default:
      throw std::runtime_error("gemm_bf16: unknown config " + std::to_string(cfg));
  }
}

}  // namespace b200
