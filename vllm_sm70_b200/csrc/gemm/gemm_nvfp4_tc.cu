// NVFP4 (W4A4) GEMM on the 5th-generation tensor cores with hardware block
// scaling: tcgen05.mma kind::mxf4nvf4, e2m1 x e2m1 operands, one e4m3 scale per
// 16 elements along K for both operands, fp32 accumulation in TMEM.
//
//   C[m, n] = rs[m] * g * sum_k e2m1(A[m,k]) sa[m,k/16] * e2m1(W[n,k]) sw[n,k/16]
//
// A (activations) is quantised per token by quant_nvfp4_act_launch: a per-row
// fp32 scale rs = amax_row / (448 * 6) keeps every block scale inside the
// e4m3 range, block scale sa = e4m3(amax_block / 6 / rs), values
// e2m1(x / (sa * rs)). W is the ModelOpt NVFP4 checkpoint layout (e2m1 pairs,
// low nibble = even k; e4m3 scale per 16 k; global fp32 scale g).
//
// Scale factors live in TMEM, as the block-scaled MMA reads them: per MMA
// (K = 64) a 128-row x 4-scale "atom" of 512 bytes, row r at byte
// (r % 32) * 16 + (r / 32) * 4 + k_sf, copied from shared memory with
// tcgen05.cp 32x128b.warpx4 (each 32-lane sub-partition gets the 32 x 16 B
// block). Both operands' scales are stored in that atom order in global
// memory ([rows / 128][K / 64][512 B]; the weight scales are reordered once at
// load time), so the producer moves them with 2 KB bulk copies per k-block.
//
// Tiles: 128 x 128 (normal: P = A tokens, Q = W rows) or swap-AB (P = W rows,
// Q = 128-token blocks: small M and the grouped MoE form, whose expert row
// blocks start at multiples of 128 in the padded permutation). 6 warps: TMA
// producer, MMA issuer (tcgen05.cp + MMA), 4 epilogue warps; double-buffered
// accumulators. All waits are bounded.
//
// Reference parity: the reference runs NVFP4 weight-only on Volta
// (sm70/csrc/turbomind/ops/tm_nvfp4_sm70.cu:269-278: e2m1 -> f16 with the e4m3
// block scale and the global scale in the operand load); the checkpoint
// format is the same.
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
#include "gemm/dequant.cuh"
#include "gemm/gemm_api.h"

namespace b200 {
namespace {

constexpr int kF4BM = 128, kF4BN = 128;
constexpr int kF4BKB = 128;         // bytes of packed e2m1 per row per k-block (256 k)
constexpr int kF4Stages = 5;
constexpr int kF4Threads = 192;
constexpr int kF4SfBytes = 2048;    // 4 atoms of 512 B: the scales of one k-block (256 k)
constexpr int kF4StageBytes = kF4BM * kF4BKB + kF4BN * kF4BKB + 2 * kF4SfBytes;
constexpr int kF4Smem = kF4Stages * kF4StageBytes + 256 + 1024;
constexpr uint32_t kF4AccCols = 128, kF4SfCol = 256;

struct F4Args {
  const uint8_t* sf_p;     // P operand scales, atom order [p_rows/128][K/64][512]
  const uint8_t* sf_q;     // Q operand scales, atom order [q_rows/128][K/64][512]
  const float* rs;         // per-token fp32 scales (P rows in normal mode, Q rows in swap)
  float g;                 // weight global scale
  int M;                   // tokens (valid range of rs)
};

__device__ __forceinline__ void umma_mxf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t tsfa, uint32_t tsfb,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;"
      "\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// 32 rows x 16 B from shared memory into TMEM lanes 0..31 of every sub-partition.
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// Descriptor of one 512-byte scale atom: no swizzle, 8-row x 16 B core
// matrices 128 B apart.
__device__ __forceinline__ uint64_t sf_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)(128u >> 4) << 16;
  d |= (uint64_t)(128u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// kind::mxf4nvf4: A/B e2m1 (format 1), e4m3 scales (scale format 0), K = 64.
__host__ __device__ constexpr uint32_t idesc_mxf4(int M, int N) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

struct F4Unit {
  int p_row, q_row, out_i0, p_lim, q_lim;
};

__device__ __forceinline__ F4Unit f4_unit(int t, int num_q, const GroupInfo& g, int p_rows,
                                          int q_rows) {
  F4Unit u;
  if (g.E > 0) {
    int lo = 0, hi = g.E;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(g.tile_off + mid) <= t) lo = mid; else hi = mid;
    }
    const int e = lo;
    const int local = t - __ldg(g.tile_off + e);
    const int nbs = g.N / kF4BM;
    const int nb = local % nbs, qb = local / nbs;
    u.p_row = e * g.N + nb * kF4BM;
    u.q_row = __ldg(g.row_off + e) + qb * kF4BN;
    u.out_i0 = nb * kF4BM;
    u.p_lim = g.N;
    u.q_lim = __ldg(g.row_off + e + 1);
    return u;
  }
  const int pb = t / num_q, qb = t - pb * num_q;
  u.p_row = pb * kF4BM;
  u.q_row = qb * kF4BN;
  u.out_i0 = pb * kF4BM;
  u.p_lim = p_rows;
  u.q_lim = q_rows;
  return u;
}

template <bool SWAP>
__global__ void __launch_bounds__(kF4Threads, 1)
gemm_nvfp4_tc_kernel(const __grid_constant__ CUtensorMap tmap_p,
                     const __grid_constant__ CUtensorMap tmap_q, __nv_bfloat16* __restrict__ C,
                     int ldc, int p_rows, int q_rows, int K, const F4Args fa, const GroupInfo grp,
                     unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kF4Stages * kF4StageBytes);
  uint64_t* empty_bar = full_bar + kF4Stages;
  uint64_t* tfull_bar = empty_bar + kF4Stages;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;          // [2]
  uint64_t* done_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_q = (q_rows + kF4BN - 1) / kF4BN;
  const int num_p = (p_rows + kF4BM - 1) / kF4BM;
  const int num_kb = K / 256;
  const int kgs = K / 64;  // atoms per 128-row block

  if (threadIdx.x == 0) {
    for (int s = 0; s < kF4Stages; ++s) {
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
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const int num_units = grp.E > 0 ? __ldg(grp.tile_off + grp.E) : num_p * num_q;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x) {
        const F4Unit uc = f4_unit(u, num_q, grp, p_rows, q_rows);
        const uint8_t* sfp = fa.sf_p + (size_t)(uc.p_row / 128) * kgs * 512;
        const uint8_t* sfq = fa.sf_q + (size_t)(uc.q_row / 128) * kgs * 512;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* sp = smem + stage * kF4StageBytes;
          mbar_arrive_expect_tx(&full_bar[stage], (uint32_t)kF4StageBytes);
          tma_load_2d(sp, &tmap_p, &full_bar[stage], kb * kF4BKB, uc.p_row);
          tma_load_2d(sp + kF4BM * kF4BKB, &tmap_q, &full_bar[stage], kb * kF4BKB, uc.q_row);
          uint8_t* ssf = sp + (kF4BM + kF4BN) * kF4BKB;
          bulk_load(ssf, sfp + (size_t)kb * 4 * 512, kF4SfBytes, &full_bar[stage]);
          bulk_load(ssf + kF4SfBytes, sfq + (size_t)kb * 4 * 512, kF4SfBytes, &full_bar[stage]);
          ++issued;
          if (++stage == kF4Stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      const long n_drain = issued < kF4Stages ? issued : kF4Stages;
      for (long j = 0; j < n_drain; ++j) {
        const long it = issued - 1 - j;
        mbar_wait(&full_bar[it % kF4Stages], (uint32_t)((it / kF4Stages) & 1), err);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_mxf4(kF4BM, kF4BN);
      const uint32_t sf_a = tmem_base + kF4SfCol;       // 16 columns: 4 atoms x 4
      const uint32_t sf_b = tmem_base + kF4SfCol + 16;  // 16 columns
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x, ++local) {
        const int acc = local & 1;
        if (!mbar_wait(&tempty_bar[acc], ((local >> 1) & 1) ^ 1u, err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * kF4AccCols;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t spa = smem_u32(smem + stage * kF4StageBytes);
          const uint32_t ssf = spa + (kF4BM + kF4BN) * kF4BKB;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            tmem_cp_32x128b_x4(sf_a + 4 * i, sf_desc(ssf + 512 * i));
            tmem_cp_32x128b_x4(sf_b + 4 * i, sf_desc(ssf + kF4SfBytes + 512 * i));
          }
          const uint64_t adesc = umma_desc_sw128(spa);
          const uint64_t bdesc = umma_desc_sw128(spa + kF4BM * kF4BKB);
#pragma unroll
          for (int k = 0; k < 4; ++k)  // K = 64 e2m1 = 32 bytes per MMA
            umma_mxf4(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                      sf_a + 4 * k, sf_b + 4 * k, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty_bar[stage]);
          if (++stage == kF4Stages) {
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
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int local = 0;
    for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x, ++local) {
      const F4Unit uc = f4_unit(u, num_q, grp, p_rows, q_rows);
      const int acc = local & 1;
      if (!mbar_wait(&tfull_bar[acc], (local >> 1) & 1, err)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t_acc = tmem_base + ((uint32_t)(q * 32) << 16) + acc * kF4AccCols;
      const int i = uc.out_i0 + row;  // output index along P
      float prow = fa.g;
      if constexpr (!SWAP) {
        const int m = uc.p_row + row;
        prow = m < fa.M ? fa.rs[m] * fa.g : 0.f;
      }
#pragma unroll 1
      for (int ch = 0; ch < kF4BN / 32; ++ch) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_acc + ch * 32, r);
        tmem_wait_ld();
        const int j0 = uc.q_row + ch * 32;
        if constexpr (!SWAP) {
          if (i < uc.p_lim) {
            __nv_bfloat16* dst = C + (size_t)i * ldc + j0;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              if (j0 + v * 8 + 8 <= uc.q_lim) {
                uint4 pk;
                pk.x = pack_bf16x2(__uint_as_float(r[8 * v]) * prow, __uint_as_float(r[8 * v + 1]) * prow);
                pk.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * prow, __uint_as_float(r[8 * v + 3]) * prow);
                pk.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * prow, __uint_as_float(r[8 * v + 5]) * prow);
                pk.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * prow, __uint_as_float(r[8 * v + 7]) * prow);
                *reinterpret_cast<uint4*>(dst + v * 8) = pk;
              }
            }
          }
        } else {
          if (i < uc.p_lim) {
#pragma unroll 4
            for (int c = 0; c < 32; ++c) {
              const int j = j0 + c;
              if (j < uc.q_lim)
                C[(size_t)j * ldc + i] = __float2bfloat16_rn(__uint_as_float(r[c]) * prow * __ldg(fa.rs + j));
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
    tmem_dealloc(tmem_base, 512);
  }
}

// Per token: rs = amax_row / (448 * 6); per 16-element block: e4m3 scale
// sa = e4m3(amax_block / 6 / rs) written in atom order, values
// e2m1(x / (sa * rs)) packed two per byte (low nibble = even k). Rows past M
// up to the 128-row atom boundary get zero scales. One CTA per row.
__global__ void __launch_bounds__(128) quant_nvfp4_act_kernel(
    const __nv_bfloat16* __restrict__ x, int ldx, int M, int K, uint8_t* __restrict__ xq,
    int ldq, uint8_t* __restrict__ sf, float* __restrict__ rs, const int* __restrict__ n_rows) {
  pdl_wait();
  const int m = blockIdx.x;
  if (n_rows != nullptr && m >= *n_rows) return;
  const int nblk = K / 16;
  const int kgs = K / 64;
  __shared__ float red[4];
  uint8_t* atom_row = sf + (size_t)(m / 128) * kgs * 512 + (m % 32) * 16 + ((m % 128) / 32) * 4;
  if (m >= M) {
    for (int b = threadIdx.x; b < nblk; b += blockDim.x) atom_row[(b / 4) * 512 + (b % 4)] = 0;
    return;
  }
  const __nv_bfloat16* row = x + (size_t)m * ldx;
  float amax = 0.f;
  for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(row + b * 16);
    const uint4 a = src[0], c = src[1];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
      amax = fmaxf(amax, fmaxf(fabsf(bf16_bits_lo(w[i])), fabsf(bf16_bits_hi(w[i]))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float r_scale = amax > 0.f ? amax / 2688.f : 1.f;  // 2688 = 448 * 6
  if (threadIdx.x == 0) rs[m] = r_scale;
  for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(row + b * 16);
    const uint4 a = src[0], c = src[1];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
    float v[16];
    float bmax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[2 * i] = bf16_bits_lo(w[i]);
      v[2 * i + 1] = bf16_bits_hi(w[i]);
      bmax = fmaxf(bmax, fmaxf(fabsf(v[2 * i]), fabsf(v[2 * i + 1])));
    }
    const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(bmax / 6.f / r_scale, __NV_SATFINITE, __NV_E4M3);
    const float sdec = e4m3_to_float((uint8_t)s8) * r_scale;
    const float inv = sdec > 0.f ? 1.f / sdec : 0.f;
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t byte;
      asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
          : "=r"(byte)
          : "f"(v[2 * i + 1] * inv), "f"(v[2 * i] * inv));
      packed[i / 4] |= (byte & 0xffu) << (8 * (i % 4));
    }
    *reinterpret_cast<uint2*>(xq + (size_t)m * ldq + b * 8) = make_uint2(packed[0], packed[1]);
    atom_row[(b / 4) * 512 + (b % 4)] = (uint8_t)s8;
  }
}

__global__ void nvfp4_grouped_tiles_kernel(const int* __restrict__ row_off, int E, int nbs,
                                           int* __restrict__ tile_off) {
  pdl_wait();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      tile_off[e] = acc;
      const int rows = row_off[e + 1] - row_off[e];
      acc += nbs * ((rows + kF4BN - 1) / kF4BN);
    }
    tile_off[E] = acc;
  }
}

template <bool SWAP>
void launch_nvfp4(const void* P, const void* Q, void* C, int p_rows, int q_rows, int K, int ldp,
                  int ldq, int ldc, const F4Args& fa, const GroupInfo& grp, long units,
                  unsigned int* err, cudaStream_t stream) {
  static_assert(kF4Smem <= 232448, "shared memory budget");
  auto kernel = gemm_nvfp4_tc_kernel<SWAP>;
  static bool attr_set[kMaxDevices] = {};
  set_smem_attr_once(kernel, kF4Smem, attr_set, "gemm_nvfp4_tc");
  const CUtensorMap tp = make_tmap_2d(P, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p_rows, K / 2,
                                      (uint64_t)ldp, kF4BM, kF4BKB);
  const CUtensorMap tq = make_tmap_2d(Q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q_rows, K / 2,
                                      (uint64_t)ldq, kF4BN, kF4BKB);
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = units < num_sms(dev) ? (int)units : num_sms(dev);
  if (grid <= 0) return;
  launch_pdl(kernel, dim3(grid), dim3(kF4Threads), kF4Smem, stream, nullptr, tp, tq,
             reinterpret_cast<__nv_bfloat16*>(C), ldc, p_rows, q_rows, K, fa, grp, err);
}

void check_nvfp4(int K, int ldq_bytes, int ldw_bytes, int ldc) {
  if (K % 256 != 0) throw std::runtime_error("gemm_nvfp4: K must be a multiple of 256");
  if (ldq_bytes % 16 != 0 || ldw_bytes % 16 != 0 || ldc % 8 != 0)
    throw std::runtime_error("gemm_nvfp4: row strides must be 16-byte multiples");
}

}  // namespace

void quant_nvfp4_act_launch(const void* x, int ldx, int M, int K, void* xq, int ldq, void* sf,
                            float* rs, cudaStream_t stream, const int* n_rows) {
  if (M <= 0) return;
  if (K % 64 != 0) throw std::runtime_error("quant_nvfp4_act: K must be a multiple of 64");
  if (ldx % 8 != 0 || ldq % 8 != 0) throw std::runtime_error("quant_nvfp4_act: row strides");
  const int rows = (M + 127) / 128 * 128;  // whole atoms: padded rows get zero scales
  launch_pdl(quant_nvfp4_act_kernel, dim3(rows), dim3(128), 0, stream, nullptr,
             reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, K, reinterpret_cast<uint8_t*>(xq),
             ldq, reinterpret_cast<uint8_t*>(sf), rs, n_rows);
}

void gemm_nvfp4_launch(const void* Aq, const void* sfa, const float* rs, const void* Wq,
                       const void* sfw, float g, void* C, int M, int N, int K, int lda, int ldw,
                       int ldc, int swap, unsigned int* err, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return;
  check_nvfp4(K, lda, ldw, ldc);
  if (N % 8 != 0) throw std::runtime_error("gemm_nvfp4: N must be a multiple of 8");
  const bool sw = swap < 0 ? M <= 128 : swap != 0;
  F4Args fa{nullptr, nullptr, rs, g, M};
  if (!sw) {
    fa.sf_p = reinterpret_cast<const uint8_t*>(sfa);
    fa.sf_q = reinterpret_cast<const uint8_t*>(sfw);
    const long units = (long)((M + 127) / 128) * ((N + 127) / 128);
    return launch_nvfp4<false>(Aq, Wq, C, M, N, K, lda, ldw, ldc, fa, GroupInfo{}, units, err,
                               stream);
  }
  fa.sf_p = reinterpret_cast<const uint8_t*>(sfw);
  fa.sf_q = reinterpret_cast<const uint8_t*>(sfa);
  const long units = (long)((N + 127) / 128) * ((M + 127) / 128);
  launch_nvfp4<true>(Wq, Aq, C, N, M, K, ldw, lda, ldc, fa, GroupInfo{}, units, err, stream);
}

void gemm_nvfp4_grouped_launch(const void* Xq, const void* sfx, const float* rs, const void* Wstk,
                               const void* sfw, float g, void* C, int rows, int E, int N, int K,
                               int ldx, int ldw, int ldc, const int* row_off, int* tile_off,
                               unsigned int* err, cudaStream_t stream) {
  if (rows <= 0 || E <= 0) return;
  check_nvfp4(K, ldx, ldw, ldc);
  if (N % 128 != 0) throw std::runtime_error("gemm_nvfp4_grouped: N per expert must be a multiple of 128");
  launch_pdl(nvfp4_grouped_tiles_kernel, dim3(1), dim3(32), 0, stream, nullptr, row_off, E,
             N / 128, tile_off);
  const GroupInfo grp{tile_off, row_off, E, N};
  F4Args fa{reinterpret_cast<const uint8_t*>(sfw), reinterpret_cast<const uint8_t*>(sfx), rs, g,
            rows};
  const long units = (long)(N / 128) * ((rows + 127) / 128 + E);
  launch_nvfp4<true>(Wstk, Xq, C, E * N, rows, K, ldw, ldx, ldc, fa, grp, units, err, stream);
}

}  // namespace b200
