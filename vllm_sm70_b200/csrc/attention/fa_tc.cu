// Prefill / chunked-prefill paged attention on the 5th-generation tensor
// cores (head_dim 128 or 256, bf16, causal with optional sliding window and
// sinks). Head_dim 256 (Qwen3-Next full attention) runs 64-key tiles: FN and
// the ring depth come from FaCfg; the description below is for head_dim 128.
//
// One CTA owns 128 query rows of one (sequence, KV head): GQA-packed rows
// r -> token t0 + r / G, head kvh * G + r % G, so every K/V tile is read once
// for the whole group. Six warps:
//   warp 0     producer: the Q tile once (3-D tensor map over q [T][Hq][D],
//              box 64 x G x 128/G, 128-byte swizzle), then each 128-key K and
//              V tile from the paged cache (3-D maps over [block][head*BS +
//              key][d], one box per (cache block, 64-column half)) into
//              separate 3-stage K and V rings, K one tile ahead of V.
//   warp 1     TMEM owner + MMA issuer: S_j = Q K_j^T (M=N=K=128) into one of
//              two TMEM S buffers, then O += P_{j-1} V_{j-1} with P read from
//              TMEM as the A operand and V as an MN-major B operand; S of the
//              next tile is issued before the PV of the previous one so the
//              tensor core works while the softmax warps do.
//   warps 2-5  softmax, one query row per thread: tcgen05.ld of its S row
//              (64 scores per wait), running max, exp2 via packed fp32 pairs,
//              row sum, P as bf16 pairs tcgen05.st into one of two TMEM P
//              buffers. Tiles that need no causal / window / padding mask run
//              a mask-free sweep. O is rescaled in TMEM only when a row's
//              running max grows by more than 2^8 over the max its
//              exponentials use, so most tiles skip the correction; at the end
//              each thread normalises its O row and stores it.
// TMEM: S0 | S1 | O | P0 | P1 = 128 + 128 + 128 + 64 + 64 columns.
// Rows of a partly filled last cache block hold stale data: their scores are
// masked by selection, and the softmax warps zero the matching V rows before
// the last PV (a zero P times a stale NaN would not be zero).
//
// Reference parity: the Flash-V100 prefill / chunked-prefill kernel
// (sm70/csrc/flash_v100/fused_mha_forward_paged.cu:357) with its paged block
// table, GQA and causal rules; the reference computes it with WMMA on sm_70.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "attention/attn_api.h"
#include "common/launch.h"
#include "common/ptx.cuh"
#include "common/tmap.h"
#include "ops_api.h"

namespace b200 {
namespace {

constexpr int FM = 128;                // query rows per CTA
constexpr int kBarBytes = 256;
constexpr int kFaThreads = 224;
constexpr uint32_t kTmemColsFa = 512;

// Tile geometry per head dim: head_dim 128 streams 128-key tiles through a
// 3-stage ring; head_dim 256 uses 64-key tiles and 2 stages so that S0 | S1
// (2 FN) + O (FD) + P0 | P1 (FN) columns fit TMEM and Q (64 KB) + the ring
// fit shared memory. Rows of every operand are 64 bf16 = 128 bytes (128-byte
// swizzle); a row of FD values is FD / 64 such chunks.
template <int D_>
struct FaCfg {
  static constexpr int FD = D_;
  static constexpr int FN = D_ == 128 ? 128 : 64;
  static constexpr int FNS = D_ == 128 ? 3 : 2;
  static constexpr int kDC = FD / 64;             // 64-column chunks per row
  static constexpr int kQChunk = FM * 128;        // Q: 128 rows x 64 bf16
  static constexpr int kKVChunk = FN * 128;       // K or V: FN keys x 64 bf16
  static constexpr int kQBytes = kDC * kQChunk;
  static constexpr int kKBytes = kDC * kKVChunk;  // K (then V) of one tile
  static constexpr int kKVBytes = 2 * kKBytes;
  static constexpr int kSmem = kQBytes + FNS * kKVBytes + kBarBytes + 1024;
  static_assert(2 * FN + FD + FN <= (int)kTmemColsFa, "TMEM columns");
  static_assert(kSmem <= 232448, "shared memory");
};

struct FaParams {
  const int* block_table;
  const int* seq_lens;
  const int* cu_q;
  const float* sinks;
  __nv_bfloat16* out;
  int num_seqs, Hq, Hkv, G, block_size, block_shift, max_blocks, window, o_stride_t;
  int num_blocks;  // cache blocks (debug-build bounds checks)
  float scale_log2;
  unsigned int* err;
  uint32_t v_lbo, v_sbo;  // V (MN-major B operand) descriptor strides, bytes
};

// Optional per-CTA timeline (profiling aid, off unless a buffer is installed
// with fa_tc_set_timeline): %globaltimer stamps, 8 slots per CTA.
__device__ unsigned long long* g_fa_timeline = nullptr;

// 2^x on the multi-function unit (P values lie in [0, 2^8]).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int D_>
__global__ void __launch_bounds__(kFaThreads, 1)
fa_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
             const __grid_constant__ CUtensorMap tmv, const FaParams p) {
  using Cfg = FaCfg<D_>;
  constexpr int FD = Cfg::FD, FN = Cfg::FN, FNS = Cfg::FNS, kDC = Cfg::kDC;
  constexpr int kQChunk = Cfg::kQChunk, kKVChunk = Cfg::kKVChunk, kQBytes = Cfg::kQBytes;
  constexpr int kKBytes = Cfg::kKBytes, kKVBytes = Cfg::kKVBytes;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kQBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + FNS * kKVBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;            // [FNS]
  uint64_t* k_empty = k_full + FNS;       // [FNS]
  uint64_t* v_full = k_empty + FNS;       // [FNS]
  uint64_t* v_empty = v_full + FNS;       // [FNS]
  uint64_t* s_full = v_empty + FNS;       // [2]
  uint64_t* s_free = s_full + 2;          // [2]
  uint64_t* p_full = s_free + 2;          // [2]
  uint64_t* p_free = p_full + 2;          // [2]
  uint64_t* o_done = p_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  unsigned long long* const tl = g_fa_timeline;
  const size_t tl_cta =
      ((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
#define FA_TL(i) \
  do { if (tl) tl[tl_cta * 64 + (i)] = globaltimer(); } while (0)
  // per-tile detail (first 8 tiles): slot 8 + 7 * j + k
#define FA_TLJ(j, k) \
  do { if (tl && (j) < 8) tl[tl_cta * 64 + 8 + 7 * (j) + (k)] = globaltimer(); } while (0)
  if (threadIdx.x == 0) FA_TL(0);
  pdl_wait();
  const int seq = blockIdx.y;
  const int kvh = blockIdx.z;
  const int G = p.G;
  const int q0 = p.cu_q[seq];
  const int q_len = p.cu_q[seq + 1] - q0;
  const int seq_len = p.seq_lens[seq];
  const int n_qt = (q_len * G + FM - 1) / FM;
  const int qt = (int)gridDim.x - 1 - (int)blockIdx.x;  // longest causal rows first
  if (qt >= n_qt) return;
  const int tpt = FM / G;  // tokens per tile
  const int t0 = qt * tpt;
  const int pos_first = seq_len - q_len + t0;
  const int pos_last = seq_len - q_len + min(q_len, t0 + tpt) - 1;
  int k_lo = p.window > 0 ? max(0, pos_first - p.window + 1) : 0;
  k_lo = (k_lo / FN) * FN;
  const int k_hi = pos_last + 1;
  const int n_tiles = (k_hi - k_lo + FN - 1) / FN;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < FNS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&p_full[b], 4);  // one arrival per softmax warp, after its P / V writes
      mbar_init(&p_free[b], 1);
    }
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmq);
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemColsFa);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) {
    pdl_trigger();
    FA_TL(1);
  }
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tS = tmem_base, tO = tmem_base + 2 * FN, tP = tO + FD;
  const int BS = p.block_size;
  const int blk_last = (seq_len - 1) >> p.block_shift;

  if (warp == 0 || warp == 6) {
    // ------------------------------------------------- producers (K: 0, V: 6)
    const bool is_v = warp == 6;
    const int* bt = p.block_table + (size_t)seq * p.max_blocks;
    const int nb = FN / BS;
    if (!is_v && lane == 0) {
      mbar_arrive_expect_tx(q_full, (uint32_t)kQBytes);
#pragma unroll
      for (int c = 0; c < kDC; ++c)
        tma_load_3d(sQ + c * kQChunk, &tmq, q_full, c * 64, kvh * G, q0 + t0);
    }
    // Cache-block ids are fetched ahead: one warp-wide load covers `per`
    // tiles (lane L: tile L / nb, block L % nb), and the next group's load is
    // in flight while the current group is issued.
    const int per = 32 / nb;
    auto load_ids = [&](int g) -> int {
      const int tile = g * per + lane / nb;
      if (tile >= n_tiles) return 0;
      const int b = ((k_lo + tile * FN) >> p.block_shift) + lane % nb;
      const int id = __ldg(bt + min(b, blk_last));
      return in_bounds(id >= 0 && id < p.num_blocks, p.err) ? id : 0;
    };
    int ids_cur = load_ids(0), ids_next = load_ids(1), g_cur = 0;
    // K and V stream from separate warps: K_j's slot frees right after S_j,
    // V_j's only after PV_j, so K never queues behind V.
    auto issue = [&](int j) -> bool {
      const int g = j / per;
      if (g > g_cur) {
        ids_cur = ids_next;
        ids_next = load_ids(++g_cur + 1);
      }
      const int ids = g == g_cur ? ids_cur : ids_next;
      const int st = j % FNS;
      const uint32_t ph = (uint32_t)((j / FNS) & 1);
      uint64_t* fullb = is_v ? &v_full[st] : &k_full[st];
      int ok = 1;
      if (lane == 0) {
        ok = mbar_wait(is_v ? &v_empty[st] : &k_empty[st], ph ^ 1u, p.err) ? 1 : 0;
        FA_TLJ(j, is_v ? 1 : 0);
        if (ok) mbar_arrive_expect_tx(fullb, (uint32_t)kKBytes);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return false;
      uint8_t* dst = sKV + st * kKVBytes + (is_v ? kKBytes : 0);
      const CUtensorMap* tm = is_v ? &tmv : &tmk;
      // One (cache block, column half) per lane: a bulk-tensor instruction
      // costs the issuing warp a few hundred ns plus a little per active
      // lane, so the tile's kDC * nb boxes go out as one warp-wide instruction.
      const int bi = lane % nb;
      const int blk = __shfl_sync(0xffffffffu, ids, (j % per) * nb + bi);
      if (lane < kDC * nb) {
        const int h = lane / nb;
        tma_load_3d(dst + h * kKVChunk + bi * BS * 128, tm, fullb, h * 64, kvh * BS, blk);
      }
      return true;
    };
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) ok = issue(j);
    if (!ok) *abort_flag = 1;
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_f16(FM, FN, true);
      constexpr uint32_t idesc_pv = umma_idesc_f16(FM, FD, true) | (1u << 16);  // B MN-major
      bool ok = mbar_wait(q_full, 0, p.err);
      FA_TL(2);
      auto pv = [&](int i) -> bool {
        const int st = i % FNS, pb = i & 1;
        if (!mbar_wait(&p_full[pb], (uint32_t)((i >> 1) & 1), p.err) ||
            !mbar_wait(&v_full[st], (uint32_t)((i / FNS) & 1), p.err))
          return false;
        FA_TLJ(i, 3);
        tc_fence_after();
        const uint32_t sv = smem_u32(sKV + st * kKVBytes + kKBytes);
#pragma unroll
        for (int s = 0; s < FN / 16; ++s) {
          const uint64_t bv = umma_desc_sw128_mn(sv + s * 16 * 128, p.v_lbo, p.v_sbo);
          umma_f16_ts(tO, tP + pb * (FN / 2) + s * 8, bv, idesc_pv, (i > 0 || s > 0) ? 1u : 0u);
        }
        umma_commit(&p_free[pb]);
        umma_commit(&v_empty[st]);
        return true;
      };
      int stage = 0;
      uint32_t phase = 0;
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int sb = j & 1;
        if (!mbar_wait(&s_free[sb], (uint32_t)(((j >> 1) & 1) ^ 1), p.err) ||
            !mbar_wait(&k_full[stage], phase, p.err)) {
          ok = false;
          break;
        }
        FA_TLJ(j, 2);
        tc_fence_after();
        const uint32_t sq = smem_u32(sQ);
        const uint32_t sk = smem_u32(sKV + stage * kKVBytes);
#pragma unroll
        for (int kb = 0; kb < kDC; ++kb) {
          const uint64_t aq = umma_desc_sw128(sq + kb * kQChunk);
          const uint64_t bk = umma_desc_sw128(sk + kb * kKVChunk);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tS + sb * FN, aq + (uint64_t)(2 * k), bk + (uint64_t)(2 * k), idesc_s,
                     (kb > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[stage]);
        if (j > 0 && !pv(j - 1)) {
          ok = false;
          break;
        }
        if (++stage == FNS) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok && n_tiles > 0) ok = pv(n_tiles - 1);
      if (!ok) *abort_flag = 1;
      umma_commit(o_done);
      mbar_wait(o_done, 0, p.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const int stid = threadIdx.x - 64;  // 0..127
    const int t = row / G;
    const int head = kvh * G + row % G;
    const bool valid_row = t0 + t < q_len;
    const int row_pos = seq_len - q_len + t0 + t;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    // Keys this row may attend to: [key_lo, key_hi] (empty for padding rows).
    const int key_hi = valid_row ? min(row_pos, seq_len - 1) : -1;
    const int key_lo = p.window > 0 ? row_pos - p.window + 1 : 0;
    const float sc = p.scale_log2;
    const uint64_t sc2 = f32x2_pack(sc, sc);
    float m_used = -INFINITY, l = 0.f;  // running max (log2 units) and row sum
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1, pb = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (uint32_t)((j >> 1) & 1), p.err));
      if (!ok) break;
      if (stid == 0 && j == 0) FA_TL(3);
      if (stid == 0) FA_TLJ(j, 4);
      tc_fence_after();
      const int kbase = k_lo + j * FN;
      const int lo = key_lo - kbase, hi = key_hi - kbase;  // in-tile bounds
      const bool masked = __any_sync(0xffffffffu, lo > 0 || hi < FN - 1);
      const uint32_t s_row = tS + lane_base + sb * FN;
      const uint32_t p_row = tP + lane_base + pb * (FN / 2);
      // One sweep over the row's 128 raw scores, 64 per TMEM wait. With
      // WRITE: P = exp2(S * scale - mu) packed as bf16 pairs into this row's
      // lane of the P buffer (key 2c, 2c+1 -> column c), row sum into *rs.
      // Returns the row max in log2 units.
      auto sweep = [&](auto masked_c, auto write_c, float mu, float* rs) -> float {
        constexpr bool kMasked = decltype(masked_c)::value;
        constexpr bool kWrite = decltype(write_c)::value;
        float mxa = -INFINITY, mxb = -INFINITY;
        uint64_t acc = f32x2_pack(0.f, 0.f);
        const float mu_eff = mu == -INFINITY ? 0.f : mu;
        const uint64_t nmu2 = f32x2_pack(-mu_eff, -mu_eff);
#pragma unroll 1
        for (int h = 0; h < FN / 64; ++h) {
          uint32_t r[2][32];
          tmem_ld_32x32b_x32(s_row + h * 64, r[0]);
          tmem_ld_32x32b_x32(s_row + h * 64 + 32, r[1]);
          tmem_wait_ld();
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float va = __uint_as_float(r[i >> 4][(2 * i) & 31]);
            float vb = __uint_as_float(r[i >> 4][(2 * i + 1) & 31]);
            if constexpr (kMasked) {
              const int k = h * 64 + 2 * i;
              if (k < lo || k > hi) va = -INFINITY;
              if (k + 1 < lo || k + 1 > hi) vb = -INFINITY;
            }
            mxa = fmaxf(mxa, va);
            mxb = fmaxf(mxb, vb);
            if constexpr (kWrite) {
              float ea, eb;
              f32x2_unpack(f32x2_fma(f32x2_pack(va, vb), sc2, nmu2), ea, eb);
              ea = fast_exp2(ea);
              eb = fast_exp2(eb);
              const uint64_t e2 = f32x2_pack(ea, eb);
              acc = f32x2_add(acc, e2);
              w[i] = pack_bf16x2(ea, eb);
            }
          }
          if constexpr (kWrite) tmem_st_32x32b_x32(p_row + h * 32, w);
        }
        if constexpr (kWrite) {
          float a0, a1;
          f32x2_unpack(acc, a0, a1);
          *rs = a0 + a1;
        }
        return fmaxf(mxa, mxb) * sc;
      };
      using T_ = std::true_type;
      using F_ = std::false_type;
      auto sweep_w = [&](float mu, float* rs) -> float {
        return masked ? sweep(T_{}, T_{}, mu, rs) : sweep(F_{}, T_{}, mu, rs);
      };
      // Rows without a finite running max yet (first tile) take this tile's
      // max first; afterwards exponentials reuse the running max and a tile
      // is redone only when its max exceeds it by more than 2^8.
      if (__any_sync(0xffffffffu, m_used == -INFINITY)) {
        const float mx = masked ? sweep(T_{}, F_{}, 0.f, nullptr) : sweep(F_{}, F_{}, 0.f, nullptr);
        if (m_used == -INFINITY) m_used = mx;
      }
      // P buffer pb is free once PV_{j-2} has completed.
      if (j >= 2) ok = mbar_wait(&p_free[pb], (uint32_t)(((j - 2) >> 1) & 1), p.err);
      if (stid == 0) FA_TLJ(j, 5);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      float rs = 0.f;
      float mx = sweep_w(m_used, &rs);
      const bool resc = mx > m_used + 8.f;
      if (__any_sync(0xffffffffu, resc)) {
        const float alpha = resc ? exp2f(m_used - mx) : 1.f;
        if (resc) {
          l *= alpha;
          m_used = mx;
        }
        if (j > 0) {
          // O (final once PV_{j-1} completes) *= alpha for this row.
          ok = __all_sync(0xffffffffu,
                          mbar_wait(&p_free[pb ^ 1], (uint32_t)(((j - 1) >> 1) & 1), p.err));
          if (!ok) break;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < FD / 32; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(tO + lane_base + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st_32x32b_x32(tO + lane_base + c * 32, o);
          }
        }
        tmem_wait_st();
        mx = sweep_w(m_used, &rs);  // redo P with the new max
      }
      l += rs;
      tmem_wait_st();
      // S buffer fully read, P and any O correction written.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sb]);
      if (j == n_tiles - 1 && kbase + FN > seq_len &&
          __all_sync(0xffffffffu, mbar_wait(&v_full[j % FNS], (uint32_t)((j / FNS) & 1), p.err))) {
        // Zero the V rows past the sequence end (stale cache-block contents).
        uint8_t* sv = sKV + (j % FNS) * kKVBytes + kKBytes;
        const int first_bad = max(0, seq_len - kbase);
        constexpr int kU = FD / 8;  // 16-byte units per key row
        for (int idx = stid; idx < (FN - first_bad) * kU; idx += 128) {
          const int key = first_bad + idx / kU, c16 = idx % kU;
          *reinterpret_cast<uint4*>(sv + (c16 >> 3) * kKVChunk + sw_off(key, c16 & 7)) =
              make_uint4(0, 0, 0, 0);
        }
        // Generic-proxy writes -> visible to the tensor core.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
      }
      if (lane == 0) mbar_arrive(&p_full[pb]);
      if (stid == 0) FA_TLJ(j, 6);
    }
    if (stid == 0) FA_TL(4);
    if (!ok) *abort_flag = 1;
    if (ok && n_tiles > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(o_done, 0, p.err));
      if (stid == 0) FA_TL(5);
      if (ok) {
        tc_fence_after();
        float denom = l;
        if (p.sinks != nullptr) {
          if (m_used == -INFINITY) denom = 1.f;
          else denom += exp2f(p.sinks[head] * 1.4426950408889634f - m_used);
        }
        const float inv = denom > 0.f ? 1.f / denom : 0.f;
        __nv_bfloat16* dst = p.out + (size_t)(q0 + t0 + t) * p.o_stride_t + (size_t)head * FD;
#pragma unroll 1
        for (int c = 0; c < FD / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tO + lane_base + c * 32, o);  // warp-collective: every lane
          tmem_wait_ld();
          if (valid_row) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[8 * v]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
              w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
              w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
              w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
              *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = w;
            }
          }
        }
      }
    }
  }
  if (threadIdx.x == 64) FA_TL(6);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemColsFa);
  }
  if (threadIdx.x == 0) FA_TL(7);
#undef FA_TL
#undef FA_TLJ
}

#include "attention/fa_tc_pp.cuh"

}  // namespace

void fa_tc_set_timeline(unsigned long long* buf) {
  cudaError_t e = cudaMemcpyToSymbol(g_fa_timeline, &buf, sizeof(buf));
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("fa_tc_set_timeline: ") + cudaGetErrorString(e));
}

bool fa_tc_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VLLM_B200_ATTN_PREFILL_TC");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}


bool fa_tc_supported(const AttnArgs& a) {
  const int G = a.Hkv > 0 ? a.Hq / a.Hkv : 0;
  if (a.head_dim != 128 && a.head_dim != 256) return false;
  const int FN = a.head_dim == 128 ? FaCfg<128>::FN : FaCfg<256>::FN;
  return !a.decode && a.num_blocks > 0 && G > 0 && FM % G == 0 && a.block_size >= 16 &&
         a.block_size <= FN && (FN % a.block_size) == 0 && a.q_stride_t % 8 == 0;
}

bool fa_pingpong_enabled();
int fa_exp2_split();

template <int D_>
void fa_tc_launch_d(const AttnArgs& a, cudaStream_t stream) {
  using Cfg = FaCfg<D_>;
  constexpr int FD = Cfg::FD;
  auto kernel = fa_tc_kernel<D_>;
  static bool attr[kMaxDevices] = {};
  set_smem_attr_once(kernel, Cfg::kSmem, attr, "fa_tc");
  const int G = a.Hq / a.Hkv;
  const int BS = a.block_size;
  const long long blk_stride = a.kv_block_stride > 0 ? a.kv_block_stride
                                                     : (long long)a.Hkv * BS * FD;
  // q [T][Hq][D] with token stride q_stride_t: box 64 d x G heads x 128/G tokens.
  CUtensorMap tq = make_tmap_3d(a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)a.num_tokens,
                                (uint64_t)a.Hq, FD, (uint64_t)FD * 2, (uint64_t)a.q_stride_t * 2,
                                (uint32_t)(FM / G), (uint32_t)G, 64);
  const uint64_t rows = (uint64_t)a.Hkv * BS;
  CUtensorMap tk = make_tmap_3d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                (uint64_t)a.num_blocks, rows, FD, (uint64_t)FD * 2,
                                (uint64_t)blk_stride * 2, 1, (uint32_t)BS, 64);
  CUtensorMap tv = make_tmap_3d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                (uint64_t)a.num_blocks, rows, FD, (uint64_t)FD * 2,
                                (uint64_t)blk_stride * 2, 1, (uint32_t)BS, 64);
  FaParams p{};
  p.block_table = a.block_table;
  p.seq_lens = a.seq_lens;
  p.cu_q = a.cu_q;
  p.sinks = a.sinks;
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.num_seqs = a.num_seqs;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.G = G;
  p.block_size = BS;
  p.block_shift = __builtin_ctz(BS);
  p.max_blocks = a.max_blocks;
  p.num_blocks = a.num_blocks;
  p.window = a.window;
  p.o_stride_t = a.o_stride_t;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  int dev = 0;
  cudaGetDevice(&dev);
  p.err = device_status_ptr(dev);
  // V as an MN-major B operand: the next 64-column block of V is a whole
  // FN-key chunk (FN x 128 bytes) away, the next group of 8 keys one
  // 1024-byte atom.
  p.v_lbo = (uint32_t)Cfg::kKVChunk;
  p.v_sbo = 1024u;
  if (D_ == 128 && fa_pingpong_enabled()) {
    // Two 128-row Q tiles per CTA (fa_tc_pp_kernel): Q boxes as above.
    const int max_qt2 = (a.max_q_len * G + 2 * FM - 1) / (2 * FM);
    if (max_qt2 <= 0 || a.num_seqs <= 0) return;
    const int split = fa_exp2_split();
    auto kpp = split == 2 ? fa_tc_pp_kernel<2> : split == 1 ? fa_tc_pp_kernel<1>
                                                           : fa_tc_pp_kernel<0>;
    static bool attr_pp[3][kMaxDevices] = {};
    set_smem_attr_once(kpp, kPpSmem, attr_pp[split], "fa_tc_pp");
    launch_pdl(kpp, dim3(max_qt2, a.num_seqs, a.Hkv), dim3(kPpThreads), kPpSmem, stream, nullptr,
               tq, tk, tv, p);
    return;
  }
  const int max_qt = (a.max_q_len * G + FM - 1) / FM;
  if (max_qt <= 0 || a.num_seqs <= 0) return;
  launch_pdl(kernel, dim3(max_qt, a.num_seqs, a.Hkv), dim3(kFaThreads), Cfg::kSmem, stream, nullptr,
             tq, tk, tv, p);
}

int fa_exp2_split() {
  static const int v = [] {
    const char* e = std::getenv("VLLM_B200_ATTN_EXP2_SPLIT");
    const int x = e ? std::atoi(e) : 1;  // measured best: a quarter on the FMA pipe
    return x < 0 ? 0 : (x > 2 ? 2 : x);
  }();
  return v;
}

bool fa_pingpong_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VLLM_B200_ATTN_PINGPONG");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

void fa_tc_launch(const AttnArgs& a, cudaStream_t stream) {
  if (a.head_dim == 256) fa_tc_launch_d<256>(a, stream);
  else fa_tc_launch_d<128>(a, stream);
}

}  // namespace b200
