// Paged flash attention over a block table (prefill, chunked prefill, decode,
// spec-verify), GQA-packed: one CTA serves one KV head of one sequence and
// packs (query token x query head of the group) into the MMA row dimension,
// so each K/V tile is read once for the whole GQA group.
//
//   q        [T, Hq, D]                       bf16 (RoPE already applied)
//   k_cache  [num_blocks, Hkv, BS, D]          bf16 (head-major inside a block:
//   v_cache  [num_blocks, Hkv, BS, D]          one (block, head) is BS*D contiguous)
//   block_table [num_seqs, max_blocks] int32, seq_lens [num_seqs] int32 (context
//   length including this step's tokens), cu_q [num_seqs + 1] int32.
//   Query token j of sequence s sits at absolute position seq_len - q_len + j and
//   attends keys [max(0, pos - window + 1), pos]. Optional per-head sink logits
//   join the softmax denominator.
//
// Prefill variant: 4 warps x 16 rows, K/V tiles of 64 keys shared through smem.
// Decode variant: 1 warp x 16 rows, tiles of 32 keys, the key range split over
// grid.z with a deterministic (index-order) combine kernel when splits > 1.
//
// Math on mma.sync.m16n8k16 (bf16 in, fp32 acc) with ldmatrix from XOR-swizzled
// smem; online softmax in base 2. The decode path is HBM-bound (K/V bytes), so
// the legacy MMA rate is not its limiter.
//
// Reference parity: Flash-V100 paged decode / prefill / verify
// (sm70/csrc/flash_v100/flash_decode_paged.cu:640-860,1421-1528,2061-2450;
// fused_mha_forward_paged.cu:357; verify_decode.cu:133-368), which uses
// m8n8k4/WMMA on sm_70 and an LBNHC cache; here the cache is [blk, Hkv, BS, D].
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "attention/attn_api.h"
#include "common/launch.h"
#include "common/ptx.cuh"
#include "common/tmap.h"
#include "ops_api.h"

namespace b200 {
namespace {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-byte chunk `ch` of row `r` in a swizzled tile whose rows
// hold D bf16 (D/8 chunks).
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int ch) {
  return (uint32_t)(r * (D * 2) + ((ch ^ (r & 7)) << 4));
}

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  __nv_bfloat16* out;
  const int* block_table;
  const int* seq_lens;
  const int* cu_q;
  const float* sinks;     // [Hq] or nullptr
  float* part_o;          // [splits, T, Hq, D] (decode split-KV) or nullptr
  float* part_ml;         // [splits, T, Hq, 2]
  int num_seqs, Hq, Hkv, block_size, block_shift, max_blocks, window;
  long long kv_block_stride;   // elements between consecutive cache blocks
  int q_stride_t, o_stride_t;  // element strides between tokens
  float scale_log2;            // softmax scale * log2(e)
  int num_splits;              // decode split-KV
  int rows_per_seq_max;        // max over seqs of q_len*G (grid sizing)
  int num_blocks;              // cache blocks (debug-build bounds checks)
};

constexpr int kBtCache = 512;  // block ids cached in smem per window

// Prefill (DECODE=false): NW warps, each owns 16 query rows; all warps walk
// every key of each shared K/V tile.
// Decode (DECODE=true): the CTA owns 16 rows (GQA group x query tokens); the
// NW warps split every K/V tile by keys (KT/NW each) and merge their softmax
// states in warp order at the end.
template <int D, int KT, int NW, int STAGES, bool DECODE>
__global__ void __launch_bounds__(NW * 32)
paged_attn_kernel(const Params p) {
  pdl_wait();
  pdl_trigger();
  constexpr int ROWS = DECODE ? 16 : 16 * NW;
  constexpr int KW = DECODE ? KT / NW : KT;  // keys per warp per tile
  static_assert(KW % 16 == 0, "keys per warp must be a multiple of 16");
  constexpr int CH = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  int* sBT = reinterpret_cast<int*>(smem + ROWS * D * 2);
  uint8_t* sKV = smem + ROWS * D * 2 + kBtCache * 4;  // STAGES x (K tile, V tile)
  constexpr int kTileBytes = KT * D * 2;

  const int seq = blockIdx.y;
  const int kvh = blockIdx.z % p.Hkv;
  const int split = DECODE ? blockIdx.z / p.Hkv : 0;
  const int G = p.Hq / p.Hkv;
  const int q0 = p.cu_q[seq];
  const int q_len = p.cu_q[seq + 1] - q0;
  const int seq_len = p.seq_lens[seq];
  const int rows_total = q_len * G;
  const int n_row_tiles = (rows_total + ROWS - 1) / ROWS;
  // Later row tiles carry more causal work: schedule them first.
  const int rt = DECODE ? blockIdx.x : (int)gridDim.x - 1 - (int)blockIdx.x;
  if (rt >= n_row_tiles || q_len == 0) return;
  const int row0 = rt * ROWS;

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;
  const int key_off = DECODE ? warp * KW : 0;
  const int warp_row0 = DECODE ? 0 : warp * 16;

  // Key range for this CTA.
  const int first_pos = seq_len - q_len + row0 / G;
  const int last_row = min(row0 + ROWS, rows_total) - 1;
  const int last_pos = seq_len - q_len + last_row / G;
  int k_begin = 0;
  if (p.window > 0) k_begin = max(0, first_pos - p.window + 1);
  int k_end = last_pos + 1;  // exclusive
  if (DECODE && p.num_splits > 1) {
    const int span = k_end - k_begin;
    const int per = ((span + p.num_splits - 1) / p.num_splits + KT - 1) / KT * KT;
    const int b = k_begin + split * per;
    const int e = min(k_end, b + per);
    k_begin = b;
    k_end = e;
  }
  k_begin = (k_begin / KT) * KT;
  const int n_tiles = k_end > k_begin ? (k_end - k_begin + KT - 1) / KT : 0;

  // ---- load Q rows (row r -> token r / G, head r % G) into smem
  for (int c = tid; c < ROWS * CH; c += NW * 32) {
    const int r = c / CH, ch = c % CH;
    const int gr = row0 + r;
    const bool valid = gr < rows_total;
    const int tok = valid ? gr / G : 0;
    const int h = kvh * G + (valid ? gr % G : 0);
    const __nv_bfloat16* src = p.q + (size_t)(q0 + tok) * p.q_stride_t + (size_t)h * D + ch * 8;
    cp_async_16(smem_addr(sQ) + swz<D>(r, ch), valid ? (const void*)src : (const void*)p.q, valid);
  }
  cp_async_commit();

  // Block ids of the key range, cached in smem window by window so the K/V
  // address computation never waits on a global load.
  const int* bt = p.block_table + (size_t)seq * p.max_blocks;
  const int blk_first = k_begin >> p.block_shift;
  const int blk_last = k_end > 0 ? (k_end - 1) >> p.block_shift : 0;
  int bt_base = -kBtCache;
  auto refill_bt = [&](int first_blk) {
    __syncthreads();
    for (int i = tid; i < kBtCache; i += NW * 32) {
      const int b = first_blk + i;
      sBT[i] = b <= blk_last ? __ldg(bt + b) : 0;
    }
    __syncthreads();
  };
  const long long head_off = (long long)kvh * p.block_size * D;
  auto load_tile = [&](int tile, int buf) {
    const int kbase = k_begin + tile * KT;
    const int kb_last = min(kbase + KT, k_end) - 1;
    if ((kb_last >> p.block_shift) >= bt_base + kBtCache) {  // uniform across the CTA
      bt_base = kbase >> p.block_shift;
      refill_bt(bt_base);
    }
    uint8_t* sK = sKV + buf * 2 * kTileBytes;
    uint8_t* sV = sK + kTileBytes;
#pragma unroll 4
    for (int c = tid; c < KT * CH; c += NW * 32) {
      const int r = c / CH, ch = c % CH;
      const int key = kbase + r;
      const bool valid = key < k_end;
      long long off = 0;
      if (valid) {
        const int blk = sBT[(key >> p.block_shift) - bt_base];
        off = (long long)blk * p.kv_block_stride + head_off +
              (long long)(key & (p.block_size - 1)) * D + ch * 8;
      }
      cp_async_16(smem_addr(sK) + swz<D>(r, ch), p.k_cache + off, valid);
      cp_async_16(smem_addr(sV) + swz<D>(r, ch), p.v_cache + off, valid);
    }
  };
  (void)blk_first;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < n_tiles) load_tile(s, s);
    cp_async_commit();
  }

  // Q fragments for this warp's 16 rows.
  cp_async_wait<STAGES - 1>();
  __syncthreads();
  uint32_t qf[D / 16][4];
  {
    const int r = warp_row0 + (lane % 8) + ((lane / 8) % 2) * 8;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int ch = kk * 2 + lane / 16;
      ldmatrix_x4(smem_addr(sQ) + swz<D>(r, ch), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }

  // Row bookkeeping: this thread holds rows (g) and (g + 8) of the warp tile.
  const int g = lane / 4, t4 = lane % 4;
  int row_pos[2];
  bool row_valid[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gr = row0 + warp_row0 + g + h * 8;
    row_valid[h] = gr < rows_total;
    row_pos[h] = seq_len - q_len + (row_valid[h] ? gr / G : 0);
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};

  for (int tile = 0; tile < n_tiles; ++tile) {
    const int buf = tile % STAGES;
    {
      const int nt = tile + STAGES - 1;
      if (nt < n_tiles) load_tile(nt, nt % STAGES);
      cp_async_commit();
    }
    cp_async_wait<STAGES - 1>();
    __syncthreads();
    const uint8_t* sK = sKV + buf * 2 * kTileBytes;
    const uint8_t* sV = sK + kTileBytes;
    const int kbase = k_begin + tile * KT + key_off;

    // S = Q K^T : 16 rows x KW keys per warp
    float s[KW / 8][4];
#pragma unroll
    for (int n = 0; n < KW / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int n2 = 0; n2 < KW / 16; ++n2) {
        const int key = key_off + n2 * 16 + (lane % 8) + (lane / 16) * 8;
        const int ch = kk * 2 + (lane / 8) % 2;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(smem_addr(sK) + swz<D>(key, ch), b0, b1, b2, b3);
        mma_bf16(s[2 * n2], qf[kk], b0, b1);
        mma_bf16(s[2 * n2 + 1], qf[kk], b2, b3);
      }
    }

    // Mask + online softmax (base 2).
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < KW / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e / 2;
        const int key = kbase + n * 8 + t4 * 2 + (e & 1);
        bool ok = row_valid[h] && key <= row_pos[h] && key < k_end;
        if (p.window > 0) ok = ok && key > row_pos[h] - p.window;
        const float v = ok ? s[n][e] * p.scale_log2 : -INFINITY;
        s[n][e] = v;
        mx[h] = fmaxf(mx[h], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 2));
      const float m_new = fmaxf(m_run[h], mx[h]);
      corr[h] = (m_new == -INFINITY) ? 1.f : exp2f(m_run[h] - m_new);
      m_run[h] = m_new;
      l_run[h] *= corr[h];
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    uint32_t pf[KW / 16][4];
#pragma unroll
    for (int n = 0; n < KW / 8; ++n) {
      float e4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e / 2;
        e4[e] = (m_run[h] == -INFINITY) ? 0.f : exp2f(s[n][e] - m_run[h]);
        l_run[h] += e4[e];
      }
      const int kk = n / 2, hi = n % 2;
      pf[kk][hi * 2 + 0] = pack2(e4[0], e4[1]);
      pf[kk][hi * 2 + 1] = pack2(e4[2], e4[3]);
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < KW / 16; ++kk) {
#pragma unroll
      for (int d2 = 0; d2 < D / 16; ++d2) {
        const int key = key_off + kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
        const int ch = d2 * 2 + lane / 16;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(smem_addr(sV) + swz<D>(key, ch), b0, b1, b2, b3);
        mma_bf16(o[2 * d2], pf[kk], b0, b1);
        mma_bf16(o[2 * d2 + 1], pf[kk], b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // Row sums across the 4 threads of a quad.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffff, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffff, l_run[h], 2);
  }

  if constexpr (DECODE && NW > 1) {
    // Merge the warps' partial softmax states in warp order through smem
    // (the K/V ring is idle now).
    __syncthreads();
    float* sO = reinterpret_cast<float*>(sKV);            // [NW][16][D]
    float* sM = sO + NW * 16 * D;                          // [NW][16]
    float* sL = sM + NW * 16;                              // [NW][16]
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g + h * 8;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        const int d = i * 8 + t4 * 2;
        sO[(warp * 16 + r) * D + d] = o[i][2 * h];
        sO[(warp * 16 + r) * D + d + 1] = o[i][2 * h + 1];
      }
      if (t4 == 0) {
        sM[warp * 16 + r] = m_run[h];
        sL[warp * 16 + r] = l_run[h];
      }
    }
    __syncthreads();
    for (int idx = tid; idx < 16 * D; idx += NW * 32) {
      const int r = idx / D, d = idx % D;
      const int gr = row0 + r;
      if (gr >= rows_total) continue;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NW; ++w) M = fmaxf(M, sM[w * 16 + r]);
      float L = 0.f, acc = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float mw = sM[w * 16 + r];
        const float sc = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
        L += sL[w * 16 + r] * sc;
        acc += sO[(w * 16 + r) * D + d] * sc;
      }
      const int tok = gr / G;
      const int head = kvh * G + gr % G;
      if (p.num_splits > 1) {
        const size_t T = (size_t)p.cu_q[p.num_seqs];
        const size_t base = ((size_t)split * T + (q0 + tok)) * p.Hq + head;
        p.part_o[base * D + d] = L > 0.f ? acc / L : 0.f;
        if (d == 0) {
          p.part_ml[base * 2 + 0] = M;
          p.part_ml[base * 2 + 1] = L;
        }
      } else {
        float denom = L;
        if (p.sinks != nullptr) {
          if (M == -INFINITY) denom = 1.f;
          else denom += exp2f(p.sinks[head] * 1.4426950408889634f - M);
        }
        const float inv = denom > 0.f ? 1.f / denom : 0.f;
        p.out[(size_t)(q0 + tok) * p.o_stride_t + (size_t)head * D + d] =
            __float2bfloat16_rn(acc * inv);
      }
    }
    return;
  }

#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (!row_valid[h]) continue;
    const int gr = row0 + warp_row0 + g + h * 8;
    const int tok = gr / G;
    const int head = kvh * G + gr % G;
    if (DECODE && p.num_splits > 1) {
      const size_t T = (size_t)p.cu_q[p.num_seqs];
      const size_t base = ((size_t)split * T + (q0 + tok)) * p.Hq + head;
      float* dst = p.part_o + base * D;
      const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        const int d = i * 8 + t4 * 2;
        *reinterpret_cast<float2*>(dst + d) = make_float2(o[i][2 * h] * inv, o[i][2 * h + 1] * inv);
      }
      if (t4 == 0) {
        p.part_ml[base * 2 + 0] = m_run[h];
        p.part_ml[base * 2 + 1] = l_run[h];
      }
    } else {
      float denom = l_run[h];
      if (p.sinks != nullptr) {
        const float sk = p.sinks[head] * 1.4426950408889634f;  // to base 2
        const float m = m_run[h];
        if (m == -INFINITY) {
          denom = 1.f;  // only the sink: output 0
        } else {
          denom += exp2f(sk - m);
        }
      }
      const float inv = denom > 0.f ? 1.f / denom : 0.f;
      __nv_bfloat16* dst = p.out + (size_t)(q0 + tok) * p.o_stride_t + (size_t)head * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        const int d = i * 8 + t4 * 2;
        *reinterpret_cast<uint32_t*>(dst + d) = pack2(o[i][2 * h] * inv, o[i][2 * h + 1] * inv);
      }
    }
  }
}

// Merge split-KV partials in split order (deterministic).
template <int D>
__global__ void combine_splits_kernel(const Params p, int T) {
  pdl_wait();
  pdl_trigger();
  const int tok = blockIdx.x;
  const int head = blockIdx.y;
  const int d = threadIdx.x;
  float m = -INFINITY;
  for (int s = 0; s < p.num_splits; ++s) {
    const size_t base = ((size_t)s * T + tok) * p.Hq + head;
    const float l = p.part_ml[base * 2 + 1];
    if (l > 0.f) m = fmaxf(m, p.part_ml[base * 2]);
  }
  float denom = 0.f;
  for (int s = 0; s < p.num_splits; ++s) {
    const size_t base = ((size_t)s * T + tok) * p.Hq + head;
    const float l = p.part_ml[base * 2 + 1];
    if (l > 0.f) denom += l * exp2f(p.part_ml[base * 2] - m);
  }
  if (p.sinks != nullptr && m != -INFINITY) denom += exp2f(p.sinks[head] * 1.4426950408889634f - m);
  const float inv = denom > 0.f ? 1.f / denom : 0.f;
  for (int dd = d; dd < D; dd += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < p.num_splits; ++s) {
      const size_t base = ((size_t)s * T + tok) * p.Hq + head;
      const float l = p.part_ml[base * 2 + 1];
      if (l > 0.f) acc += p.part_o[base * D + dd] * l * exp2f(p.part_ml[base * 2] - m);
    }
    p.out[(size_t)tok * p.o_stride_t + (size_t)head * D + dd] = __float2bfloat16_rn(acc * inv);
  }
}

// ---------------------------------------------------------------------------
// Decode / spec-verify on TMA. Four consumer warps do the math of the decode
// variant above (16 GQA-packed rows, each warp a quarter of every K/V tile,
// warp-order merge); a fifth warp streams the K/V tiles with 3-D tensor
// copies (box 64 columns x min(BS, KT) keys of one cache block, 128-byte
// swizzle) into a STAGES-deep mbarrier ring. The copies of one tile go out as
// one warp-wide instruction, a cache block (and column half, K or V) per
// lane: a bulk-tensor instruction costs its warp a few hundred ns however many
// lanes it carries, so per-block serial issue would cap the stream far below
// HBM rate. The consumers issue no load instructions at all, so their issue
// slots go to the MMAs and the softmax; tiles that need no mask skip the
// masking code, and O is rescaled only when a row's max grows by more than
// 2^8 over the max its exponentials use.
// Rows of a cache block past the sequence end hold stale data: their scores
// are masked by selection and each warp zeroes its V rows there before PV.
//
// Shared layout of a K (or V) tile: D/64 column halves of KT rows x 128 B,
// 16-byte chunk c of row r at (c ^ (r & 7)) within the row.
__device__ __forceinline__ uint32_t tma_tile_off(int r, int ch, int rows) {
  return (uint32_t)((ch >> 3) * rows * 128 + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

constexpr int kDecThreads = 160;

template <int D, int KT, int STAGES>
constexpr int decode_tma_smem() {
  return STAGES * 4 * KT * D + 16 * D * 2 + 2 * STAGES * 8 + 1024;
}

// CTAs per SM the shared-memory footprint allows (228 KB per SM, 1 KB
// reserved per CTA); the register budget is capped to match.
template <int D, int KT, int STAGES>
constexpr int decode_tma_ctas() {
  return (decode_tma_smem<D, KT, STAGES>() + 1024) * 3 <= 228 * 1024   ? 3
         : (decode_tma_smem<D, KT, STAGES>() + 1024) * 2 <= 228 * 1024 ? 2
                                                                         : 1;
}

template <int D, int KT, int STAGES>
__global__ void __launch_bounds__(kDecThreads, (decode_tma_ctas<D, KT, STAGES>()))
decode_tma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const Params p, unsigned int* err) {
  constexpr int NW = 4, ROWS = 16, KW = KT / NW, CH = D / 8, H = D / 64;
  constexpr int kTile = KT * D * 2;
  constexpr int kStage = 2 * kTile;
  static_assert(KW % 16 == 0, "keys per warp must be a multiple of 16");
  constexpr int DS = D + 8;  // merge row stride (floats): 8 rows of a warp hit distinct banks
  static_assert(STAGES * kStage >= (NW * 16 * DS + NW * 32) * 4, "merge buffer must fit the ring");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* ring = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = ring + STAGES * kStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(sQ + ROWS * D * 2);
  uint64_t* empty = full + STAGES;

  pdl_wait();
  pdl_trigger();
  const int seq = blockIdx.y;
  const int kvh = blockIdx.z % p.Hkv;
  const int split = blockIdx.z / p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int q0 = p.cu_q[seq];
  const int q_len = p.cu_q[seq + 1] - q0;
  const int seq_len = p.seq_lens[seq];
  const int rows_total = q_len * G;
  const int rt = blockIdx.x;
  if (rt * ROWS >= rows_total || q_len == 0) return;
  const int row0 = rt * ROWS;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

  const int first_pos = seq_len - q_len + row0 / G;
  const int last_row = min(row0 + ROWS, rows_total) - 1;
  const int last_pos = seq_len - q_len + last_row / G;
  int k_begin = p.window > 0 ? max(0, first_pos - p.window + 1) : 0;
  int k_end = last_pos + 1;
  if (p.num_splits > 1) {
    const int span = k_end - k_begin;
    const int per = ((span + p.num_splits - 1) / p.num_splits + KT - 1) / KT * KT;
    const int b = k_begin + split * per;
    k_end = min(k_end, b + per);
    k_begin = b;
  }
  k_begin = (k_begin / KT) * KT;
  const int n_tiles = k_end > k_begin ? (k_end - k_begin + KT - 1) / KT : 0;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_barrier_init();
  }
  // Q rows (row r -> token r / G, head r % G); padding rows are zero.
  for (int c = tid; c < ROWS * CH; c += kDecThreads) {
    const int r = c / CH, ch = c % CH;
    const int gr = row0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (gr < rows_total) {
      const int tok = gr / G, h = kvh * G + gr % G;
      v = *reinterpret_cast<const uint4*>(p.q + (size_t)(q0 + tok) * p.q_stride_t + (size_t)h * D +
                                          ch * 8);
    }
    *reinterpret_cast<uint4*>(sQ + swz<D>(r, ch)) = v;
  }
  __syncthreads();

  if (warp == NW) {
    // ------------------------------------------------------------ producer
    const int BS = p.block_size;
    const int nb = BS >= KT ? 1 : KT / BS;
    const int rows_box = BS >= KT ? KT : BS;
    const int nlanes = 2 * H * nb;
    const int* bt = p.block_table + (size_t)seq * p.max_blocks;
    const int blk_last = k_end > 0 ? (k_end - 1) >> p.block_shift : 0;
    auto blk_of = [&](int t) -> int {
      const int b = ((k_begin + t * KT) >> p.block_shift) + lane % nb;
      const int id = __ldg(bt + min(b, blk_last));
      return in_bounds(id >= 0 && id < p.num_blocks, err) ? id : 0;
    };
    int cur = n_tiles > 0 ? blk_of(0) : 0;
    for (int t = 0; t < n_tiles; ++t) {
      const int nxt = t + 1 < n_tiles ? blk_of(t + 1) : 0;  // ids one tile ahead
      const int st = t % STAGES;
      int ok = 1;
      if (lane == 0) {
        ok = mbar_wait(&empty[st], (uint32_t)(((t / STAGES) & 1) ^ 1), err) ? 1 : 0;
        if (ok) mbar_arrive_expect_tx(&full[st], (uint32_t)kStage);
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      const int kbase = k_begin + t * KT;
      const int y = kvh * BS + (BS > KT ? (kbase & (BS - 1)) : 0);
      uint8_t* stage = ring + st * kStage;
      for (int idx = lane; idx < nlanes; idx += 32) {
        const int kv = idx / (H * nb), h = (idx / nb) % H, i = idx % nb;
        tma_load_3d(stage + kv * kTile + h * KT * 128 + i * rows_box * 128, kv ? &tmv : &tmk,
                    &full[st], h * 64, y, cur);
      }
      cur = nxt;
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int key_off = warp * KW;
  // Q fragments stay in registers up to D = 128; wider heads (D = 256, whose
  // O accumulator alone takes 128 registers) re-read them from shared memory
  // for every K/V tile.
  constexpr bool kQReg = D <= 128;
  const int q_r = (lane % 8) + ((lane / 8) % 2) * 8;
  uint32_t qf[kQReg ? D / 16 : 1][4];
  if constexpr (kQReg) {
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int ch = kk * 2 + lane / 16;
      ldmatrix_x4(smem_addr(sQ) + swz<D>(q_r, ch), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }
  const int g = lane / 4, t4 = lane % 4;
  int row_pos[2];
  bool row_valid[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gr = row0 + g + h * 8;
    row_valid[h] = gr < rows_total;
    row_pos[h] = seq_len - q_len + (row_valid[h] ? gr / G : 0);
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};  // max the exponentials use
  float l_run[2] = {0.f, 0.f};

  bool ok = true;
  for (int tile = 0; tile < n_tiles; ++tile) {
    const int st = tile % STAGES;
    ok = mbar_wait(&full[st], (uint32_t)((tile / STAGES) & 1), err);
    if (!__all_sync(0xffffffffu, ok)) break;
    const uint32_t sK = smem_addr(ring + st * kStage);
    const uint32_t sV = sK + kTile;
    const int kbase = k_begin + tile * KT + key_off;
    if (kbase + KW > k_end) {
      // This warp's rows past the range end: zero V (stale cache rows).
      uint8_t* v = ring + st * kStage + kTile;
      for (int c = lane; c < KW * CH; c += 32) {
        const int r = key_off + c / CH;
        if (k_begin + tile * KT + r >= k_end)
          *reinterpret_cast<uint4*>(v + tma_tile_off(r, c % CH, KT)) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }

    float s[KW / 8][4];
#pragma unroll
    for (int n = 0; n < KW / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t qa[4];
      if constexpr (kQReg) {
        qa[0] = qf[kk][0]; qa[1] = qf[kk][1]; qa[2] = qf[kk][2]; qa[3] = qf[kk][3];
      } else {
        ldmatrix_x4(smem_addr(sQ) + swz<D>(q_r, kk * 2 + lane / 16), qa[0], qa[1], qa[2], qa[3]);
      }
#pragma unroll
      for (int n2 = 0; n2 < KW / 16; ++n2) {
        const int key = key_off + n2 * 16 + (lane % 8) + (lane / 16) * 8;
        const int ch = kk * 2 + (lane / 8) % 2;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(sK + tma_tile_off(key, ch, KT), b0, b1, b2, b3);
        mma_bf16(s[2 * n2], qa, b0, b1);
        mma_bf16(s[2 * n2 + 1], qa, b2, b3);
      }
    }

    // Every key of this warp's slice visible to every row?
    const bool need_mask = kbase + KW - 1 > first_pos || kbase + KW > k_end ||
                           (p.window > 0 && kbase <= last_pos - p.window);
    float mx[2] = {-INFINITY, -INFINITY};
    if (need_mask) {
#pragma unroll
      for (int n = 0; n < KW / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = e / 2;
          const int key = kbase + n * 8 + t4 * 2 + (e & 1);
          bool in = row_valid[h] && key <= row_pos[h] && key < k_end;
          if (p.window > 0) in = in && key > row_pos[h] - p.window;
          s[n][e] = in ? s[n][e] * p.scale_log2 : -INFINITY;
          mx[h] = fmaxf(mx[h], s[n][e]);
        }
      }
    } else {
#pragma unroll
      for (int n = 0; n < KW / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[n][e] *= p.scale_log2;
          mx[e / 2] = fmaxf(mx[e / 2], s[n][e]);
        }
      }
    }
    bool resc = false;
    float corr[2] = {1.f, 1.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 2));
      if (mx[h] > m_run[h] + 8.f) {  // also the first finite max (m_run = -inf)
        corr[h] = exp2f(m_run[h] - mx[h]);
        m_run[h] = mx[h];
        l_run[h] *= corr[h];
        resc = true;
      }
    }
    if (__any_sync(0xffffffffu, resc)) {
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][0] *= corr[0];
        o[i][1] *= corr[0];
        o[i][2] *= corr[1];
        o[i][3] *= corr[1];
      }
    }
    const float mu0 = m_run[0] == -INFINITY ? 0.f : m_run[0];
    const float mu1 = m_run[1] == -INFINITY ? 0.f : m_run[1];
    uint32_t pf[KW / 16][4];
#pragma unroll
    for (int n = 0; n < KW / 8; ++n) {
      const float e0 = exp2f(s[n][0] - mu0), e1 = exp2f(s[n][1] - mu0);
      const float e2 = exp2f(s[n][2] - mu1), e3 = exp2f(s[n][3] - mu1);
      l_run[0] += e0 + e1;
      l_run[1] += e2 + e3;
      const int kk = n / 2, hi = n % 2;
      pf[kk][hi * 2 + 0] = pack2(e0, e1);
      pf[kk][hi * 2 + 1] = pack2(e2, e3);
    }
#pragma unroll
    for (int kk = 0; kk < KW / 16; ++kk) {
#pragma unroll
      for (int d2 = 0; d2 < D / 16; ++d2) {
        const int key = key_off + kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
        const int ch = d2 * 2 + lane / 16;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(sV + tma_tile_off(key, ch, KT), b0, b1, b2, b3);
        mma_bf16(o[2 * d2], pf[kk], b0, b1);
        mma_bf16(o[2 * d2 + 1], pf[kk], b2, b3);
      }
    }
    // Generic-proxy reads (and any zeroing) done before the TMA refills.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }

#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffff, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffff, l_run[h], 2);
  }
  // Warp-order merge through the (now idle) ring; consumer warps only.
  named_barrier_sync(1, NW * 32);
  float* sO = reinterpret_cast<float*>(ring);  // [NW][16][DS]
  float* sM = sO + NW * 16 * DS;                // [NW][16]
  float* sL = sM + NW * 16;                     // [NW][16]
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g + h * 8;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int d = i * 8 + t4 * 2;
      *reinterpret_cast<float2*>(&sO[(warp * 16 + r) * DS + d]) = make_float2(o[i][2 * h], o[i][2 * h + 1]);
    }
    if (t4 == 0) {
      sM[warp * 16 + r] = m_run[h];
      sL[warp * 16 + r] = l_run[h];
    }
  }
  named_barrier_sync(1, NW * 32);
  for (int idx = tid; idx < 16 * D; idx += NW * 32) {
    const int r = idx / D, d = idx % D;
    const int gr = row0 + r;
    if (gr >= rows_total) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sM[w * 16 + r]);
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float mw = sM[w * 16 + r];
      const float sc = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      L += sL[w * 16 + r] * sc;
      acc += sO[(w * 16 + r) * DS + d] * sc;
    }
    const int tok = gr / G;
    const int head = kvh * G + gr % G;
    if (p.num_splits > 1) {
      const size_t T = (size_t)p.cu_q[p.num_seqs];
      const size_t base = ((size_t)split * T + (q0 + tok)) * p.Hq + head;
      p.part_o[base * D + d] = L > 0.f ? acc / L : 0.f;
      if (d == 0) {
        p.part_ml[base * 2 + 0] = L > 0.f ? M : -INFINITY;
        p.part_ml[base * 2 + 1] = L;
      }
    } else {
      float denom = L;
      if (p.sinks != nullptr) {
        if (M == -INFINITY || L == 0.f) denom = 1.f;
        else denom += exp2f(p.sinks[head] * 1.4426950408889634f - M);
      }
      const float inv = denom > 0.f ? 1.f / denom : 0.f;
      p.out[(size_t)(q0 + tok) * p.o_stride_t + (size_t)head * D + d] = __float2bfloat16_rn(acc * inv);
    }
  }
}

template <int D, int KT, int STAGES>
void launch_decode_tma(const Params& p, const AttnArgs& a, cudaStream_t stream) {
  constexpr int smem = decode_tma_smem<D, KT, STAGES>();
  auto kernel = decode_tma_kernel<D, KT, STAGES>;
  static bool attr[kMaxDevices] = {};
  set_smem_attr_once(kernel, smem, attr, "decode_tma");
  const int BS = a.block_size;
  const uint32_t rows_box = (uint32_t)(BS >= KT ? KT : BS);
  const uint64_t rows = (uint64_t)a.Hkv * BS;
  const uint64_t bstride = (uint64_t)p.kv_block_stride * 2;
  CUtensorMap tk = make_tmap_3d(a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                (uint64_t)a.num_blocks, rows, D, (uint64_t)D * 2, bstride, 1,
                                rows_box, 64);
  CUtensorMap tv = make_tmap_3d(a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                (uint64_t)a.num_blocks, rows, D, (uint64_t)D * 2, bstride, 1,
                                rows_box, 64);
  int dev = 0;
  cudaGetDevice(&dev);
  const int row_tiles = (p.rows_per_seq_max + 15) / 16;
  dim3 grid(row_tiles, p.num_seqs, p.Hkv * p.num_splits);
  launch_pdl(kernel, grid, dim3(kDecThreads), smem, stream, nullptr, tk, tv, p,
             device_status_ptr(dev));
}

bool decode_tma_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VLLM_B200_ATTN_DECODE_TMA");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

template <int D, int KT, int NW, int STAGES, bool DECODE>
void launch_attn(const Params& p, cudaStream_t stream) {
  constexpr int ROWS = DECODE ? 16 : 16 * NW;
  constexpr int smem = ROWS * D * 2 + kBtCache * 4 + STAGES * 2 * KT * D * 2;
  static_assert(!DECODE || STAGES * 2 * KT * D * 2 >= (NW * 16 * D + NW * 32) * 4,
                "decode merge buffer must fit in the K/V ring");
  auto kernel = paged_attn_kernel<D, KT, NW, STAGES, DECODE>;
  static bool attr[kMaxDevices] = {};
  set_smem_attr_once(kernel, smem, attr, "paged_attn");
  const int row_tiles = (p.rows_per_seq_max + ROWS - 1) / ROWS;
  dim3 grid(row_tiles, p.num_seqs, p.Hkv * (DECODE ? p.num_splits : 1));
  launch_pdl(kernel, grid, dim3(NW * 32), smem, stream, nullptr, p);
}

}  // namespace

void paged_attention_launch(const AttnArgs& a, cudaStream_t stream) {
  if (a.Hq % a.Hkv != 0) throw std::runtime_error("paged_attention: Hq % Hkv != 0");
  if (a.block_size < 8 || (a.block_size & (a.block_size - 1)) != 0)
    throw std::runtime_error("paged_attention: block_size must be a power of two >= 8");
  Params p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(a.q);
  p.k_cache = reinterpret_cast<const __nv_bfloat16*>(a.k_cache);
  p.v_cache = reinterpret_cast<const __nv_bfloat16*>(a.v_cache);
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.block_table = a.block_table;
  p.seq_lens = a.seq_lens;
  p.cu_q = a.cu_q;
  p.sinks = a.sinks;
  p.part_o = a.part_o;
  p.part_ml = a.part_ml;
  p.num_seqs = a.num_seqs;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.block_size = a.block_size;
  p.block_shift = __builtin_ctz(a.block_size);
  p.kv_block_stride = a.kv_block_stride > 0 ? a.kv_block_stride
                                            : (long long)a.Hkv * a.block_size * a.head_dim;
  p.max_blocks = a.max_blocks;
  p.window = a.window;
  p.q_stride_t = a.q_stride_t;
  p.o_stride_t = a.o_stride_t;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.num_splits = a.decode ? (a.num_splits > 0 ? a.num_splits : 1) : 1;
  p.rows_per_seq_max = a.max_q_len * (a.Hq / a.Hkv);
  p.num_blocks = a.num_blocks;
  if (p.num_splits > 1 && (a.part_o == nullptr || a.part_ml == nullptr))
    throw std::runtime_error("paged_attention: split-KV needs partial buffers");
  const bool tma_ok = a.num_blocks > 0 && a.block_size >= 8 && a.q_stride_t % 8 == 0 &&
                      p.kv_block_stride % 8 == 0 &&
                      (reinterpret_cast<uintptr_t>(a.k_cache) & 15u) == 0 &&
                      (reinterpret_cast<uintptr_t>(a.v_cache) & 15u) == 0;
  if (!a.decode && fa_tc_enabled() && fa_tc_supported(a)) {
    fa_tc_launch(a, stream);
  } else if (a.decode && tma_ok && decode_tma_enabled() &&
             (a.head_dim == 128 || a.head_dim == 64 || a.head_dim == 256)) {
    // Two 64-key stages per CTA and three CTAs per SM measured faster than
    // three stages at two CTAs per SM (more consumer warps per SM keep the
    // same bytes in flight). D = 256: one CTA per SM with three 64-key stages
    // (192 KB of K/V in flight per SM).
    if (a.head_dim == 128)
      launch_decode_tma<128, 64, 2>(p, a, stream);
    else if (a.head_dim == 256)
      launch_decode_tma<256, 64, 3>(p, a, stream);
    else
      launch_decode_tma<64, 64, 4>(p, a, stream);
  } else if (a.head_dim == 128) {
    if (a.decode)
      launch_attn<128, 64, 4, 3, true>(p, stream);
    else
      launch_attn<128, 64, 4, 2, false>(p, stream);
  } else if (a.head_dim == 256) {
    if (a.decode)
      launch_attn<256, 64, 4, 2, true>(p, stream);
    else
      launch_attn<256, 32, 4, 2, false>(p, stream);
  } else if (a.head_dim == 64) {
    if (a.decode)
      launch_attn<64, 64, 4, 3, true>(p, stream);
    else
      launch_attn<64, 64, 4, 2, false>(p, stream);
  } else {
    throw std::runtime_error("paged_attention: head_dim must be 64, 128 or 256");
  }
  if (p.num_splits > 1) {
    dim3 grid(a.num_tokens, a.Hq);
    if (a.head_dim == 128)
      launch_pdl(combine_splits_kernel<128>, grid, dim3(128), 0, stream, nullptr, p, a.num_tokens);
    else if (a.head_dim == 256)
      launch_pdl(combine_splits_kernel<256>, grid, dim3(128), 0, stream, nullptr, p, a.num_tokens);
    else
      launch_pdl(combine_splits_kernel<64>, grid, dim3(64), 0, stream, nullptr, p, a.num_tokens);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("paged_attention launch: ") + cudaGetErrorString(e));
}

}  // namespace b200
