// Chunked gated-DeltaNet prefill (the WY / UT form of the gated delta rule),
// chunks of 64 tokens, all matrix products on the tensor cores.
//
// Recurrence (per v-head, state S [DV, DK], token t with L2-normalised k_t,
// q_t (q scaled by DK^-1/2), log-decay g_t <= 0 and beta_t):
//   S_t = exp(g_t) S_{t-1} (I - beta_t k_t k_t^T) + beta_t v_t k_t^T,  o_t = S_t q_t
// Within a chunk, with cumulative log-decay G_i (G_i = g_1 + ... + g_i) and
// the chunk's initial state S0, the new values nu_t = beta_t (v_t - exp(g_t)
// S_{t-1} k_t) solve the unit lower-triangular system
//   (I + A) N = diag(beta) V - diag(beta exp(G)) K S0^T,
//   A_ij = beta_i exp(G_i - G_j) k_i . k_j  (j < i)
// so with T = (I + A)^-1:  U = T diag(beta) V,  W = T diag(beta exp(G)) K,
//   N = U - W S0^T
//   O = diag(exp(G)) Q S0^T + ((Q K^T) o exp(G_i - G_j) [j <= i]) N
//   S_L = exp(G_L) S0 + N^T diag(exp(G_L - G)) K
// (the derivation unrolls the recurrence over the chunk; it is exact up to
// rounding). T is found by forward substitution in fp32; every product runs
// on mma.sync m16n8k16 (bf16 operands, fp32 accumulators). The state stays in
// fp32 registers across chunks: warp w owns rows [32w, 32w + 32) of S, and
// its accumulator fragments double as the B operand of W S0^T and Q S0^T
// (the fragment layouts coincide), so S never goes through shared memory.
//
// One CTA (4 warps) per (sequence, v-head), chunks in order; decode and
// speculative verify keep the token-serial kernel (gdn.cu), whose state
// semantics (slots, reset, write_state) this kernel shares.
//
// Reference parity: FlashQLA GDN prefill (sm70/csrc/gdn/gdn_forward.cu:90-237)
// is token-serial; the chunked form is the standard gated-delta-rule
// chunking (FLA chunk_gated_delta_rule semantics, g/beta gating identical to
// the recurrent kernel here).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>

#include "common/launch.h"
#include "gdn/gdn_api.h"

namespace b200 {
namespace {

constexpr int kC = 64;       // chunk length
constexpr int kD = 128;      // DK = DV
constexpr int kSD = kD + 8;  // padded row stride (bf16) of [64][128] tiles: 272 B
constexpr int kSC = kC + 8;  // padded row stride (bf16) of [64][64] tiles: 144 B
constexpr int kSA = kC + 1;  // fp32 [64][64] stride

// Shared layout (bytes).
constexpr int kOffK = 0;                       // Kn  [64][kSD] bf16
constexpr int kOffQ = kOffK + kC * kSD * 2;    // Qn  [64][kSD] bf16
constexpr int kOffV = kOffQ + kC * kSD * 2;    // V, later N [64][kSD] bf16
constexpr int kOffA = kOffV + kC * kSD * 2;    // A / T fp32 [64][kSA], later W [64][kSD] bf16
constexpr int kSizeA = (kC * kSA * 4 > kC * kSD * 2) ? kC * kSA * 4 : kC * kSD * 2;
constexpr int kOffT1 = kOffA + (kSizeA + 15) / 16 * 16;  // T diag(beta), later P [64][kSC] bf16
constexpr int kOffT2 = kOffT1 + kC * kSC * 2;            // T diag(beta exp G) [64][kSC] bf16
constexpr int kOffG = kOffT2 + kC * kSC * 2;             // G [64] fp32
constexpr int kOffB = kOffG + kC * 4;                    // beta [64] fp32
constexpr int kSmem = kOffB + kC * 4;

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                    uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pk(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 upk(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}
__device__ __forceinline__ float bfv(__nv_bfloat16 x) { return __bfloat162float(x); }

// A fragment (16 x 16) of a row-major bf16 tile: rows r0.., cols c0.. (stride in elements).
__device__ __forceinline__ void lda(uint32_t base, int stride, int r0, int c0, int lane,
                                    uint32_t (&a)[4]) {
  const int r = r0 + (lane & 7) + ((lane >> 3) & 1) * 8, c = c0 + (lane >> 4) * 8;
  ldsm4(base + (uint32_t)((r * stride + c) * 2), a);
}
// A fragment (16 x 16) of the TRANSPOSE of a row-major tile X: A[m][k] = X[k][m],
// m in [m0, m0+16), k in [k0, k0+16).
__device__ __forceinline__ void lda_t(uint32_t base, int stride, int m0, int k0, int lane,
                                      uint32_t (&a)[4]) {
  const int k = k0 + (lane & 7) + (lane >> 4) * 8, m = m0 + ((lane >> 3) & 1) * 8;
  ldsm4t(base + (uint32_t)((k * stride + m) * 2), a);
}
// B fragments of two n8 tiles from a tile stored [n][k] (row n contiguous over k):
// b[0], b[1] for n in [n0, n0+8), b[2], b[3] for [n0+8, n0+16); k in [k0, k0+16).
__device__ __forceinline__ void ldb_nk(uint32_t base, int stride, int n0, int k0, int lane,
                                       uint32_t (&b)[4]) {
  const int n = n0 + (lane & 7) + (lane >> 4) * 8, k = k0 + ((lane >> 3) & 1) * 8;
  ldsm4(base + (uint32_t)((n * stride + k) * 2), b);
}
// Same from a tile stored [k][n] (row k contiguous over n).
__device__ __forceinline__ void ldb_kn(uint32_t base, int stride, int n0, int k0, int lane,
                                       uint32_t (&b)[4]) {
  const int k = k0 + (lane & 7) + ((lane >> 3) & 1) * 8, n = n0 + (lane >> 4) * 8;
  ldsm4t(base + (uint32_t)((k * stride + n) * 2), b);
}

__global__ void __launch_bounds__(128, 2) gdn_chunk_kernel(const GdnParams p) {
  pdl_wait();
  extern __shared__ __align__(16) uint8_t sm[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(sm + kOffK);
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(sm + kOffQ);
  __nv_bfloat16* sV = reinterpret_cast<__nv_bfloat16*>(sm + kOffV);  // V, then N
  float* sA = reinterpret_cast<float*>(sm + kOffA);                    // A / T
  __nv_bfloat16* sW = reinterpret_cast<__nv_bfloat16*>(sm + kOffA);   // W (after T)
  __nv_bfloat16* sT1 = reinterpret_cast<__nv_bfloat16*>(sm + kOffT1); // T diag(b), then P
  __nv_bfloat16* sT2 = reinterpret_cast<__nv_bfloat16*>(sm + kOffT2); // T diag(b e^G)
  float* sG = reinterpret_cast<float*>(sm + kOffG);
  float* sB = reinterpret_cast<float*>(sm + kOffB);
  const uint32_t aK = saddr(sK), aQ = saddr(sQ), aV = saddr(sV), aW = saddr(sW),
                 aT1 = saddr(sT1), aT2 = saddr(sT2);

  const int s = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int hk = h / (p.HV / p.HK);
  const int t0 = p.cu[s], t1 = p.cu[s + 1];
  const int slot = p.slots[s];
  const float A_h = -__expf(p.A_log[h]);
  const float dtb = p.dt_bias[h];
  const float qscale = rsqrtf((float)kD);

  // State rows [32 warp, +32): S[mt][nt][4] in C-fragment layout
  // (row = 32 warp + 16 mt + g8 (+8), col = 8 nt + 2 t4 (+1)).
  float S[2][16][4];
  const size_t lds = p.ld_state ? (size_t)p.ld_state : (size_t)p.HV * kD * kD;
  float* gst = slot >= 0 ? p.state + (size_t)slot * lds + (size_t)h * kD * kD : nullptr;
  const bool fresh = p.reset_state || (p.has_init != nullptr && p.has_init[s] == 0);
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int r = warp * 32 + mt * 16 + g8, c = nt * 8 + 2 * t4;
      if (gst != nullptr && !fresh) {
        const float2 lo = *reinterpret_cast<const float2*>(gst + (size_t)r * kD + c);
        const float2 hi = *reinterpret_cast<const float2*>(gst + (size_t)(r + 8) * kD + c);
        S[mt][nt][0] = lo.x; S[mt][nt][1] = lo.y; S[mt][nt][2] = hi.x; S[mt][nt][3] = hi.y;
      } else {
        S[mt][nt][0] = S[mt][nt][1] = S[mt][nt][2] = S[mt][nt][3] = 0.f;
      }
    }

  for (int c0 = t0; c0 < t1; c0 += kC) {
    const int L = min(kC, t1 - c0);
    // ---- 1. chunk inputs: normalised k, q; v; log-decay and beta.
    for (int i = warp; i < kC; i += 4) {
      const int t = c0 + i;
      float kv[4] = {0.f, 0.f, 0.f, 0.f}, qv[4] = {0.f, 0.f, 0.f, 0.f}, vv[4] = {0.f, 0.f, 0.f, 0.f};
      if (i < L) {
        const uint2 kr = *reinterpret_cast<const uint2*>(p.k + (size_t)t * p.ldk + hk * kD + lane * 4);
        const uint2 qr = *reinterpret_cast<const uint2*>(p.q + (size_t)t * p.ldq + hk * kD + lane * 4);
        const uint2 vr = *reinterpret_cast<const uint2*>(p.v + (size_t)t * p.ldv + h * kD + lane * 4);
        float2 f;
        f = upk(kr.x); kv[0] = f.x; kv[1] = f.y; f = upk(kr.y); kv[2] = f.x; kv[3] = f.y;
        f = upk(qr.x); qv[0] = f.x; qv[1] = f.y; f = upk(qr.y); qv[2] = f.x; qv[3] = f.y;
        f = upk(vr.x); vv[0] = f.x; vv[1] = f.y; f = upk(vr.y); vv[2] = f.x; vv[3] = f.y;
      }
      float nk = kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3];
      float nq = qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        nk += __shfl_xor_sync(0xffffffffu, nk, o);
        nq += __shfl_xor_sync(0xffffffffu, nq, o);
      }
      const float ik = rsqrtf(nk + 1e-6f), iq = rsqrtf(nq + 1e-6f) * qscale;
      uint2 w;
      w.x = pk(kv[0] * ik, kv[1] * ik); w.y = pk(kv[2] * ik, kv[3] * ik);
      *reinterpret_cast<uint2*>(sK + i * kSD + lane * 4) = w;
      w.x = pk(qv[0] * iq, qv[1] * iq); w.y = pk(qv[2] * iq, qv[3] * iq);
      *reinterpret_cast<uint2*>(sQ + i * kSD + lane * 4) = w;
      w.x = pk(vv[0], vv[1]); w.y = pk(vv[2], vv[3]);
      *reinterpret_cast<uint2*>(sV + i * kSD + lane * 4) = w;
      if (lane == 0) {
        float gl = 0.f, beta = 0.f;
        if (i < L) {
          const float x = bfv(p.a[(size_t)t * p.ldab + h]) + dtb;
          const float sp = x > 20.f ? x : log1pf(__expf(x));
          gl = A_h * sp;
          beta = 1.f / (1.f + __expf(-bfv(p.b[(size_t)t * p.ldab + h])));
        }
        sG[i] = gl;
        sB[i] = beta;
      }
    }
    __syncthreads();
    // ---- 2. cumulative log-decay G (warp 0 scan, 2 tokens per lane).
    if (warp == 0) {
      float a0 = sG[2 * lane], a1 = sG[2 * lane + 1];
      float incl = a0 + a1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const float excl = incl - (a0 + a1);
      sG[2 * lane] = excl + a0;
      sG[2 * lane + 1] = excl + a0 + a1;
    }
    __syncthreads();
    // ---- 3. A_ij = beta_i exp(G_i - G_j) k_i.k_j (j < i), rows [16 warp, +16).
    {
      float acc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        uint32_t a[4];
        lda(aK, kSD, warp * 16, kk * 16, lane, a);
#pragma unroll
        for (int n2 = 0; n2 < 4; ++n2) {
          uint32_t b[4];
          ldb_nk(aK, kSD, n2 * 16, kk * 16, lane, b);
          mma(acc[2 * n2], a, b[0], b[1]);
          mma(acc[2 * n2 + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = warp * 16 + g8 + (e >> 1) * 8, j = n * 8 + 2 * t4 + (e & 1);
          sA[i * kSA + j] = j < i ? sB[i] * __expf(sG[i] - sG[j]) * acc[n][e] : (j == i ? 1.f : 0.f);
        }
    }
    __syncthreads();
    // ---- 4. T = (I + A)^-1 (unit lower triangular, in place over sA = I + A),
    //         by 16 x 16 blocks: the diagonal blocks by forward substitution,
    //         one warp each; then block rows 1..3 in order,
    //         T_ij = -T_ii sum_{j <= m < i} L_im T_mj  (j < i).
    {
      // (a) diagonal block b = warp: rows [16b, 16b + 16); lane c < 16 owns column c.
      const int b0 = warp * 16;
      for (int r = 1; r < 16; ++r) {
        float t = 0.f;
        if (lane < r) {
          float acc = sA[(b0 + r) * kSA + b0 + lane];  // m = c term (T_cc = 1)
          for (int m = lane + 1; m < r; ++m)
            acc += sA[(b0 + r) * kSA + b0 + m] * sA[(b0 + m) * kSA + b0 + lane];
          t = -acc;
        }
        __syncwarp();
        if (lane < r) sA[(b0 + r) * kSA + b0 + lane] = t;
        __syncwarp();
      }
      __syncthreads();
      // (b) off-diagonal block rows.
      float* X = reinterpret_cast<float*>(sm + kOffT1);  // [3][16][16] scratch
      for (int i = 1; i < 4; ++i) {
        for (int idx = tid; idx < i * 256; idx += 128) {
          const int j = idx >> 8, r = (idx >> 4) & 15, c = idx & 15;
          float acc = 0.f;
          for (int m = 16 * j; m < 16 * i; ++m)
            acc += sA[(16 * i + r) * kSA + m] * sA[m * kSA + 16 * j + c];
          X[idx] = acc;
        }
        __syncthreads();
        for (int idx = tid; idx < i * 256; idx += 128) {
          const int j = idx >> 8, r = (idx >> 4) & 15, c = idx & 15;
          float acc = 0.f;
          for (int m = 0; m <= r; ++m)
            acc += sA[(16 * i + r) * kSA + 16 * i + m] * X[(j << 8) + (m << 4) + c];
          sA[(16 * i + r) * kSA + 16 * j + c] = -acc;
        }
        __syncthreads();
      }
    }
    // T diag(beta) and T diag(beta exp(G)) in bf16 (T_ij = 0 for j > i).
    for (int idx = tid; idx < kC * kC; idx += 128) {
      const int i = idx >> 6, j = idx & 63;
      const float t = j <= i ? sA[i * kSA + j] : 0.f;
      sT1[i * kSC + j] = __float2bfloat16_rn(t * sB[j]);
      sT2[i * kSC + j] = __float2bfloat16_rn(t * sB[j] * __expf(sG[j]));
    }
    __syncthreads();
    // ---- 5. W[:, 32 warp ..] = T2 K -> smem (over T, read only before the last
    //         sync); then U[:, 32 warp ..] = T1 V -> registers.
    {
      float Wf[4][4][4];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int n = 0; n < 4; ++n) Wf[mt][n][0] = Wf[mt][n][1] = Wf[mt][n][2] = Wf[mt][n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kC / 16; ++kk) {
        uint32_t bk[2][4];
#pragma unroll
        for (int n2 = 0; n2 < 2; ++n2) ldb_kn(aK, kSD, warp * 32 + n2 * 16, kk * 16, lane, bk[n2]);
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          uint32_t a2[4];
          lda(aT2, kSC, mt * 16, kk * 16, lane, a2);
#pragma unroll
          for (int n2 = 0; n2 < 2; ++n2) {
            mma(Wf[mt][2 * n2], a2, bk[n2][0], bk[n2][1]);
            mma(Wf[mt][2 * n2 + 1], a2, bk[n2][2], bk[n2][3]);
          }
        }
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int r = mt * 16 + g8, c = warp * 32 + n * 8 + 2 * t4;
          *reinterpret_cast<uint32_t*>(sW + r * kSD + c) = pk(Wf[mt][n][0], Wf[mt][n][1]);
          *reinterpret_cast<uint32_t*>(sW + (r + 8) * kSD + c) = pk(Wf[mt][n][2], Wf[mt][n][3]);
        }
    }
    float U[4][4][4];
#pragma unroll
    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
      for (int n = 0; n < 4; ++n) U[mt][n][0] = U[mt][n][1] = U[mt][n][2] = U[mt][n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kC / 16; ++kk) {
      uint32_t bv[2][4];
#pragma unroll
      for (int n2 = 0; n2 < 2; ++n2) ldb_kn(aV, kSD, warp * 32 + n2 * 16, kk * 16, lane, bv[n2]);
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t a1[4];
        lda(aT1, kSC, mt * 16, kk * 16, lane, a1);
#pragma unroll
        for (int n2 = 0; n2 < 2; ++n2) {
          mma(U[mt][2 * n2], a1, bv[n2][0], bv[n2][1]);
          mma(U[mt][2 * n2 + 1], a1, bv[n2][2], bv[n2][3]);
        }
      }
    }
    __syncthreads();
    // ---- 6. N[:, 32 warp ..] = U - W S0^T (B fragments straight from the state).
#pragma unroll
    for (int kk = 0; kk < kD / 16; ++kk) {
      uint32_t b[2][2][2];  // [mt of S][half g8 / g8+8][b0, b1]
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        b[mt][0][0] = pk(S[mt][2 * kk][0], S[mt][2 * kk][1]);
        b[mt][0][1] = pk(S[mt][2 * kk + 1][0], S[mt][2 * kk + 1][1]);
        b[mt][1][0] = pk(S[mt][2 * kk][2], S[mt][2 * kk][3]);
        b[mt][1][1] = pk(S[mt][2 * kk + 1][2], S[mt][2 * kk + 1][3]);
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t a[4];
        lda(aW, kSD, mt * 16, kk * 16, lane, a);
#pragma unroll
        for (int q = 0; q < 4; ++q) a[q] ^= 0x80008000u;  // -W
#pragma unroll
        for (int n = 0; n < 4; ++n) mma(U[mt][n], a, b[n >> 1][n & 1][0], b[n >> 1][n & 1][1]);
      }
    }
    __syncthreads();  // every warp has read V (step 5) and W before N overwrites V
#pragma unroll
    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int r = mt * 16 + g8, c = warp * 32 + n * 8 + 2 * t4;
        *reinterpret_cast<uint32_t*>(sV + r * kSD + c) = pk(U[mt][n][0], U[mt][n][1]);
        *reinterpret_cast<uint32_t*>(sV + (r + 8) * kSD + c) = pk(U[mt][n][2], U[mt][n][3]);
      }
    // ---- 7. P = (Q K^T) o exp(G_i - G_j) [j <= i], rows [16 warp, +16) -> smem (over T1).
    {
      float acc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        uint32_t a[4];
        lda(aQ, kSD, warp * 16, kk * 16, lane, a);
#pragma unroll
        for (int n2 = 0; n2 < 4; ++n2) {
          uint32_t b[4];
          ldb_nk(aK, kSD, n2 * 16, kk * 16, lane, b);
          mma(acc[2 * n2], a, b[0], b[1]);
          mma(acc[2 * n2 + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int i0 = warp * 16 + g8, j = n * 8 + 2 * t4;
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = i0 + (e >> 1) * 8, jj = j + (e & 1);
          v[e] = jj <= i ? acc[n][e] * __expf(sG[i] - sG[jj]) : 0.f;
        }
        *reinterpret_cast<uint32_t*>(sT1 + i0 * kSC + j) = pk(v[0], v[1]);
        *reinterpret_cast<uint32_t*>(sT1 + (i0 + 8) * kSC + j) = pk(v[2], v[3]);
      }
    }
    __syncthreads();
    // ---- 8. O[:, 32 warp ..] = diag(exp G) Q S0^T + P N  -> global (real tokens).
    {
      float O[4][4][4];
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int n = 0; n < 4; ++n) O[mt][n][0] = O[mt][n][1] = O[mt][n][2] = O[mt][n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        uint32_t b[2][2][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          b[mt][0][0] = pk(S[mt][2 * kk][0], S[mt][2 * kk][1]);
          b[mt][0][1] = pk(S[mt][2 * kk + 1][0], S[mt][2 * kk + 1][1]);
          b[mt][1][0] = pk(S[mt][2 * kk][2], S[mt][2 * kk][3]);
          b[mt][1][1] = pk(S[mt][2 * kk + 1][2], S[mt][2 * kk + 1][3]);
        }
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          uint32_t a[4];
          lda(aQ, kSD, mt * 16, kk * 16, lane, a);
          // rows mt*16 + g8 (a0, a2) and + 8 (a1, a3): scale by exp(G_row)
          const float e0 = __expf(sG[mt * 16 + g8]), e1 = __expf(sG[mt * 16 + g8 + 8]);
          float2 f;
          f = upk(a[0]); a[0] = pk(f.x * e0, f.y * e0);
          f = upk(a[2]); a[2] = pk(f.x * e0, f.y * e0);
          f = upk(a[1]); a[1] = pk(f.x * e1, f.y * e1);
          f = upk(a[3]); a[3] = pk(f.x * e1, f.y * e1);
#pragma unroll
          for (int n = 0; n < 4; ++n) mma(O[mt][n], a, b[n >> 1][n & 1][0], b[n >> 1][n & 1][1]);
        }
      }
#pragma unroll
      for (int kk = 0; kk < kC / 16; ++kk) {
        uint32_t bn[2][4];
#pragma unroll
        for (int n2 = 0; n2 < 2; ++n2) ldb_kn(aV, kSD, warp * 32 + n2 * 16, kk * 16, lane, bn[n2]);
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          uint32_t a[4];
          lda(aT1, kSC, mt * 16, kk * 16, lane, a);
#pragma unroll
          for (int n2 = 0; n2 < 2; ++n2) {
            mma(O[mt][2 * n2], a, bn[n2][0], bn[n2][1]);
            mma(O[mt][2 * n2 + 1], a, bn[n2][2], bn[n2][3]);
          }
        }
      }
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int r = mt * 16 + g8, c = warp * 32 + n * 8 + 2 * t4;
          if (r < L)
            *reinterpret_cast<uint32_t*>(p.o + (size_t)(c0 + r) * p.ldo + h * kD + c) =
                pk(O[mt][n][0], O[mt][n][1]);
          if (r + 8 < L)
            *reinterpret_cast<uint32_t*>(p.o + (size_t)(c0 + r + 8) * p.ldo + h * kD + c) =
                pk(O[mt][n][2], O[mt][n][3]);
        }
    }
    // ---- 9. S = exp(G_L) S + N^T diag(exp(G_L - G)) K   (rows [32 warp, +32)).
    {
      const float GL = sG[kC - 1];
      const float eL = __expf(GL);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) S[mt][nt][e] *= eL;
#pragma unroll
      for (int kk = 0; kk < kC / 16; ++kk) {
        uint32_t a[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) lda_t(aV, kSD, warp * 32 + mt * 16, kk * 16, lane, a[mt]);
        // B rows (k = tokens) 2 t4, 2 t4 + 1 (b0) and + 8 (b1) of this k16 slab.
        const int kb = kk * 16 + 2 * t4;
        const float d0 = __expf(GL - sG[kb]), d1 = __expf(GL - sG[kb + 1]);
        const float d2 = __expf(GL - sG[kb + 8]), d3 = __expf(GL - sG[kb + 9]);
#pragma unroll
        for (int n2 = 0; n2 < 8; ++n2) {
          uint32_t b[4];
          ldb_kn(aK, kSD, n2 * 16, kk * 16, lane, b);
          float2 f;
          f = upk(b[0]); b[0] = pk(f.x * d0, f.y * d1);
          f = upk(b[1]); b[1] = pk(f.x * d2, f.y * d3);
          f = upk(b[2]); b[2] = pk(f.x * d0, f.y * d1);
          f = upk(b[3]); b[3] = pk(f.x * d2, f.y * d3);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            mma(S[mt][2 * n2], a[mt], b[0], b[1]);
            mma(S[mt][2 * n2 + 1], a[mt], b[2], b[3]);
          }
        }
      }
    }
    __syncthreads();  // shared buffers are rewritten by the next chunk
  }

  if (gst != nullptr && p.write_state) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        const int r = warp * 32 + mt * 16 + g8, c = nt * 8 + 2 * t4;
        *reinterpret_cast<float2*>(gst + (size_t)r * kD + c) = make_float2(S[mt][nt][0], S[mt][nt][1]);
        *reinterpret_cast<float2*>(gst + (size_t)(r + 8) * kD + c) =
            make_float2(S[mt][nt][2], S[mt][nt][3]);
      }
  }
}

}  // namespace

bool gdn_chunk_supported(int dk, int dv) { return dk == kD && dv == kD; }

void gdn_chunk_launch(const GdnParams& p, int nseq, int dk, int dv, cudaStream_t stream) {
  if (nseq <= 0) return;
  if (!gdn_chunk_supported(dk, dv)) throw std::runtime_error("gdn_chunk: head dims must be 128");
  if (p.HV % p.HK != 0) throw std::runtime_error("gdn_chunk: HV % HK != 0");
  if (p.ldq % 4 || p.ldk % 4 || p.ldv % 4 || p.ldo % 2)
    throw std::runtime_error("gdn_chunk: row strides must be multiples of 4 elements");
  static bool attr[kMaxDevices] = {};
  set_smem_attr_once(gdn_chunk_kernel, kSmem, attr, "gdn_chunk");
  launch_pdl(gdn_chunk_kernel, dim3(nseq, p.HV), dim3(128), kSmem, stream, nullptr, p);
}

}  // namespace b200
