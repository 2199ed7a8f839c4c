// Gated DeltaNet (Qwen3-Next linear attention) kernels.
//
//   causal_conv1d   depthwise causal conv (kernel W <= 4) + SiLU over the
//                   packed [q | k | v] channels, varlen, with a per-sequence
//                   rolling state [slot, C, W-1] read and updated in place
//                   (prefill and decode share the kernel: decode = 1 token).
//   gdn_recurrent   the gated delta rule, token-serial per (sequence, v-head):
//                     g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(b)
//                     q, k L2-normalised, q *= dk^-1/2
//                     S <- exp(g) S ;  S <- S + beta (v - S k) k^T ;  o = S q
//                   fp32 state [slot, HV, dv, dk] updated in place (thread j of
//                   the CTA owns row j of S in registers for the whole sequence).
//   gated_rmsnorm   o <- rmsnorm(o) * w * silu(z) per head.
//
// Speculative verify: both state kernels take write_state = false for the
// verify forward (states read, not advanced); after acceptance the same
// kernels run once more over the accepted tokens with write_state = true, so
// the stored state ends exactly at the last accepted token (rollback without
// per-position state copies).
//
// Reference parity: FlashQLA GDN (sm70/csrc/gdn/gdn_forward.cu:90-430:
// token-serial varlen recurrence with the state in registers, the decode
// kernel with mixed qkv and slot-indexed global state, slot <= 0 = null
// block), and the FLA gating / conv semantics it serves.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>

#include "gdn/gdn_api.h"

namespace b200 {
namespace {

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

// One thread per (token, channel). x [T, C] -> y [T, C]; state [slots, C, W-1].
__global__ void conv1d_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                              const __nv_bfloat16* __restrict__ w,  // [C, W]
                              const __nv_bfloat16* __restrict__ bias,  // [C] or null
                              __nv_bfloat16* __restrict__ y, int ldy, float* __restrict__ state,
                              const int* __restrict__ cu, const int* __restrict__ slots, int nseq,
                              int C, int W, bool silu, bool write_state) {
  const int s = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= nseq || c >= C) return;
  const int t0 = cu[s], t1 = cu[s + 1];
  const int slot = slots[s];
  float hist[3] = {0.f, 0.f, 0.f};  // x[t-3], x[t-2], x[t-1]
  float* st = slot >= 0 ? state + ((size_t)slot * C + c) * (W - 1) : nullptr;
  if (st)
    for (int i = 0; i < W - 1; ++i) hist[3 - (W - 1) + i] = st[i];
  float wv[4] = {0.f, 0.f, 0.f, 0.f};
  for (int i = 0; i < W; ++i) wv[4 - W + i] = bf(w[(size_t)c * W + i]);
  const float b = bias ? bf(bias[c]) : 0.f;
  for (int t = t0; t < t1; ++t) {
    const float xt = bf(x[(size_t)t * ldx + c]);
    float acc = b + wv[3] * xt + wv[2] * hist[2] + wv[1] * hist[1] + wv[0] * hist[0];
    if (silu) acc = acc / (1.f + __expf(-acc));
    y[(size_t)t * ldy + c] = __float2bfloat16_rn(acc);
    hist[0] = hist[1];
    hist[1] = hist[2];
    hist[2] = xt;
  }
  if (st && write_state)
    for (int i = 0; i < W - 1; ++i) st[i] = hist[3 - (W - 1) + i];
}

// CTA per (sequence, v-head); DV threads; thread j owns S[j, :] (DK floats).
template <int DK, int DV>
__global__ void __launch_bounds__(DV) gdn_recurrent_kernel(const GdnParams p) {
  const int s = blockIdx.x;
  const int h = blockIdx.y;  // v-head
  const int j = threadIdx.x;
  const int hk = h / (p.HV / p.HK);
  const int t0 = p.cu[s], t1 = p.cu[s + 1];
  const int slot = p.slots[s];
  __shared__ float sq[DK], sk[DK];
  __shared__ float sgb[2];
  float S[DK];
  const size_t lds = p.ld_state ? (size_t)p.ld_state : (size_t)p.HV * DV * DK;
  float* st = slot >= 0 ? p.state + (size_t)slot * lds + ((size_t)h * DV + j) * DK : nullptr;
  const bool fresh = p.reset_state || (p.has_init != nullptr && p.has_init[s] == 0);
  if (st && !fresh) {
#pragma unroll
    for (int i = 0; i < DK; i += 4) {
      const float4 v = *reinterpret_cast<const float4*>(st + i);
      S[i] = v.x; S[i + 1] = v.y; S[i + 2] = v.z; S[i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < DK; ++i) S[i] = 0.f;
  }
  const float A = -__expf(p.A_log[h]);
  const float dtb = p.dt_bias[h];
  const float qscale = rsqrtf((float)DK);
  for (int t = t0; t < t1; ++t) {
    const __nv_bfloat16* qrow = p.q + (size_t)t * p.ldq + (size_t)hk * DK;
    const __nv_bfloat16* krow = p.k + (size_t)t * p.ldk + (size_t)hk * DK;
    // L2-normalise q and k (warp 0 reduces, then broadcast through smem)
    if (j < DK) {
      sq[j] = bf(qrow[j]);
      sk[j] = bf(krow[j]);
    }
    if (j == 0) {
      const float a = bf(p.a[(size_t)t * p.ldab + h]);
      const float b = bf(p.b[(size_t)t * p.ldab + h]);
      const float x = a + dtb;
      const float sp = x > 20.f ? x : log1pf(__expf(x));
      sgb[0] = __expf(A * sp);               // exp(g)
      sgb[1] = 1.f / (1.f + __expf(-b));     // beta
    }
    __syncthreads();
    float nq = 0.f, nk = 0.f;
#pragma unroll 8
    for (int i = 0; i < DK; ++i) {
      nq += sq[i] * sq[i];
      nk += sk[i] * sk[i];
    }
    const float iq = rsqrtf(nq + 1e-6f) * qscale;
    const float ik = rsqrtf(nk + 1e-6f);
    const float decay = sgb[0], beta = sgb[1];
    const float vj = bf(p.v[(size_t)t * p.ldv + (size_t)h * DV + j]);
    float u = 0.f;
#pragma unroll
    for (int i = 0; i < DK; ++i) {
      S[i] *= decay;
      u += S[i] * sk[i];
    }
    const float delta = beta * (vj - u * ik);
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < DK; ++i) {
      S[i] += delta * sk[i] * ik;
      o += S[i] * sq[i];
    }
    p.o[(size_t)t * p.ldo + (size_t)h * DV + j] = __float2bfloat16_rn(o * iq);
    __syncthreads();
  }
  if (st && p.write_state) {
#pragma unroll
    for (int i = 0; i < DK; i += 4)
      *reinterpret_cast<float4*>(st + i) = make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
  }
}

// One warp per (token, head): o <- rmsnorm(o) * w * silu(z).
__global__ void gated_rmsnorm_kernel(__nv_bfloat16* __restrict__ o, int ldo,
                                     const __nv_bfloat16* __restrict__ z, int ldz,
                                     const __nv_bfloat16* __restrict__ w, int T, int H, int D,
                                     float eps) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= T * H) return;
  const int t = gw / H, h = gw % H;
  __nv_bfloat16* orow = o + (size_t)t * ldo + (size_t)h * D;
  const __nv_bfloat16* zrow = z + (size_t)t * ldz + (size_t)h * D;
  float ss = 0.f;
  for (int i = lane; i < D; i += 32) {
    const float v = bf(orow[i]);
    ss += v * v;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, off);
  const float inv = rsqrtf(ss / (float)D + eps);
  for (int i = lane; i < D; i += 32) {
    const float zv = bf(zrow[i]);
    const float n = __bfloat162float(__float2bfloat16_rn(bf(orow[i]) * inv)) * bf(w[i]);
    orow[i] = __float2bfloat16_rn(n * (zv / (1.f + __expf(-zv))));
  }
}

}  // namespace

void causal_conv1d_launch(const void* x, int ldx, const void* w, const void* bias, void* y,
                          int ldy, float* state, const int* cu, const int* slots, int nseq, int C,
                          int W, bool silu, bool write_state, cudaStream_t stream) {
  if (nseq <= 0) return;
  if (W < 2 || W > 4) throw std::runtime_error("causal_conv1d: kernel width must be 2..4");
  dim3 grid((C + 127) / 128, nseq);
  conv1d_kernel<<<grid, 128, 0, stream>>>((const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)w,
                                          (const __nv_bfloat16*)bias, (__nv_bfloat16*)y, ldy,
                                          state, cu, slots, nseq, C, W, silu, write_state);
}

void gdn_recurrent_launch(const GdnParams& p, int nseq, int dk, int dv, cudaStream_t stream) {
  if (nseq <= 0) return;
  if (p.HV % p.HK != 0) throw std::runtime_error("gdn: HV % HK != 0");
  dim3 grid(nseq, p.HV);
  if (dk == 128 && dv == 128)
    gdn_recurrent_kernel<128, 128><<<grid, 128, 0, stream>>>(p);
  else if (dk == 64 && dv == 64)
    gdn_recurrent_kernel<64, 64><<<grid, 64, 0, stream>>>(p);
  else
    throw std::runtime_error("gdn: head dims must be 64 or 128");
}

void gated_rmsnorm_launch(void* o, int ldo, const void* z, int ldz, const void* w, int T, int H,
                          int D, float eps, cudaStream_t stream) {
  if (T <= 0) return;
  const long warps = (long)T * H;
  gated_rmsnorm_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream>>>(
      (__nv_bfloat16*)o, ldo, (const __nv_bfloat16*)z, ldz, (const __nv_bfloat16*)w, T, H, D, eps);
}

}  // namespace b200
