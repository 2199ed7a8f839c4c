// Host API of the gated-DeltaNet kernels (gdn.cu).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace b200 {

struct GdnParams {
  const __nv_bfloat16* q;  // [T, HK*DK] (conv output, pre-normalisation), row stride ldq
  const __nv_bfloat16* k;  // [T, HK*DK]
  const __nv_bfloat16* v;  // [T, HV*DV]
  const __nv_bfloat16* a;  // [T, HV] (decay input)
  const __nv_bfloat16* b;  // [T, HV] (beta logit)
  const float* A_log;      // [HV]
  const float* dt_bias;    // [HV]
  __nv_bfloat16* o;        // [T, HV*DV]
  float* state;            // [slots, HV, DV, DK] fp32; slot stride ld_state
  const int* cu;           // [nseq + 1]
  const int* slots;        // [nseq] state slot (< 0: no state)
  int ldq, ldk, ldv, ldab, ldo;
  int HK, HV;
  int reset_state;         // 1: start every sequence from a zero state
  int write_state = 1;     // 0: read the state but do not store it (spec verify)
  long long ld_state = 0;  // floats between state slots (0: dense, HV * DV * DK)
  const unsigned char* has_init = nullptr;  // [nseq] 0: this sequence starts from a zero
                                            // state (null: every sequence reads its slot)
};

void causal_conv1d_launch(const void* x, int ldx, const void* w, const void* bias, void* y,
                          int ldy, float* state, const int* cu, const int* slots, int nseq, int C,
                          int W, bool silu, bool write_state, cudaStream_t stream);
void gdn_recurrent_launch(const GdnParams& p, int nseq, int dk, int dv, cudaStream_t stream);
// Chunked (WY / UT form, 64-token chunks) gated delta rule for prefill:
// same parameters and state semantics as gdn_recurrent_launch (DK = DV = 128).
bool gdn_chunk_supported(int dk, int dv);
void gdn_chunk_launch(const GdnParams& p, int nseq, int dk, int dv, cudaStream_t stream);
void gated_rmsnorm_launch(void* o, int ldo, const void* z, int ldz, const void* w, int T, int H,
                          int D, float eps, cudaStream_t stream);

}  // namespace b200
