// Host API of the tcgen05 GEMM family (implemented in gemm_*.cu).
#pragma once
#include <cuda_runtime.h>

namespace b200 {

enum GemmEpilogue : int {
  kEpiNone = 0,     // C = A W^T (bf16)
  kEpiSiluMul = 1,  // W rows interleaved in [gate 64 | up 64] blocks; C = silu(g) * u, N/2 cols
};

enum GemmConfig : int {
  kCfgAuto = -1,
  kCfgN256 = 0,    // 128 x 256 tile, 4 stages
  kCfgN128 = 1,    // 128 x 128 tile, 6 stages
  kCfgSwap16 = 2,  // swap-AB: 128 weight rows x 16 tokens
  kCfgSwap32 = 3,
  kCfgSwap64 = 4,
  kCfgCount = 5,
};

// C[M, N] = A[M, K] . W[N, K]^T  (bf16 in, fp32 accumulate, bf16 out).
void gemm_bf16_launch(const void* A, const void* W, void* C, int M, int N, int K, int lda, int ldw,
                      int ldc, int epi, int cfg, unsigned int* err, cudaStream_t stream);

int gemm_bf16_pick_config(int M, int N, int K, int epi, int num_sm);

}  // namespace b200
