// Host API of the tcgen05 GEMM family (implemented in gemm_*.cu).
#pragma once
#include <cuda_runtime.h>

#include <vector>

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
  kCfgN192 = 5,    // 128 x 192
  kCfgN96 = 6,     // 128 x 96
  kCfgN64 = 7,     // 128 x 64
  kCfgSwap128 = 8, // swap-AB: 128 weight rows x 128 tokens
  kCfgCount = 9,
};

constexpr int kMaxSplits = 8;

struct GemmPlan {
  int cfg;
  int splits;  // split-K factor (1 = none); partials reduced in-kernel, fixed order
};

// Tile config + split-K choice from a wave-quantisation cost model.
GemmPlan gemm_bf16_plan(int M, int N, int K, int epi, int num_sm);

// Tuned dispatch table (consulted by gemm_bf16_plan before the cost model).
void gemm_set_plan(int M, int N, int K, int epi, int cfg, int splits);  // cfg < 0 erases
void gemm_clear_plans();
std::vector<int> gemm_export_plans();  // flat [M, N, K, epi, cfg, splits] * n

// Process-wide split-K workspace (fp32 partials + self-re-arming counters).
void gemm_configure_workspace(int device, size_t ws_bytes, int n_counters);
size_t gemm_workspace_bytes(int device);
float* gemm_ws_ptr(int device);
int* gemm_counters_ptr(int device);
int gemm_n_counters(int device);

// C[M, N] = A[M, K] . W[N, K]^T  (bf16 in, fp32 accumulate, bf16 out).
// cfg < 0: planned automatically (tile + split-K over the configured workspace).
void gemm_bf16_launch(const void* A, const void* W, void* C, int M, int N, int K, int lda, int ldw,
                      int ldc, int epi, int cfg, unsigned int* err, cudaStream_t stream);

int gemm_bf16_pick_config(int M, int N, int K, int epi, int num_sm);

// Explicit-workspace variant: splits > 1 needs ws >= tiles*splits*128*BN*4
// bytes and counters[tiles] zeroed (they are re-armed by the kernel).
void gemm_bf16_launch_split(const void* A, const void* W, void* C, int M, int N, int K, int lda,
                            int ldw, int ldc, int epi, int cfg, int splits, float* ws,
                            size_t ws_bytes, int* counters, int n_counters, unsigned int* err,
                            cudaStream_t stream);

}  // namespace b200
