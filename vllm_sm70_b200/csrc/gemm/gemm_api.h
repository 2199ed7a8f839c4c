// Host API of the tcgen05 GEMM family (implemented in gemm_*.cu).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

#include <vector>

#include "comm/comm_api.h"

namespace b200 {

enum GemmEpilogue : int {
  kEpiNone = 0,     // C = A W^T (bf16)
  kEpiSiluMul = 1,  // W rows interleaved in [gate 64 | up 64] blocks; C = silu(g) * u, N/2 cols
  kEpiArNorm = 2,   // C = this rank's stage of a TP all-reduce; the kernel then runs the fused
                    // all-reduce + residual add + RMSNorm over NVLink peer memory (WQParams::ar)
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
  kCfgM2N256 = 9,  // tall tile: 256 x 256 (two M=128 accumulators), 3 stages
  kCfgM2N224 = 10, // 256 x 224
  kCfgM2N128 = 11, // 256 x 128
  kCfgM2N112 = 12, // 256 x 112
  kCfgM2N64 = 13,  // 256 x 64
  // Cluster split-K (the K slices of a tile form one cluster, reduced through
  // distributed shared memory; needs splits >= 2, else runs as the plain tile):
  kCfgClN256 = 14,   // 128 x 256
  kCfgClN128 = 15,   // 128 x 128
  kCfgClM2N128 = 16, // 256 x 128
  kCfgClM2N112 = 17, // 256 x 112
  kCfgClM2N64 = 18,  // 256 x 64
  // CTA pairs (tcgen05 cta_group::2): one 256-row tile over two SMs, each
  // holding 128 rows of A, half of B's rows and its half of the accumulator.
  kCfgP2N256 = 19,   // 256 x 256, 6 stages
  kCfgP2N128 = 20,   // 256 x 128, 8 stages
  kCfgP2N192 = 21,   // 256 x 192, 7 stages
  kCfgP2N64 = 22,    // 256 x 64, 10 stages
  kCfgP2N96 = 23,    // 256 x 96, 9 stages (decode: 64 pairs over N = 6144)
  kCfgCount = 24,
};

constexpr int kMaxSplits = 8;

// Weight formats of the weight-only quantised GEMMs (activations bf16).
enum WeightFormat : int {
  kWBf16 = 0,
  kWFp8 = 1,    // e4m3 [N, K], fp32 scale per 128x128 block: scales_f32[N/128][K/128]
  kWAwq = 2,    // int4 [N, K/2] (low nibble = even k), per (row, 128-group) bf16x2 (s, -z*s)
  kWNvfp4 = 3,  // e2m1 [N, K/2] (low nibble = even k), e4m3 scale per (row, 16 k); x out_scale
};

// Raw bytes of one weight row per 64-wide k-block.
__host__ __device__ constexpr int raw_row_bytes(int wf) {
  return wf == kWFp8 ? 64 : (wf == kWBf16 ? 0 : 32);
}

// All-gather -> GEMM: this rank's row shard is copied into every rank's gather
// buffer by the GEMM's epilogue warps (before their first accumulator), and the
// producer TMA-loads each A tile from the local gather buffer once the ranks
// whose rows it covers have raised their ready flag (world 0: off). Gather
// buffers hold two halves of t_max rows, used by alternate epochs; pad words:
// ready[8], arrive, done, epoch.
struct AgParams {
  uint8_t* xfull_peer[kMaxRanks] = {};  // every rank's gather buffer [2][t_max][K] bf16
  uint32_t* pad_peer[kMaxRanks] = {};   // every rank's signal pad
  uint32_t* pad_local = nullptr;
  const void* shard = nullptr;          // this rank's rows [rows_per_rank][K] bf16
  int rank = 0, world = 0;
  int rows_per_rank = 0;
  int t_max = 0;
  int K = 0;
  unsigned long long timeout_ns = 0;
};
constexpr int kAgPadReady = 0, kAgPadArrive = 8, kAgPadDone = 9, kAgPadEpoch = 10;

struct WQParams {
  const float* scales_f32 = nullptr;                // kWFp8
  const __nv_bfloat162* scale_zero = nullptr;       // kWAwq
  const uint8_t* scales_u8 = nullptr;               // kWNvfp4
  int scale_ld = 0;                                 // elements per scale row
  float out_scale = 1.f;                            // kWNvfp4 global scale
  ArRmsNormParams ar{};                             // kEpiArNorm: the collective after the GEMM
  AgParams ag{};                                    // all-gather -> GEMM (plain normal-mode tiles)
};

// Grouped (MoE) GEMM: per-expert tiles read from device arrays.
struct GroupInfo {
  const int* tile_off = nullptr;  // [E + 1] tile prefix (filled by the launcher's setup kernel)
  const int* row_off = nullptr;   // [E + 1] expert row offsets into X (expert-sorted rows)
  int E = 0;                      // 0 = not grouped
  int N = 0;                      // weight rows per expert
};

// C[r, :] = X[r, :] . W_e^T for r in expert e's rows [row_off[e], row_off[e+1]);
// W stacked [E * N, K] (bf16, or raw quantised rows with stacked scales).
// Swap-AB tiles (weights on the 128-row side), counts read on the device, so
// the launch is CUDA-graph capturable. tile_off: int32 scratch [E + 1].
void gemm_grouped_launch(const void* X, const void* Wstk, void* C, int rows, int E, int N, int K,
                         int ldx, int ldw, int ldc, const int* row_off, int* tile_off, int wf,
                         const WQParams& wq, int bn, unsigned int* err, cudaStream_t stream);

void dequant_weight_launch(const void* raw, long long ld_raw, void* out, int N, int K, int wf,
                           const WQParams& q, cudaStream_t stream);

// C[M, N] = A[M, K] (bf16) . dequant(W)[N, K]^T, M <= 256 (decode shapes),
// swap-AB tiles with split-K (bn/splits <= 0: automatic).
void gemm_wq_launch(const void* A, const void* Wraw, void* C, int M, int N, int K, int lda,
                    int ld_raw, int ldc, int wf, const WQParams& wq, int bn, int splits,
                    unsigned int* err, cudaStream_t stream);

// ---- Block-scaled FP8 (W8A8) on kind::f8f6f4 (gemm_fp8_tc.cu) ----
// Per-token, 128-wide-group activation quantisation: xq e4m3 [M, K] (row
// stride ldq bytes), sa fp32 [ceil(K/128)][ld_sa] (ld_sa >= M).
void quant_fp8_act_launch(const void* x, int ldx, int M, int K, void* xq, int ldq, float* sa,
                          int ld_sa, cudaStream_t stream);
// C[M, N] (bf16) = dequant(Aq, sa) . dequant(Wq, sw)^T with exact fp32 scale
// promotion per 128-wide K block; sw fp32 [ceil(N/128)][ld_sw]. bn <= 0:
// automatic (128 x 128 tiles for M > 64, swap-AB tiles of 32 / 64 tokens below).
void gemm_fp8_launch(const void* Aq, const float* sa, int ld_sa, const void* Wq, const float* sw,
                     int ld_sw, void* C, int M, int N, int K, int lda, int ldw, int ldc, int bn,
                     unsigned int* err, cudaStream_t stream);
// Grouped (MoE) form over expert-sorted rows: C[r, :] = X[r] . W_e^T for r in
// [row_off[e], row_off[e+1]); W stacked [E * N, K] e4m3 with sw [E * N / 128][ld_sw];
// X e4m3 [rows, K] with sa [ceil(K/128)][ld_sa]. tile_off: int32 scratch [E + 1].
void gemm_fp8_grouped_launch(const void* Xq, const float* sa, int ld_sa, const void* Wstk,
                             const float* sw, int ld_sw, void* C, int rows, int E, int N, int K,
                             int ldx, int ldw, int ldc, const int* row_off, int* tile_off, int bn,
                             unsigned int* err, cudaStream_t stream);

// ---- NVFP4 W4A4 on kind::mxf4nvf4 (gemm_nvfp4_tc.cu) ----
// Scale tensors (bytes) are in atom order [rows/128][K/64][512]: row r's 4
// scales of 64-k group kg at ((r/128) * K/64 + kg) * 512 + (r%32)*16 + ((r%128)/32)*4.
// Activations: xq [M, K/2] packed e2m1, sf atoms, rs [M] per-token fp32 scales.
// n_rows (device, optional): rows at or past *n_rows are skipped (padded
// MoE permutations whose used length is only known on the device).
void quant_nvfp4_act_launch(const void* x, int ldx, int M, int K, void* xq, int ldq, void* sf,
                            float* rs, cudaStream_t stream, const int* n_rows = nullptr);
// C = rs[m] * g * (Aq . Wq^T with both block scales); swap < 0: automatic.
void gemm_nvfp4_launch(const void* Aq, const void* sfa, const float* rs, const void* Wq,
                       const void* sfw, float g, void* C, int M, int N, int K, int lda, int ldw,
                       int ldc, int swap, unsigned int* err, cudaStream_t stream);
// Grouped over expert-sorted rows whose expert blocks start at multiples of 128.
void gemm_nvfp4_grouped_launch(const void* Xq, const void* sfx, const float* rs, const void* Wstk,
                               const void* sfw, float g, void* C, int rows, int E, int N, int K,
                               int ldx, int ldw, int ldc, const int* row_off, int* tile_off,
                               unsigned int* err, cudaStream_t stream);

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

// Profiling aid: install (or with nullptr remove) a device buffer of
// 16 x grid uint64 that the next GEMM launches fill with per-CTA %globaltimer
// stamps (entry, set-up, first TMA, first stage ready, last MMA, first
// accumulator, epilogue done, exit, then split-K epilogue phases).
void gemm_set_timeline(unsigned long long* buf);

// Tile width (N side of the accumulator) and swap-AB flag of a config (0 / false if unknown).
int gemm_cfg_tile_n(int cfg);
int gemm_cfg_tile_m(int cfg);  // 128 or 256 (tall tiles)

// Tile geometry the launcher uses for (M, N, K, cfg, splits): rows per P
// tile (swap-AB tiles are fitted to the SM count), tile count, and the fp32
// split-K workspace it needs.
struct SplitGeometry {
  int tile_rows = 128;
  long tiles = 0;
  size_t ws_bytes = 0;
  long counters = 0;  // arrival counters the split needs
};
SplitGeometry gemm_split_geometry(int M, int N, int K, int cfg, int splits, int num_sm);
bool gemm_cfg_is_cluster(int cfg);  // split-K reduced in a cluster (no workspace)
bool gemm_cfg_is_swap(int cfg);

// Explicit-workspace variant: splits > 1 needs ws >= tiles*splits*128*BN*4
// bytes and counters[tiles] zeroed (they are re-armed by the kernel).
// ext_reduce: a one-round plain split may leave its fp32 partials in ws as
// [splits][M][N] and sum them in a second kernel on the stream (needs
// splits x M x N floats of workspace; opt-in with VLLM_B200_GEMM_EXT_REDUCE=1).
void gemm_bf16_launch_split(const void* A, const void* W, void* C, int M, int N, int K, int lda,
                            int ldw, int ldc, int epi, int cfg, int splits, float* ws,
                            size_t ws_bytes, int* counters, int n_counters, unsigned int* err,
                            cudaStream_t stream, bool ext_reduce = false);

// Row-parallel GEMM fused with the TP all-reduce + residual add + RMSNorm in one
// kernel: C = A W^T goes into this rank's symmetric stage (ar.stage_peer[rank]),
// then the same CTAs run the collective over NVLink peer memory. N == ar.H,
// M == ar.T. Returns false (nothing launched) for shapes it does not take.
// All-gather -> GEMM (AgParams): C[T, N] = gather(x shards)[T, K] . W^T.
void gemm_ag_launch(const void* W, void* C, int T, int N, int K, int ldw, int ldc, int cfg,
                    int splits, const AgParams& ag, unsigned int* err, cudaStream_t stream);

bool gemm_ar_rmsnorm_launch(const void* A, const void* W, int M, int N, int K, int lda, int ldw,
                            int cfg, int splits, const ArRmsNormParams& ar, unsigned int* err,
                            cudaStream_t stream);

}  // namespace b200
