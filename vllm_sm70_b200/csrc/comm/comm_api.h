// Host API of the fused NVLink collectives.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cuda_bf16.h>

namespace b200 {

constexpr int kMaxRanks = 8;

// Signal-pad layout per rank (uint32): ready[W], done[W], epoch, done_target.
struct ArRmsNormParams {
  const __nv_bfloat16* stage_peer[kMaxRanks];  // every rank's stage buffer (peer-mapped)
  __nv_bfloat16* res_peer[kMaxRanks];          // every rank's residual buffer
  __nv_bfloat16* out_peer[kMaxRanks];          // every rank's normalised-output buffer
  uint32_t* flags_peer[kMaxRanks];             // every rank's signal pad
  uint32_t* flags_local;                       // this rank's signal pad
  const __nv_bfloat16* res_local;              // this rank's residual (== res_peer[rank])
  const __nv_bfloat16* w;                      // RMSNorm weight [H]
  // NVLS: multicast addresses of the stage / residual / output buffers (all
  // null: plain peer loads and stores). With them, each owned row is summed in
  // the switch (multimem.ld_reduce, fp32 accumulation, one bf16 result) and
  // stored to every rank with one multimem.st.
  const __nv_bfloat16* mc_stage;
  __nv_bfloat16* mc_res;
  __nv_bfloat16* mc_out;
  int rank, world, T, H;
  float eps;
  unsigned long long timeout_ns;
  unsigned int* err;
};

void ar_rmsnorm_launch(const ArRmsNormParams& p, int grid, cudaStream_t stream);

// Expert-parallel token exchange over peer memory (ep_a2a.cu). Buffers per
// rank (symmetric): recv_x [W][T_cap][H] bf16, recv_meta [W][T_cap][2k] int32,
// back_y [W][T_cap][H] bf16, pad [64] uint32.
struct EpParams {
  __nv_bfloat16* recv_x_peer[kMaxRanks];
  int* recv_meta_peer[kMaxRanks];
  __nv_bfloat16* back_y_peer[kMaxRanks];
  uint32_t* pad_peer[kMaxRanks];
  const __nv_bfloat16* recv_x_local;
  const int* recv_meta_local;
  const __nv_bfloat16* back_y_local;
  uint32_t* pad_local;
  int rank, world, H, k, E_local, T_cap;
  unsigned long long timeout_ns;
  unsigned int* err;
};
// Source side: slot[T][W] and send_count[W] (local scratch), rows + routing
// stored into the destinations' recv buffers, epoch flag raised.
void ep_dispatch_launch(const EpParams& p, const void* x, const int* ids, const float* w, int T,
                        int* slot, int* send_count, cudaStream_t stream);
// Destination side: waits for every source, compacts received rows into
// xc [n_max, H] / idc, wc [n_max, k] / row_src [n_max]; *n_rows = rows received.
void ep_receive_launch(const EpParams& p, void* xc, int* idc, float* wc, int* row_src,
                       int* n_rows, int n_max, cudaStream_t stream);
// Destination side: partial rows y [n_rows, H] back to their sources.
void ep_return_launch(const EpParams& p, const void* y, const int* row_src, const int* n_rows,
                      int n_max, cudaStream_t stream);
// Source side: out[t] = bf16(sum over destinations in rank order + shared[t]).
void ep_finish_launch(const EpParams& p, const int* slot, int T, const void* shared, void* out,
                      cudaStream_t stream);

// Vocab-parallel sampler exchange over peer memory (tp_exchange.cu). Buffers
// per rank (symmetric): recv [2][W][cap] bytes, pad [W + 3] uint32. The
// message is src0 (n0 bytes) followed by src1 (n1 bytes), 4-byte words.
constexpr int kTpXchgTop1 = 0;    // src0 = values [rows] fp32, src1 = ids [rows] int32
constexpr int kTpXchgGather = 1;  // src0 = values [rows, C] fp32, src1 = ids [rows, C] int32
struct TpExchangeParams {
  uint8_t* recv_peer[kMaxRanks];
  uint32_t* pad_peer[kMaxRanks];
  const uint8_t* recv_local;
  uint32_t* pad_local;
  int rank, world, mode, rows, C;
  long long cap;
  const void* src0;
  long long n0;
  const void* src1;
  long long n1;
  int* out_ids;  // kTpXchgTop1: [rows]
  float* out_v;  // kTpXchgGather: [rows, W * C]
  int* out_i;
  unsigned long long timeout_ns;
  unsigned int* err;
};
void tp_exchange_launch(const TpExchangeParams& p, cudaStream_t stream);

}  // namespace b200
