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
  int rank, world, T, H;
  float eps;
  unsigned long long timeout_ns;
  unsigned int* err;
};

void ar_rmsnorm_launch(const ArRmsNormParams& p, int grid, cudaStream_t stream);

}  // namespace b200
