// Fused tensor-parallel all-reduce + residual add + RMSNorm over NVLink peer
// memory (one process per GPU, symmetric buffers exchanged at start-up).
//
//   stage_r  [T, H] bf16   rank r's partial sums (written by the row-parallel
//                          GEMM directly: the GEMM's output buffer IS the stage)
//   res      [T, H] bf16   residual (identical on every rank), updated in place
//   out_x    [T, H] bf16   normalised output, written on every rank
//
// Two-shot, row-partitioned: rank r owns rows [r*T/W, (r+1)*T/W). For each of
// its rows it loads the W partial rows from the peers' stages (NVLink P2P
// loads, summed in rank order in fp32 -- deterministic and identical on every
// rank), rounds the sum to bf16, adds the residual (bf16 round, as the unfused
// fused_add_rms_norm does), RMS-normalises, and stores the new residual row and
// the normalised row into EVERY rank's res / out_x (P2P stores). Traffic per
// rank: (W-1)/W of the tensor in, (W-1)/W * 2 out.
//
// Synchronisation (epoch flags in each rank's signal pad, .sys scope):
//   start : CTA 0 of rank r release-stores ready[r] = epoch on every peer;
//           every CTA acquire-spins until ready[p] >= epoch for all p.
//   end   : every CTA release-adds 1 to done[r] on every peer after its stores;
//           CTA 0 acquire-spins until done[p] reaches the cumulative CTA count
//           of all launches so far (the grid is rank-uniform), then bumps the
//           local epoch. The kernel therefore ends only after every
//           peer has finished reading this rank's stage and writing its rows
//           here, so the next launch may overwrite the stage and the next
//           kernel on the stream may read res / out_x.
// Every spin is bounded (%globaltimer); on timeout the kernel records
// kErrPeerTimeout in the status word and returns -- it never traps.
//
// Reference parity: the TP2 AR + add + RMSNorm kernel
// (sm70/csrc/custom_ar/tp2_ar_fused_add_rms_norm.cu:67-174: stage -> membar.sys
// flag barrier -> peer read -> fp32 sum -> one rounding -> +residual -> RMSNorm
// -> end-flag barrier). Differences: W in {2,4,8}, two-shot row partition
// instead of every rank reducing every row, release/acquire flags with
// bounded waits, and no extra staging copy.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "comm/ar_rmsnorm_dev.cuh"
#include "comm/comm_api.h"
#include "common/launch.h"

namespace b200 {
namespace {

__global__ void __launch_bounds__(512) ar_rmsnorm_kernel(ArRmsNormParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ float part[ardev::kMaxVec * 512];
  __shared__ float bcast;
  __shared__ int s_ok;
  ardev::run_any(p, /*gated=*/false, part, &bcast, &s_ok);
}

}  // namespace

void ar_rmsnorm_launch(const ArRmsNormParams& p, int grid, cudaStream_t stream) {
  if (p.H % 8 != 0) throw std::runtime_error("ar_rmsnorm: H % 8 != 0");
  int threads = ((p.H / 8 + ardev::kMaxVec - 1) / ardev::kMaxVec + 31) / 32 * 32;
  if (threads < 64) threads = 64;
  if (threads > 512) throw std::runtime_error("ar_rmsnorm: H too large");
  if (p.world != 2 && p.world != 4 && p.world != 8)
    throw std::runtime_error("ar_rmsnorm: world size must be 2, 4 or 8");
  launch_pdl(ar_rmsnorm_kernel, dim3(grid), dim3(threads), 0, stream, nullptr, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("ar_rmsnorm: ") + cudaGetErrorString(e));
}

}  // namespace b200
