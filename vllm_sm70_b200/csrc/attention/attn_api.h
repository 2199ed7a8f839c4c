// Host API of the paged attention kernels.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include <cstdint>

namespace b200 {

struct AttnArgs {
  const void* q;        // [T, Hq, D] bf16, token stride q_stride_t elements
  const void* k_cache;  // [num_blocks, Hkv, block_size, D] bf16
  const void* v_cache;
  void* out;            // [T, Hq, D] bf16, token stride o_stride_t elements
  const int* block_table;  // [num_seqs, max_blocks]
  const int* seq_lens;     // [num_seqs]
  const int* cu_q;         // [num_seqs + 1]
  const float* sinks;      // [Hq] or nullptr
  float* part_o;           // split-KV partial outputs [splits, T, Hq, D] (decode only)
  float* part_ml;          // [splits, T, Hq, 2]
  int num_seqs, num_tokens, Hq, Hkv, head_dim, block_size, max_blocks;
  int max_q_len;  // max tokens per sequence in this batch (grid sizing)
  int window;     // sliding window (0 = full)
  int q_stride_t, o_stride_t;
  float scale;
  bool decode;     // use the decode (1-warp, split-KV) variant
  int num_splits;  // decode split-KV factor (1 = none)
  long long kv_block_stride = 0;  // elements between cache blocks (0 = Hkv*BS*D, packed)
  int num_blocks = 0;             // cache blocks (the tensor-core prefill path needs it)
};

void paged_attention_launch(const AttnArgs& a, cudaStream_t stream);

// tcgen05 prefill attention (attention/fa_tc.cu): used by paged_attention_launch
// for the shapes fa_tc_supported accepts (VLLM_B200_ATTN_PREFILL_TC=0 disables).
bool fa_tc_enabled();
bool fa_tc_supported(const AttnArgs& a);
void fa_tc_launch(const AttnArgs& a, cudaStream_t stream);
// Bring-up aid: override the V operand descriptor strides (0, 0 = defaults).
// Profiling aid: 8 x grid uint64 %globaltimer stamps per launch (nullptr = off):
// entry, set-up done, Q landed, first S ready, softmax loop done, last PV
// done, epilogue stored, exit.
void fa_tc_set_timeline(unsigned long long* buf);

}  // namespace b200
