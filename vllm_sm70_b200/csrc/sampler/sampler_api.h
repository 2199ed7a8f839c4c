// Host API of the sampling kernels (sample.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace b200 {

// row_offsets (optional, device): per-row counter added to `offset`, so a
// CUDA graph replays fresh randomness (e.g. the row's generated-token count).
void gumbel_argmax_launch(const void* logits, bool bf16, int rows, int V, int ld,
                          const float* temperature, const int64_t* seeds, uint64_t offset,
                          const int64_t* row_offsets, int id_offset, int* ids, float* vals,
                          cudaStream_t stream);
void topk_candidates_launch(const void* logits, bool bf16, int rows, int V, int ld, int K,
                            int id_offset, float* out_v, int* out_i, cudaStream_t stream);
void sample_candidates_launch(const float* cand_v, const int* cand_i, int rows, int C,
                              const float* temperature, const int* top_k, const float* top_p,
                              const int64_t* seeds, uint64_t offset, int* out,
                              cudaStream_t stream);

// Speculative-decoding verification: target logits [rows, k+1, V], draft
// logits [rows, k, V] (bf16), draft ids [rows, k] -> out_tokens [rows, k+1],
// num_out [rows].
void rejection_sample_launch(const void* target_logits, const void* draft_logits,
                             const int* draft_ids, int rows, int k, int V, const float* temperature,
                             const int64_t* seeds, uint64_t offset, int* out_tokens, int* num_out,
                             cudaStream_t stream);

}  // namespace b200
