// Host API of the MoE routing kernels (moe_route.cu).
#pragma once
#include <cuda_runtime.h>

namespace b200 {

void moe_topk_launch(const void* logits, bool bf16, int ld, int T, int E, int k, bool sigmoid,
                     bool renorm, const float* bias, float* w, int* ids, cudaStream_t stream);

// Fused router (small T): logits [T, E] fp32 scratch, tile_ctr [ceil(T/8)]
// int32 zeroed once (the kernel re-arms it), w fp32 [T, k], ids int32 [T, k].
void moe_router_launch(const void* x, int ldx, const void* wr, int T, int E, int H, int k,
                       bool sigmoid, bool renorm, const float* bias, float* logits,
                       int* tile_ctr, float* w, int* ids, cudaStream_t stream);

// ids [T*k] global expert ids; experts [e_base, e_base + E) are local.
// align > 1: every local expert's rows start at a multiple of `align` in x_perm
// (x_perm / src_row then need T*k + E*(align-1) rows).
void moe_permute_launch(const int* ids, int T, int k, int E, int e_base, const void* x, int H,
                        void* x_perm, int* counts, int* offsets, int* rank_scratch, int* pos,
                        int* src_row, cudaStream_t stream, int align = 1);

void moe_combine_launch(const void* y, const int* pos, const float* w, int T, int k, int H,
                        const void* shared, float shared_scale, void* out, cudaStream_t stream);

}  // namespace b200
