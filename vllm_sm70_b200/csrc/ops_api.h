// Launcher declarations shared by the kernel translation units and the torch
// bindings. Launchers take raw device pointers + a stream; the bindings do
// the tensor checks.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "attention/attn_api.h"
#include "gemm/gemm_api.h"

namespace b200 {

constexpr int kAbiVersion = 1;

// Per-device status word (bounded-wait timeouts, overflow flags), allocated once.
unsigned int* device_status_ptr(int device);

void rms_norm_launch(void* out, int ld_out, const void* x, int ld_x, const void* w, int rows, int H,
                     float eps, cudaStream_t stream);
void fused_add_rms_norm_launch(void* x, int ld_x, void* residual, int ld_r, const void* w, int rows,
                               int H, float eps, cudaStream_t stream);
void rope_kv_write_launch(void* qkv, const int64_t* pos, const float* cos_sin, void* k_cache,
                          void* v_cache, const int64_t* slots, const void* q_norm,
                          const void* k_norm, int T, int Hq, int Hkv, int D, int BS, float eps,
                          int rot_dim, long long blk_stride, cudaStream_t stream);
void kv_cache_write_launch(const void* k, const void* v, long long ldk, long long ldv,
                           void* k_cache, void* v_cache, const int64_t* slots, int T, int Hkv,
                           int D, int BS, long long blk_stride, cudaStream_t stream);
void argmax_launch(const void* logits, bool is_bf16, int rows, int V, int ld, int* ids, float* vals,
                   int id_offset, cudaStream_t stream);
// block = 0: x = [gate | up]; block > 0: gate / up interleaved in blocks of
// `block` columns.
void silu_mul_launch(void* out, const void* x, int T, int I, int ld_x, int ld_o,
                     cudaStream_t stream, int block = 0, const int* n_rows = nullptr);
void embedding_launch(void* out, const int64_t* ids, const void* table, int T, int H,
                      int64_t vocab_start, int64_t vocab_end, cudaStream_t stream);

}  // namespace b200
