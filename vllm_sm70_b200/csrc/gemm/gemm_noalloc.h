// C entry point of the split-K bf16 GEMM that allocates no device memory.
//
// This entry point has no counterpart in the reference: it exists for callers
// that cannot allocate device memory at the moment they need a GEMM. Examples:
// a C or C++ runtime that embeds this library without libtorch (no caching
// allocator to draw scratch from, and a cudaMalloc on the hot path would
// synchronise the whole device), or code that runs after a serving engine has
// reserved almost all HBM for its KV cache, where a late cudaMalloc can fail.
// The split-K partial sums, the arrival counters and the status word live in
// fixed-size file-scope __device__ arrays of this library instead.
//
// Limits: at most B200_NOALLOC_WS_BYTES of fp32 partial tiles and
// B200_NOALLOC_MAX_TILES output tiles per call; a call that needs more returns
// B200_NOALLOC_ETOOBIG and launches nothing (use splits = 1, or the
// workspace-backed entry points, for such shapes).
//
// Concurrency: the scratch is one region per device. Two calls that are in
// flight on the same device at the same time (different streams, or different
// host threads) overwrite each other's partial sums and counters, so their
// results are undefined. Issue the calls of one device on one stream, or order
// them with events.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_NOALLOC_WS_BYTES (8u << 20)  // fp32 split-K partials per device
#define B200_NOALLOC_MAX_TILES 2048       // arrival counters per device

enum {
  B200_NOALLOC_OK = 0,
  B200_NOALLOC_EINVAL = 1,   // bad arguments (sizes, alignment, config)
  B200_NOALLOC_ETOOBIG = 2,  // the shape needs more scratch than the static region holds
  B200_NOALLOC_ECUDA = 3,    // a CUDA runtime call failed (see the message)
};

// C[M, N] = A[M, K] . W[N, K]^T, bf16 in / fp32 accumulate / bf16 out, on the
// current device and `stream`. Row strides lda, ldw, ldc are in elements
// (multiples of 8); K and N multiples of 8. cfg < 0 picks the tile config
// (and, if splits <= 0, the split factor) with the same planner as the
// workspace-backed entry point; splits is clamped to [1, 8] and to the number
// of 64-wide k-blocks.
//
// The first call on each device does one-time setup: it looks up the address
// of the static scratch with cudaGetSymbolAddress and sets the kernel's shared
// memory attribute. Make that first call before any stream capture.
//
// The arrival counters must be zero when a launch starts. They are zero when
// the library is loaded and every completed launch leaves them zero again; a
// launch that ended with an error status (a bounded wait that gave up) may
// leave them nonzero, after which b200_gemm_bf16_noalloc_reset must run.
int b200_gemm_bf16_noalloc(const void* A, int lda, const void* W, int ldw, void* C, int ldc, int M,
                           int N, int K, int cfg, int splits, cudaStream_t stream);

// Message of the last failed call on this host thread ("" if none).
const char* b200_gemm_bf16_noalloc_last_error(void);

// Copies the device status word of the static region (0 = no kernel gave up
// a wait) into *out; synchronous.
int b200_gemm_bf16_noalloc_status(unsigned int* out);

// Zeroes the counters and the status word of the current device on `stream`.
int b200_gemm_bf16_noalloc_reset(cudaStream_t stream);

#ifdef __cplusplus
}
#endif
