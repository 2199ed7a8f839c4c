// Split-K bf16 GEMM over file-scope static scratch (no device allocation).
// The kernel is the same tcgen05 persistent GEMM as the workspace-backed
// entry point; only where its partial tiles, counters and status word live
// differs. Declarations and the caller contract are in gemm_noalloc.h.
#include <cuda_runtime.h>

#include <cstdio>
#include <exception>
#include <mutex>

#include "common/tmap.h"
#include "gemm/gemm_api.h"
#include "gemm/gemm_noalloc.h"

namespace {

// Zero-initialised when the module loads (the counters' required start state).
__device__ __align__(256) float g_noalloc_ws[B200_NOALLOC_WS_BYTES / sizeof(float)];
__device__ __align__(256) int g_noalloc_counters[B200_NOALLOC_MAX_TILES];
__device__ __align__(256) unsigned int g_noalloc_status[16];

struct Region {
  float* ws = nullptr;
  int* counters = nullptr;
  unsigned int* status = nullptr;
};

constexpr int kMaxDevices = 64;
Region g_regions[kMaxDevices];
std::mutex g_region_mu;

thread_local char g_last_error[256] = "";

int fail(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

int fail_cuda(const char* what, cudaError_t e) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what, cudaGetErrorString(e));
  return B200_NOALLOC_ECUDA;
}

// Device addresses of the static arrays for the current device, looked up
// once per device (the current device at the time of the call is the one
// whose module instance the symbols resolve to).
int region_for_current_device(Region** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return fail(B200_NOALLOC_EINVAL, "device index out of range");
  std::lock_guard<std::mutex> g(g_region_mu);
  Region& r = g_regions[dev];
  if (r.ws == nullptr) {
    Region n;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&n.ws), g_noalloc_ws);
    if (e != cudaSuccess) return fail_cuda("cudaGetSymbolAddress(scratch)", e);
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&n.counters), g_noalloc_counters);
    if (e != cudaSuccess) return fail_cuda("cudaGetSymbolAddress(counters)", e);
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&n.status), g_noalloc_status);
    if (e != cudaSuccess) return fail_cuda("cudaGetSymbolAddress(status)", e);
    r = n;
  }
  *out = &r;
  return B200_NOALLOC_OK;
}

}  // namespace

extern "C" int b200_gemm_bf16_noalloc(const void* A, int lda, const void* W, int ldw, void* C,
                                      int ldc, int M, int N, int K, int cfg, int splits,
                                      cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (M <= 0 || N <= 0 || K <= 0) return fail(B200_NOALLOC_EINVAL, "M, N, K must be positive");
  if (!A || !W || !C) return fail(B200_NOALLOC_EINVAL, "null operand pointer");
  if (K % 8 || N % 8 || lda % 8 || ldw % 8 || ldc % 8 || lda < K || ldw < K || ldc < N)
    return fail(B200_NOALLOC_EINVAL, "K, N and the row strides must be multiples of 8 (strides >= rows)");
  Region* r = nullptr;
  int rc = region_for_current_device(&r);
  if (rc != B200_NOALLOC_OK) return rc;
  try {
    int dev = 0;
    cudaGetDevice(&dev);
    // Resolve config and split factor exactly as the launcher will, so the
    // scratch check below sees the split that actually runs.
    if (cfg < 0) {
      const b200::GemmPlan pl = b200::gemm_bf16_plan(M, N, K, b200::kEpiNone, b200::num_sms(dev));
      cfg = pl.cfg;
      if (splits <= 0) splits = pl.splits;
    }
    const int bn = b200::gemm_cfg_tile_n(cfg);
    if (bn == 0) return fail(B200_NOALLOC_EINVAL, "unknown tile config");
    if (splits <= 0) splits = 1;
    if (splits > b200::kMaxSplits) splits = b200::kMaxSplits;
    const int num_kb = (K + 63) / 64;
    if (splits > num_kb) splits = num_kb;
    if (splits > 1 && !b200::gemm_cfg_is_cluster(cfg)) {
      const b200::SplitGeometry geo =
          b200::gemm_split_geometry(M, N, K, cfg, splits, b200::num_sms(dev));
      const long tiles = geo.tiles;
      const size_t need = geo.ws_bytes;
      if (need > B200_NOALLOC_WS_BYTES || geo.counters > B200_NOALLOC_MAX_TILES) {
        std::snprintf(g_last_error, sizeof(g_last_error),
                      "split-K scratch too small: need %zu bytes / %ld tiles, static limit %u bytes "
                      "/ %d tiles (use fewer splits)",
                      need, tiles, (unsigned)B200_NOALLOC_WS_BYTES, B200_NOALLOC_MAX_TILES);
        return B200_NOALLOC_ETOOBIG;
      }
    }
    b200::gemm_bf16_launch_split(A, W, C, M, N, K, lda, ldw, ldc, b200::kEpiNone, cfg, splits,
                                 r->ws, B200_NOALLOC_WS_BYTES, r->counters,
                                 B200_NOALLOC_MAX_TILES, r->status, stream);
  } catch (const std::exception& ex) {
    return fail(B200_NOALLOC_ECUDA, ex.what());
  }
  return B200_NOALLOC_OK;
}

extern "C" const char* b200_gemm_bf16_noalloc_last_error(void) { return g_last_error; }

extern "C" int b200_gemm_bf16_noalloc_status(unsigned int* out) {
  if (!out) return fail(B200_NOALLOC_EINVAL, "null output pointer");
  Region* r = nullptr;
  int rc = region_for_current_device(&r);
  if (rc != B200_NOALLOC_OK) return rc;
  cudaError_t e = cudaMemcpy(out, r->status, sizeof(unsigned int), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? B200_NOALLOC_OK : fail_cuda("cudaMemcpy(status)", e);
}

extern "C" int b200_gemm_bf16_noalloc_reset(cudaStream_t stream) {
  Region* r = nullptr;
  int rc = region_for_current_device(&r);
  if (rc != B200_NOALLOC_OK) return rc;
  cudaError_t e = cudaMemsetAsync(r->counters, 0, sizeof(int) * B200_NOALLOC_MAX_TILES, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(r->status, 0, sizeof(unsigned int) * 16, stream);
  return e == cudaSuccess ? B200_NOALLOC_OK : fail_cuda("cudaMemsetAsync", e);
}
