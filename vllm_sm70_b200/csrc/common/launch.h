// Kernel launches with programmatic dependent launch (PDL).
//
// A kernel launched through launch_pdl may begin while the previous kernel on
// the stream is still running: its CTAs are scheduled as soon as every CTA of
// the previous grid has executed griddepcontrol.launch_dependents (or exited).
// Contract for every kernel launched this way:
//   * pdl_wait() before reading anything an earlier kernel wrote and before
//     writing anything an earlier kernel may still read (it returns once the
//     previous grid has completed and its memory is visible);
//   * work that touches only data no earlier kernel in the stream writes
//     (weights, tensor-map descriptors, shared memory / TMEM set-up) may run
//     before it -- that is the overlap PDL buys;
//   * pdl_trigger() once this kernel may let its dependent start launching
//     (early is fine: a dependent only starts after all of this grid's CTAs
//     are resident and it waits for this grid's completion itself).
// pdl_wait / pdl_trigger are no-ops for a kernel launched without the
// attribute. VLLM_B200_PDL=0 launches everything without it.
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>
#include <stdexcept>
#include <string>
#include <utility>

namespace b200 {

#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#endif

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VLLM_B200_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

// cudaFuncSetAttribute applies to the current device only: a process that
// drives several GPUs sets the dynamic shared-memory limit once per device.
// `done` is one flag array per kernel instantiation (a function-local static).
constexpr int kMaxDevices = 64;
template <typename Kernel>
inline void set_smem_attr_once(Kernel kernel, int bytes, bool (&done)[kMaxDevices],
                               const char* what) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices)
    throw std::runtime_error(std::string(what) + ": device index out of range");
  if (done[dev]) return;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + " attribute: " + cudaGetErrorString(e));
  done[dev] = true;
}

// cudaLaunchKernelEx with the programmatic-serialization attribute (when
// enabled) plus up to one extra attribute (e.g. a cluster shape).
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, const cudaLaunchAttribute* extra, Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (extra != nullptr) attr[n++] = *extra;
  lc.attrs = attr;
  lc.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&lc, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) throw std::runtime_error(std::string("kernel launch: ") + cudaGetErrorString(e));
}

}  // namespace b200
