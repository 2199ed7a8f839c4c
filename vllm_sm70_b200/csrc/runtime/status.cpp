// Per-device status word shared by every kernel that has a bounded wait.
// Allocated once per device on first use (outside graph capture: the engine
// touches it at start-up through `_b200_C::init_device`).
#include <cuda_runtime.h>
#include <mutex>
#include <stdexcept>
#include <string>

#include "ops_api.h"

namespace b200 {

unsigned int* device_status_ptr(int device) {
  static std::mutex mu;
  static unsigned int* ptrs[64] = {nullptr};
  if (device < 0 || device >= 64) throw std::runtime_error("device index out of range");
  std::lock_guard<std::mutex> g(mu);
  if (!ptrs[device]) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, 64);
    if (e == cudaSuccess) e = cudaMemset(p, 0, 64);
    cudaSetDevice(prev);
    if (e != cudaSuccess)
      throw std::runtime_error(std::string("status word allocation failed: ") +
                               cudaGetErrorString(e));
    ptrs[device] = static_cast<unsigned int*>(p);
  }
  return ptrs[device];
}

}  // namespace b200
