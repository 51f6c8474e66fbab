// Host-side error helpers for the plain-C++ launchers (no torch headers here, so the
// kernel translation units stay cheap to compile).  Failures throw std::runtime_error,
// which the torch bindings surface as Python RuntimeError.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <utility>

#define B200_REQUIRE(cond, msg)                                                           \
  do {                                                                                    \
    if (!(cond))                                                                          \
      throw std::runtime_error(std::string("b200: ") + (msg) + " [" + __FILE__ + ":" +    \
                               std::to_string(__LINE__) + "]");                          \
  } while (0)

#define B200_CUDA_OK(expr)                                                                \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    if (_e != cudaSuccess)                                                                \
      throw std::runtime_error(std::string("b200: CUDA error: ") + cudaGetErrorString(_e) + \
                               " [" + __FILE__ + ":" + std::to_string(__LINE__) + "]");  \
  } while (0)

namespace b200 {
// Number of kernels this library has launched (or recorded into a CUDA graph) in this process.
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> c{0};
  return c;
}
inline void count_launch(int n = 1) { launch_counter().fetch_add(n, std::memory_order_relaxed); }

// Raise a kernel's dynamic shared-memory limit once per (kernel address, device).
inline void ensure_dynamic_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  B200_CUDA_OK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (done.insert({kernel, dev}).second) {
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
      done.erase({kernel, dev});
      B200_CUDA_OK(e);
    }
  }
}

inline int num_sms() {
  static int n = -1;
  if (n < 0) {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n = v > 0 ? v : 148;
  }
  return n;
}
}  // namespace b200
