// Shared helpers for the visionattn CUDA library: status codes, the per-thread
// error string, launch checking and bf16/f32 load/store helpers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "../../include/visionattn.h"

namespace va {

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();

// Counts one kernel launch (reported by va_launch_count()).
void count_launch();

// Checks the launch that was just issued (invalid configuration, missing
// kernel image, …).  Asynchronous faults surface at the caller's next sync.
inline int check_launch(const char* what) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return VA_OK;
}

// One-time set-up that must run once on every device, such as
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize), which applies to the
// current device only.  run(f) calls f() with the calling thread's current
// device unless it already succeeded there; safe from several host threads.
// Devices with an index ≥ 64 run f() on every call.
class PerDeviceOnce {
 public:
  template <typename F>
  int run(F&& f) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(VA_ERR_LAUNCH, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return f();
    const uint64_t bit = 1ull << dev;
    if (done_.load(std::memory_order_acquire) & bit) return VA_OK;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_.load(std::memory_order_relaxed) & bit) return VA_OK;
    const int rc = f();
    if (rc == VA_OK) done_.fetch_or(bit, std::memory_order_release);
    return rc;
  }

 private:
  std::atomic<uint64_t> done_{0};
  std::mutex mu_;
};

inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

// Scalar element access for the templated SIMT kernels (f32 or bf16 storage,
// f32 arithmetic).
template <typename T> __device__ __forceinline__ float ld(const T* p);
template <> __device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T> __device__ __forceinline__ void st(T* p, float v);
template <> __device__ __forceinline__ void st<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}

template <typename T> __device__ __forceinline__ float ldg(const T* p);
template <> __device__ __forceinline__ float ldg<float>(const float* p) { return __ldg(p); }
template <> __device__ __forceinline__ float ldg<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

}  // namespace va

#define VA_CHECK_ARG(cond, ...)                                  \
  do {                                                           \
    if (!(cond)) return ::va::set_error(VA_ERR_SHAPE, __VA_ARGS__); \
  } while (0)
