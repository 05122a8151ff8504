// Shared helpers of the theria sm_100a kernels: element conversion, the
// problem descriptor every kernel receives, and launch-error plumbing.
#pragma once

#include <cstdio>
#include <cstdlib>

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <atomic>

#include "../../include/theria_sdpa.h"

namespace theria {

// One (B, H, T, M, D) problem on contiguous [B, H, rows, D] tensors.
struct Shape {
  int64_t B, H, T, M, D;
  float scale;
  int causal;
};

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Store a float into a buffer whose element type is chosen at run time.
__device__ __forceinline__ void store_any(void* base, int64_t idx, int dtype, float x) {
  if (dtype == THERIA_F32) {
    static_cast<float*>(base)[idx] = x;
  } else if (dtype == THERIA_F16) {
    static_cast<__half*>(base)[idx] = __float2half_rn(x);
  } else {
    static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(x);
  }
}

__device__ __forceinline__ float load_any(const void* base, int64_t idx, int dtype) {
  if (dtype == THERIA_F32) return static_cast<const float*>(base)[idx];
  if (dtype == THERIA_F16) return __half2float(static_cast<const __half*>(base)[idx]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// Process-wide count of kernels this library has launched (all devices).
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> n{0};
  return n;
}

// Call right after each kernel launch: counts it and maps the launch error.
// With THERIA_DEBUG set in the environment the CUDA error text goes to stderr.
inline int launch_status() {
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return THERIA_OK;
  static const bool debug = std::getenv("THERIA_DEBUG") != nullptr;
  if (debug) std::fprintf(stderr, "theria: kernel launch failed: %s\n", cudaGetErrorString(e));
  return THERIA_ERR_LAUNCH;
}

inline int64_t elem_size(int dtype) { return dtype == THERIA_F32 ? 4 : 2; }

// Device-side error word (one per device that loads the library); a kernel
// whose bounded wait runs out sets it instead of spinning forever.  The
// library is one translation unit, so a plain __device__ variable serves.
__device__ int g_device_error = 0;

}  // namespace theria
