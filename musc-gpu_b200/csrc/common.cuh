// Shared helpers for the MuSc B200 library: status codes, the thread-local
// error string behind musc_b200_last_error(), and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "../../include/musc_b200.h"

namespace musc {

// Set the thread-local error message and return the status code.
int fail(int status, const std::string& message);

// Map a CUDA runtime error to MUSC_B200_ERR_CUDA with a message naming the call.
int cuda_fail(cudaError_t err, const char* what);

// Enqueue-time check after a kernel launch.
inline int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err, what);
  return MUSC_B200_OK;
}

// The device behind the current context must be sm_100 (B200 family).
int require_sm100(void);

// Number of SMs of the current device (cached per device).
int sm_count(void);

// Maximum dynamic shared memory per block with opt-in (cached per device).
int smem_optin(void);

// Device address of the error word that kernels set when a bounded wait
// expires (cached per device; nullptr on failure).
int* device_error_ptr(void);

}  // namespace musc

#define MUSC_TRY(expr)                          \
  do {                                          \
    int musc_status_ = (expr);                  \
    if (musc_status_ != MUSC_B200_OK) return musc_status_; \
  } while (0)

#define MUSC_CUDA(expr)                                   \
  do {                                                    \
    cudaError_t musc_err_ = (expr);                       \
    if (musc_err_ != cudaSuccess) return musc::cuda_fail(musc_err_, #expr); \
  } while (0)

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
namespace musc {

template <typename T>
__device__ __forceinline__ float4 load4(const T* p);

template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
  uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
  __half2 a = *reinterpret_cast<__half2*>(&raw.x);
  __half2 b = *reinterpret_cast<__half2*>(&raw.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

// Same conversions from shared memory (plain loads).
__device__ __forceinline__ float4 load4_shared(const float* p) { return *reinterpret_cast<const float4*>(p); }

__device__ __forceinline__ float4 load4_shared(const __half* p) {
  uint2 raw = *reinterpret_cast<const uint2*>(p);
  float2 fa = __half22float2(*reinterpret_cast<__half2*>(&raw.x));
  float2 fb = __half22float2(*reinterpret_cast<__half2*>(&raw.y));
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

__device__ __forceinline__ float4 load4_shared(const __nv_bfloat16* p) {
  uint2 raw = *reinterpret_cast<const uint2*>(p);
  float2 fa = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&raw.x));
  float2 fb = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&raw.y));
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

}  // namespace musc
