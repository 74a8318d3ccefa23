// Shared definitions for the dion_b200 CUDA extension.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace bdion {

// Status codes written to the host-mapped status word when a device-side
// wait gives up. The host reads the word without synchronising
// (dion_b200.ops.check_status) and raises.
enum StatusCode : int {
  kStatusOk = 0,
  kStatusGemmProducerTimeout = 0x101,
  kStatusGemmMmaTimeout = 0x102,
  kStatusGemmEpilogueTimeout = 0x103,
  kStatusCommTimeout = 0x201,
  kStatusCholeskyNotPD = 0x301,
};

// Default limit for one bounded wait inside a kernel (2 s of wall clock).
constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;

int* status_device_ptr();  // host-mapped status word (device view)
uint64_t wait_limit_ns();

__device__ __forceinline__ void report_status(int* status, int code) {
  if (status != nullptr) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(status), "r"(code) : "memory");
  }
}

__device__ __forceinline__ float bf16_to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Load/store 8 consecutive elements (16 bytes for bf16, 32 bytes for fp32).
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float* v) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void store8(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
// One 16-byte store: 8 bf16 or 4 fp32 elements.
__device__ __forceinline__ void store8or4(__nv_bfloat16* p, const float* v) { store8(p, v); }
__device__ __forceinline__ void store8or4(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

}  // namespace bdion
