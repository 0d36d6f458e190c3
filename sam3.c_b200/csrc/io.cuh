// io.cuh - four-element vector loads / stores of f32, bf16 and f16 rows
// with f32 arithmetic (used by the HBM-bound kernels).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "sam3cu_internal.h"

namespace s3 {

template <int T>
struct IO;
template <>
struct IO<kF32> {
  static __device__ __forceinline__ float4 ld4(const void* p, int64_t i) {
    return *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
  }
  static __device__ __forceinline__ void st4(void* p, int64_t i, float4 v) {
    *reinterpret_cast<float4*>(static_cast<float*>(p) + i) = v;
  }
};
template <>
struct IO<kBF16> {
  static __device__ __forceinline__ float4 ld4(const void* p, int64_t i) {
    uint2 r = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p) + i);
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&r.x);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&r.y);
    float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
  }
  static __device__ __forceinline__ void st4(void* p, int64_t i, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 r;
    r.x = *reinterpret_cast<uint32_t*>(&a);
    r.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p) + i) = r;
  }
};
template <>
struct IO<kF16> {
  static __device__ __forceinline__ float4 ld4(const void* p, int64_t i) {
    uint2 r = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p) + i);
    __half2 a = *reinterpret_cast<__half2*>(&r.x);
    __half2 b = *reinterpret_cast<__half2*>(&r.y);
    float2 fa = __half22float2(a), fb = __half22float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
  }
  static __device__ __forceinline__ void st4(void* p, int64_t i, float4 v) {
    __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    uint2 r;
    r.x = *reinterpret_cast<uint32_t*>(&a);
    r.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(static_cast<__half*>(p) + i) = r;
  }
};

}  // namespace s3
