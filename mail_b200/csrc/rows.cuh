// 8-element vector helpers of the row kernels (gather, quant, combine,
// convert, decode prep): 16-byte loads and stores of bf16 / fp16 / fp32 rows
// through fp32 registers, and the per-token int8 quantisation arithmetic.
#pragma once
#include "common.cuh"

namespace moe {
namespace rows {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const __half* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void store8(__half* p, const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Copies 8 elements of T (16 bytes for 16-bit T, 32 bytes for fp32).
template <typename T>
__device__ __forceinline__ void copy8(const T* s, T* d) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(d) = *reinterpret_cast<const float4*>(s);
    *reinterpret_cast<float4*>(d + 4) = *reinterpret_cast<const float4*>(s + 4);
  } else {
    *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(s);
  }
}
template <typename T>
__device__ __forceinline__ void zero8(T* d) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(d) = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(d + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
  } else if constexpr (sizeof(T) == 2) {
    *reinterpret_cast<uint4*>(d) = make_uint4(0, 0, 0, 0);
  } else {
    *reinterpret_cast<uint2*>(d) = make_uint2(0, 0);
  }
}

// Per-token symmetric int8 quantisation of 8 values: q = clamp(rint(x * inv),
// -127, 127) with inv = 127 / absmax (one correctly rounded division per row,
// an exactly rounded multiply per element); inv = 0 for an all-zero row.
__device__ __forceinline__ uint2 quant8(const float (&v)[8], float inv) {
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int q = __float2int_rn(__fmul_rn(v[i], inv));
    q = max(-127, min(127, q));
    w[i >> 2] |= (uint32_t)(q & 0xff) << (8 * (i & 3));
  }
  return make_uint2(w[0], w[1]);
}

// Row scale s = absmax / 127 and quantisation multiplier 127 / absmax.
__device__ __forceinline__ void row_scales(float amax, float& scale, float& inv) {
  scale = __fdiv_rn(amax, 127.0f);
  inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
}

}  // namespace rows
}  // namespace moe
