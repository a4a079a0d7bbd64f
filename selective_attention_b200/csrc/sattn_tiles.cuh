// sattn_tiles.cuh - shared pieces of the CUDA-core selective-attention kernels (sattn.cu,
// sattn_train.cu): 8-element row loads in any input type, 64-row tiles staged into shared
// memory as fp32, and the half-warp reductions of the per-row softmax state.
#pragma once

#include "common.cuh"

namespace ssdb200 {
namespace {

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&o)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&o)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
template <typename T>
__device__ __forceinline__ void load8_16(const T* p, float (&o)[8]) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  const float2 a = unpack2<T>(w.x), b = unpack2<T>(w.y), c = unpack2<T>(w.z), d = unpack2<T>(w.w);
  o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  o[4] = c.x; o[5] = c.y; o[6] = d.x; o[7] = d.y;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&o)[8]) { load8_16(p, o); }
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&o)[8]) { load8_16(p, o); }

constexpr int kPT = 64;

template <typename T>
__device__ __forceinline__ void stage_rows64(float* dst, int ld, const T* src, int r0, int L, int D) {
  const int vpr = D >> 3, nv = kPT * vpr;  // <= 1024 vectors of 8
  float v[4][8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int vi = threadIdx.x + 256 * j, r = vi / vpr, c = (vi - r * vpr) * 8;
    if (vi < nv && r0 + r < L) {
      load8<T>(src + (long long)(r0 + r) * D + c, v[j]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = 0.f;
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int vi = threadIdx.x + 256 * j, r = vi / vpr, c = (vi - r * vpr) * 8;
    if (vi >= nv) continue;
    *reinterpret_cast<float4*>(dst + r * ld + c) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
    *reinterpret_cast<float4*>(dst + r * ld + c + 4) = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
  }
}

__device__ __forceinline__ float hw_max(float v) {
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ float hw_sum(float v) {
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

}  // namespace
}  // namespace ssdb200
