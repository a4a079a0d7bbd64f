// ssu.cu - single-token selective state update (ssu/forward_kernel.py:6-78),
// with the optional D-skip / z-gate of modules/ssm.py:199-202 fused.
//
// One CTA (4 warps) per (batch, head). The (P, N) state is streamed once: each
// row p is covered by TPR lanes holding E consecutive state elements, loaded and
// stored with 16-byte (or 8-byte) streaming accesses; UNR rows per thread are in
// flight before any is consumed. y[p] is a shuffle reduction over the row's lanes.
#include "common.cuh"
#include "kernels.h"

namespace ssdb200 {

template <typename S, int E> struct StateVec;
template <> struct StateVec<float, 4> {
  static __device__ __forceinline__ void load(const float* p, float* v) {
    float4 a = __ldcs(reinterpret_cast<const float4*>(p));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  }
  static __device__ __forceinline__ void store(float* p, const float* v) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
  }
};
template <> struct StateVec<float, 8> {
  static __device__ __forceinline__ void load(const float* p, float* v) {
    StateVec<float, 4>::load(p, v);
    StateVec<float, 4>::load(p + 4, v + 4);
  }
  static __device__ __forceinline__ void store(float* p, const float* v) {
    StateVec<float, 4>::store(p, v);
    StateVec<float, 4>::store(p + 4, v + 4);
  }
};
template <> struct StateVec<__nv_bfloat16, 4> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* v) {
    uint2 a = __ldcs(reinterpret_cast<const uint2*>(p));
    float2 f0 = unpack2<__nv_bfloat16>(a.x), f1 = unpack2<__nv_bfloat16>(a.y);
    v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float* v) {
    uint2 a;
    a.x = pack2<__nv_bfloat16>(v[0], v[1]);
    a.y = pack2<__nv_bfloat16>(v[2], v[3]);
    __stcs(reinterpret_cast<uint2*>(p), a);
  }
};
template <> struct StateVec<__nv_bfloat16, 8> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* v) {
    uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
    float2 f0 = unpack2<__nv_bfloat16>(a.x), f1 = unpack2<__nv_bfloat16>(a.y);
    float2 f2 = unpack2<__nv_bfloat16>(a.z), f3 = unpack2<__nv_bfloat16>(a.w);
    v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
    v[4] = f2.x; v[5] = f2.y; v[6] = f3.x; v[7] = f3.y;
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float* v) {
    uint4 a;
    a.x = pack2<__nv_bfloat16>(v[0], v[1]);
    a.y = pack2<__nv_bfloat16>(v[2], v[3]);
    a.z = pack2<__nv_bfloat16>(v[4], v[5]);
    a.w = pack2<__nv_bfloat16>(v[6], v[7]);
    __stcs(reinterpret_cast<uint4*>(p), a);
  }
};

__device__ __forceinline__ float load_dt_any(const void* p, int dtype, long long i) {
  if (dtype == SSD_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == SSD_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// NS: dstate (64, 128 or 256). TPR lanes per state row, E elements per lane.
template <typename T, typename S, int NS>
__global__ void __launch_bounds__(128) ssu_kernel(const T* __restrict__ u, const float* __restrict__ A,
                                                  const T* __restrict__ Bm, const T* __restrict__ Cm,
                                                  const void* __restrict__ dr, int dt_dtype,
                                                  const float* __restrict__ bias, S* __restrict__ h,
                                                  T* __restrict__ y, const float* __restrict__ D,
                                                  const T* __restrict__ z, int H, int P, int G, int use_sp,
                                                  float dmin, float dmax) {
  constexpr int TPR = NS >= 128 ? 32 : NS / 4;
  constexpr int E = NS / TPR;
  constexpr int RPW = 32 / TPR;        // rows per warp per pass
  constexpr int RPP = 4 * RPW;         // rows per pass (4 warps)
  constexpr int UNR = (E == 8 || sizeof(S) == 2) ? 4 : 8;
  const int bh = blockIdx.x;
  const int b = bh / H, hd = bh - b * H;
  const int g = hd / (H / G);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane % TPR, rsub = lane / TPR;

  float d = load_dt_any(dr, dt_dtype, bh);
  if (bias) d += bias[hd];
  d = dt_transform(d, use_sp, dmin, dmax);
  const float dA = expf(A[hd] * d);

  float bd[E], cc[E];
  const long long bgo = ((long long)b * G + g) * NS + sub * E;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    bd[e] = Ld<T>::f(Bm + bgo + e) * d;
    cc[e] = Ld<T>::f(Cm + bgo + e);
  }
  S* hb = h + (long long)bh * P * NS;
  const T* ub = u + (long long)bh * P;

  for (int p0 = 0; p0 < P; p0 += RPP * UNR) {
    float hv[UNR][E];
    float xv[UNR];
#pragma unroll
    for (int q = 0; q < UNR; ++q) {
      const int p = p0 + q * RPP + warp * RPW + rsub;
      if (p < P) {
        StateVec<S, E>::load(hb + (long long)p * NS + sub * E, hv[q]);
        xv[q] = Ld<T>::f(ub + p);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) hv[q][e] = 0.f;
        xv[q] = 0.f;
      }
    }
#pragma unroll
    for (int q = 0; q < UNR; ++q) {
      const int p = p0 + q * RPP + warp * RPW + rsub;
      float part = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        hv[q][e] = hv[q][e] * dA + bd[e] * xv[q];
        part = fmaf(hv[q][e], cc[e], part);
      }
      if (p < P) StateVec<S, E>::store(hb + (long long)p * NS + sub * E, hv[q]);
#pragma unroll
      for (int off = TPR / 2; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
      if (sub == 0 && p < P) {
        float yv = part;
        if (D) yv = fmaf(D[hd * P + p], xv[q], yv);
        if (z) yv *= silu(Ld<T>::f(z + (long long)bh * P + p));
        y[(long long)bh * P + p] = from_f32<T>(yv);
      }
    }
  }
}

// Any dstate: one warp per row, lanes stride over the state; B*dt and C staged in
// shared memory (dstate <= 1024).
template <typename T, typename S>
__global__ void __launch_bounds__(128) ssu_generic_kernel(const T* __restrict__ u, const float* __restrict__ A,
                                                          const T* __restrict__ Bm, const T* __restrict__ Cm,
                                                          const void* __restrict__ dr, int dt_dtype,
                                                          const float* __restrict__ bias, S* __restrict__ h,
                                                          T* __restrict__ y, const float* __restrict__ D,
                                                          const T* __restrict__ z, int H, int P, int N, int G,
                                                          int use_sp, float dmin, float dmax) {
  __shared__ float sb[1024], sc[1024];
  const int bh = blockIdx.x;
  const int b = bh / H, hd = bh - b * H;
  const int g = hd / (H / G);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float d = load_dt_any(dr, dt_dtype, bh);
  if (bias) d += bias[hd];
  d = dt_transform(d, use_sp, dmin, dmax);
  const float dA = expf(A[hd] * d);
  for (int n = threadIdx.x; n < N; n += 128) {
    sb[n] = Ld<T>::f(Bm + ((long long)b * G + g) * N + n) * d;
    sc[n] = Ld<T>::f(Cm + ((long long)b * G + g) * N + n);
  }
  __syncthreads();
  for (int p = warp; p < P; p += 4) {
    const float x = Ld<T>::f(u + (long long)bh * P + p);
    S* row = h + ((long long)bh * P + p) * N;
    float part = 0.f;
    for (int n = lane; n < N; n += 32) {
      float v = to_f32<S>(row[n]) * dA + sb[n] * x;
      row[n] = from_f32<S>(v);
      part = fmaf(v, sc[n], part);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    if (lane == 0) {
      float yv = part;
      if (D) yv = fmaf(D[hd * P + p], x, yv);
      if (z) yv *= silu(Ld<T>::f(z + (long long)bh * P + p));
      y[(long long)bh * P + p] = from_f32<T>(yv);
    }
  }
}

template <typename T, typename S>
static cudaError_t ssu_launch_ts(const void* u, const float* A, const void* B, const void* C, const void* dr,
                                 const float* bias, void* h, void* y, const float* D, const void* z, int b, int H,
                                 int P, int N, int G, int dt_dtype, int use_sp, float dmin, float dmax,
                                 cudaStream_t s) {
  dim3 grid((unsigned)(b * H));
#define SSU_ARGS                                                                                           \
  (const T*)u, A, (const T*)B, (const T*)C, dr, dt_dtype, bias, (S*)h, (T*)y, D, (const T*)z, H, P, G, use_sp, \
      dmin, dmax
  // The vectorised kernels need 16-byte aligned rows of (E * sizeof(S)) bytes.
  const bool aligned = ((reinterpret_cast<uintptr_t>(h) & 15u) == 0);
  if (aligned && N == 128) ssu_kernel<T, S, 128><<<grid, 128, 0, s>>>(SSU_ARGS);
  else if (aligned && N == 64) ssu_kernel<T, S, 64><<<grid, 128, 0, s>>>(SSU_ARGS);
  else if (aligned && N == 256) ssu_kernel<T, S, 256><<<grid, 128, 0, s>>>(SSU_ARGS);
  else
    ssu_generic_kernel<T, S><<<grid, 128, 0, s>>>((const T*)u, A, (const T*)B, (const T*)C, dr, dt_dtype, bias,
                                                  (S*)h, (T*)y, D, (const T*)z, H, P, N, G, use_sp, dmin, dmax);
#undef SSU_ARGS
  return cudaGetLastError();
}

template <typename T>
static cudaError_t ssu_launch_t(int h_dtype, const void* u, const float* A, const void* B, const void* C,
                                const void* dr, const float* bias, void* h, void* y, const float* D, const void* z,
                                int b, int H, int P, int N, int G, int dt_dtype, int use_sp, float dmin, float dmax,
                                cudaStream_t s) {
  if (h_dtype == SSD_F32)
    return ssu_launch_ts<T, float>(u, A, B, C, dr, bias, h, y, D, z, b, H, P, N, G, dt_dtype, use_sp, dmin, dmax, s);
  if (h_dtype == SSD_BF16)
    return ssu_launch_ts<T, __nv_bfloat16>(u, A, B, C, dr, bias, h, y, D, z, b, H, P, N, G, dt_dtype, use_sp, dmin,
                                           dmax, s);
  return cudaErrorInvalidValue;
}

cudaError_t launch_ssu(const void* u, const float* A, const void* B, const void* C, const void* dr,
                       const float* bias, void* h, void* y, const float* D, const void* z, int b, int H, int P,
                       int N, int G, int x_dtype, int dt_dtype, int h_dtype, int y_dtype, int use_sp, float dmin,
                       float dmax, cudaStream_t s) {
  if (y_dtype != x_dtype) return cudaErrorInvalidValue;
  switch (x_dtype) {
    case SSD_F32:
      return ssu_launch_t<float>(h_dtype, u, A, B, C, dr, bias, h, y, D, z, b, H, P, N, G, dt_dtype, use_sp, dmin,
                                 dmax, s);
    case SSD_BF16:
      return ssu_launch_t<__nv_bfloat16>(h_dtype, u, A, B, C, dr, bias, h, y, D, z, b, H, P, N, G, dt_dtype, use_sp,
                                         dmin, dmax, s);
    case SSD_F16:
      return ssu_launch_t<__half>(h_dtype, u, A, B, C, dr, bias, h, y, D, z, b, H, P, N, G, dt_dtype, use_sp, dmin,
                                  dmax, s);
  }
  return cudaErrorInvalidValue;
}

SSDB200_DEFINE_ERROR_FETCH(fetch_error_ssu)

}  // namespace ssdb200
