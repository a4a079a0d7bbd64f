// ssm_conv.cu - the SSM layer's prefill front end between the input projection and the
// scan (modules/ssm.py:112-134, inference/ssm_cache.py:10-36):
//   conv_ctx = the last K pre-activation inputs of every (row, channel) before the row's
//              length (zeros where the row is shorter), the decode cache;
//   s        = silu(hBC), rounded to the activation type as F.silu on such a tensor is;
//   out[t,c] = bias[c] + sum_k w[c,k] s[t-K+1+k, c]   (depthwise causal conv, zero padding);
//   x, B, C  = out split along the channels into (b, L, inner), (b, L, G*N), (b, L, G*N).
// The reference runs these as separate torch passes over (b, conv_dim, L) transposes; here
// one pass reads hBC (any token stride, e.g. a slice of the projection output) and writes
// the three contiguous tensors the scan takes.
//
// Layout of the work: a thread owns VEC adjacent channels (one 8-byte load per token) and
// walks a block of TB tokens, keeping the previous K-1 activations in registers; a warp's
// loads and stores are contiguous along the channels.
#include "common.cuh"
#include "kernels.h"

namespace ssdb200 {

template <typename T> __device__ __forceinline__ float round_to(float v) { return to_f32(from_f32<T>(v)); }
// silu(v) = v / (1 + exp(-v)) with the fast exponential and division (relative error a few
// 1e-7), rounded to T as F.silu on a T tensor rounds. exp(-v) = inf gives -0.
template <typename T> __device__ __forceinline__ float silu_t(float v) {
  return round_to<T>(__fdividef(v, 1.f + __expf(-v)));
}
// silu of a pair of 16-bit values in the 16-bit type itself: h = v/2 (exact),
// silu = h + h tanh(h) with one packed MUFU tanh for both values and a packed FMA. The
// result is a 16-bit value as the reference's F.silu on a 16-bit tensor gives, within
// about an ulp for v >= 0; for v << 0 (tanh near -1) the absolute error stays below
// ~3e-3, the size of the 16-bit rounding of values near 1.
template <typename T16> __device__ __forceinline__ uint32_t silu2(uint32_t w);
template <> __device__ __forceinline__ uint32_t silu2<__nv_bfloat16>(uint32_t w) {
  const __nv_bfloat162 h = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&w), __float2bfloat162_rn(0.5f));
  uint32_t hw = *reinterpret_cast<const uint32_t*>(&h), tw;
  asm("tanh.approx.bf16x2 %0, %1;" : "=r"(tw) : "r"(hw));
  const __nv_bfloat162 r = __hfma2(h, *reinterpret_cast<const __nv_bfloat162*>(&tw), h);
  return *reinterpret_cast<const uint32_t*>(&r);
}
template <> __device__ __forceinline__ uint32_t silu2<__half>(uint32_t w) {
  const __half2 h = __hmul2(*reinterpret_cast<const __half2*>(&w), __float2half2_rn(0.5f));
  uint32_t hw = *reinterpret_cast<const uint32_t*>(&h), tw;
  asm("tanh.approx.f16x2 %0, %1;" : "=r"(tw) : "r"(hw));
  const __half2 r = __hfma2(h, *reinterpret_cast<const __half2*>(&tw), h);
  return *reinterpret_cast<const uint32_t*>(&r);
}

template <typename T> struct Vec8;  // 8 bytes of T
template <> struct Vec8<float> {
  static constexpr int N = 2;
  static __device__ __forceinline__ void load(const float* p, float* v) {
    const float2 a = *reinterpret_cast<const float2*>(p);
    v[0] = a.x; v[1] = a.y;
  }
  static __device__ __forceinline__ void store(float* p, const float* v) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  }
  static __device__ __forceinline__ void load_silu(const float* p, float* v) {
    load(p, v);
    v[0] = silu_t<float>(v[0]);
    v[1] = silu_t<float>(v[1]);
  }
};
template <typename T16> struct Vec8_16 {
  static constexpr int N = 4;
  static __device__ __forceinline__ void load(const T16* p, float* v) {
    const uint2 a = *reinterpret_cast<const uint2*>(p);
    const float2 f0 = unpack2<T16>(a.x), f1 = unpack2<T16>(a.y);
    v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
  }
  static __device__ __forceinline__ void store(T16* p, const float* v) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack2<T16>(v[0], v[1]), pack2<T16>(v[2], v[3]));
  }
  static __device__ __forceinline__ void load_silu(const T16* p, float* v) {
    const uint2 a = *reinterpret_cast<const uint2*>(p);
    const float2 f0 = unpack2<T16>(silu2<T16>(a.x)), f1 = unpack2<T16>(silu2<T16>(a.y));
    v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
  }
};
template <> struct Vec8<__nv_bfloat16> : Vec8_16<__nv_bfloat16> {};
template <> struct Vec8<__half> : Vec8_16<__half> {};

// Scalar access (VEC = 1): any alignment.
template <typename T, int VEC> struct Access {
  static __device__ __forceinline__ void load(const T* p, float* v) { Vec8<T>::load(p, v); }
  static __device__ __forceinline__ void load_silu(const T* p, float* v) { Vec8<T>::load_silu(p, v); }
  static __device__ __forceinline__ void store(T* p, const float* v) { Vec8<T>::store(p, v); }
};
template <typename T> struct Access<T, 1> {
  static __device__ __forceinline__ void load(const T* p, float* v) { v[0] = to_f32(p[0]); }
  static __device__ __forceinline__ void load_silu(const T* p, float* v) { v[0] = silu_t<T>(to_f32(p[0])); }
  static __device__ __forceinline__ void store(T* p, const float* v) { p[0] = from_f32<T>(v[0]); }
};

constexpr int kConvTB = 32;        // tokens per thread
constexpr int kConvU = 8;          // tokens loaded ahead (loads in flight per thread)
constexpr int kConvThreads = 128;  // threads per CTA (channel groups)

// grid: (channel groups / kConvThreads, token blocks, batch)
template <typename T, int VEC, int K, bool W4>
__global__ void __launch_bounds__(kConvThreads) ssm_conv_prefill_kernel(
    const T* __restrict__ hbc, long long row_stride, const float* __restrict__ w, const float* __restrict__ bias,
    T* __restrict__ x, T* __restrict__ Bo, T* __restrict__ Co, int L, int inner, int gn) {
  const int conv_dim = inner + 2 * gn;
  const int cg = blockIdx.x * kConvThreads + threadIdx.x;
  const int c0 = cg * VEC;
  if (c0 >= conv_dim) return;
  const int b = blockIdx.z;
  const int t0 = blockIdx.y * kConvTB;
  const int t1 = min(L, t0 + kConvTB);
  const T* in = hbc + (long long)b * L * row_stride + c0;

  // Weights of this thread's VEC channels: VEC x K contiguous floats. With K = 4 and a
  // 16-byte aligned array (W4) they are read as 16-byte pieces (a warp reads one
  // contiguous span); otherwise element-wise.
  float wk[K][VEC], bs[VEC];
  if constexpr (W4) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float4 q = *reinterpret_cast<const float4*>(w + (long long)(c0 + e) * 4);
      wk[0][e] = q.x; wk[1][e] = q.y; wk[2][e] = q.z; wk[3][e] = q.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e)
#pragma unroll
      for (int k = 0; k < K; ++k) wk[k][e] = w[(long long)(c0 + e) * K + k];
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) bs[e] = bias ? bias[c0 + e] : 0.f;
  // destination: which of x / B / C, and the channel inside it (VEC never straddles)
  T* dst;
  long long dstride;
  if (c0 < inner) {
    dst = x + (long long)b * L * inner + c0;
    dstride = inner;
  } else if (c0 < inner + gn) {
    dst = Bo + (long long)b * L * gn + (c0 - inner);
    dstride = gn;
  } else {
    dst = Co + (long long)b * L * gn + (c0 - inner - gn);
    dstride = gn;
  }
  // window of activations s[t-K+1 .. t-1]
  float win[K > 1 ? K - 1 : 1][VEC];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const int t = t0 - (K - 1) + j;
    float v[VEC];
    if (t >= 0) {
      Access<T, VEC>::load_silu(in + (long long)t * row_stride, v);
#pragma unroll
      for (int e = 0; e < VEC; ++e) win[j][e] = v[e];
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) win[j][e] = 0.f;
    }
  }
  for (int tb = t0; tb < t1; tb += kConvU) {
    // kConvU tokens' loads first, then the dependent arithmetic
    float v[kConvU][VEC];
#pragma unroll
    for (int u = 0; u < kConvU; ++u) {
      if (tb + u < t1) {
        Access<T, VEC>::load_silu(in + (long long)(tb + u) * row_stride, v[u]);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[u][e] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kConvU; ++u) {
      float o[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float sv = v[u][e];
        float acc = bs[e];
#pragma unroll
        for (int k = 0; k < K - 1; ++k) acc = fmaf(wk[k][e], win[k][e], acc);
        o[e] = fmaf(wk[K - 1][e], sv, acc);
#pragma unroll
        for (int k = 0; k < K - 2; ++k) win[k][e] = win[k + 1][e];
        if (K > 1) win[K > 1 ? K - 2 : 0][e] = sv;
      }
      if (tb + u < t1) Access<T, VEC>::store(dst + (long long)(tb + u) * dstride, o);
    }
  }
}

// Tiled form for 16-byte aligned rows: the CTA first copies its tile, kConvTB tokens plus
// the K - 1 before them by 1 KB of channels, into shared memory with 16-byte cp.async
// copies (all in flight at once), then each thread runs the same register window over
// its VEC channels from shared memory. Grid: (channel KB blocks, token blocks, batch).
constexpr int kTileBytes = 1024;  // channels per CTA: 1 KB of the row
template <typename T, int K, bool W4>
__global__ void __launch_bounds__(kConvThreads) ssm_conv_prefill_tiled_kernel(
    const T* __restrict__ hbc, long long row_stride, const float* __restrict__ w, const float* __restrict__ bias,
    T* __restrict__ x, T* __restrict__ Bo, T* __restrict__ Co, T* __restrict__ ctx,
    const int64_t* __restrict__ lengths, int L, int inner, int gn) {
  constexpr int VEC = Vec8<T>::N;                   // channels a thread owns (8 bytes)
  constexpr int CPR = kTileBytes / sizeof(T);        // channels per CTA row
  constexpr int R = kConvTB + K - 1;                 // rows in the tile
  extern __shared__ __align__(16) uint8_t tile[];   // [R][kTileBytes]
  const int conv_dim = inner + 2 * gn;
  const int b = blockIdx.z, t0 = blockIdx.y * kConvTB;
  const int cb = blockIdx.x * CPR;                   // first channel of the CTA
  const int tid = threadIdx.x;
  const T* in = hbc + (long long)b * L * row_stride + cb;
  // copy in: 16-byte pieces; rows before token 0 are zeros, pieces past conv_dim skipped
  constexpr int PPR = kTileBytes / 16;
  for (int q = tid; q < R * PPR; q += kConvThreads) {
    const int r = q / PPR, pc = q % PPR;
    const int t = t0 - (K - 1) + r;
    const int c = pc * (16 / (int)sizeof(T));
    uint8_t* dsts = tile + r * kTileBytes + pc * 16;
    if (t >= 0 && t < L && cb + c < conv_dim) {
      const T* src = in + (long long)t * row_stride + c;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dsts)),
                   "l"(src)
                   : "memory");
    } else if (t < 0) {
      *reinterpret_cast<uint4*>(dsts) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  const int c0 = cb + tid * VEC;
  if (c0 >= conv_dim) return;
  if (ctx) {
    // decode cache (inference/ssm_cache.py:22-34): the CTA whose tile holds the row's last
    // valid token has all K context rows, unactivated, in shared memory (rows before
    // token 0 are zeros); an empty row's cache is written by the first token block.
    const long long len = lengths ? lengths[b] : L;
    const long long last = (len < L ? len : L) - 1;
    if ((last >= t0 && last < t0 + kConvTB) || (last < 0 && blockIdx.y == 0)) {
      T* cp = ctx + ((long long)b * conv_dim + c0) * K;
#pragma unroll
      for (int e = 0; e < VEC; ++e)
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const long long t = len - K + k;
          T v = from_f32<T>(0.f);
          if (t >= 0 && t <= last) v = reinterpret_cast<const T*>(tile + (int)(t - (t0 - (K - 1))) * kTileBytes)[tid * VEC + e];
          cp[e * K + k] = v;
        }
    }
  }
  float wk[K][VEC], bs[VEC];
  if constexpr (W4) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float4 q = *reinterpret_cast<const float4*>(w + (long long)(c0 + e) * 4);
      wk[0][e] = q.x; wk[1][e] = q.y; wk[2][e] = q.z; wk[3][e] = q.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e)
#pragma unroll
      for (int k = 0; k < K; ++k) wk[k][e] = w[(long long)(c0 + e) * K + k];
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) bs[e] = bias ? bias[c0 + e] : 0.f;
  T* dst;
  long long dstride;
  if (c0 < inner) {
    dst = x + (long long)b * L * inner + c0;
    dstride = inner;
  } else if (c0 < inner + gn) {
    dst = Bo + (long long)b * L * gn + (c0 - inner);
    dstride = gn;
  } else {
    dst = Co + (long long)b * L * gn + (c0 - inner - gn);
    dstride = gn;
  }
  const T* srow = reinterpret_cast<const T*>(tile) + tid * VEC;
  float win[K > 1 ? K - 1 : 1][VEC];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) Vec8<T>::load_silu(srow + j * CPR, win[j]);
  const int n = min(kConvTB, L - t0);
#pragma unroll 4
  for (int u = 0; u < n; ++u) {
    float sv[VEC], o[VEC];
    Vec8<T>::load_silu(srow + (u + K - 1) * CPR, sv);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      float acc = bs[e];
#pragma unroll
      for (int k = 0; k < K - 1; ++k) acc = fmaf(wk[k][e], win[k][e], acc);
      o[e] = fmaf(wk[K - 1][e], sv[e], acc);
#pragma unroll
      for (int k = 0; k < K - 2; ++k) win[k][e] = win[k + 1][e];
      if (K > 1) win[K > 1 ? K - 2 : 0][e] = sv[e];
    }
    Vec8<T>::store(dst + (long long)(t0 + u) * dstride, o);
  }
}

// conv_ctx[b, c, k] = hbc[b, len_b - K + k, c] when 0 <= len_b - K + k < len_b, else 0
// (inference/ssm_cache.py:22-34; without lengths len_b = L). One thread per (b, c).
template <typename T>
__global__ void ssm_conv_ctx_kernel(const T* __restrict__ hbc, long long row_stride,
                                    const int64_t* __restrict__ lengths, T* __restrict__ ctx, int B, int L,
                                    int conv_dim, int K) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * conv_dim) return;
  const int b = (int)(i / conv_dim), c = (int)(i % conv_dim);
  long long len = lengths ? lengths[b] : L;
  for (int k = 0; k < K; ++k) {
    const long long t = len - K + k;
    T v = from_f32<T>(0.f);
    if (t >= 0 && t < len && t < L) v = hbc[((long long)b * L + t) * row_stride + c];
    ctx[((long long)b * conv_dim + c) * K + k] = v;
  }
}

template <typename T, int K, bool W4>
static cudaError_t conv_tiled_k(const T* hbc, long long rs, const float* w, const float* bias, T* x, T* Bo, T* Co,
                                T* ctx, const int64_t* lengths, int b, int L, int inner, int gn, cudaStream_t s) {
  constexpr int CPR = kTileBytes / sizeof(T);
  const int smem = (kConvTB + K - 1) * kTileBytes;
  auto kern = ssm_conv_prefill_tiled_kernel<T, K, W4>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((inner + 2 * gn + CPR - 1) / CPR, (L + kConvTB - 1) / kConvTB, b);
  kern<<<grid, kConvThreads, smem, s>>>(hbc, rs, w, bias, x, Bo, Co, ctx, lengths, L, inner, gn);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t conv_tiled(const T* hbc, long long rs, const float* w, const float* bias, T* x, T* Bo, T* Co,
                              T* ctx, const int64_t* lengths, int b, int L, int inner, int gn, int K, cudaStream_t s) {
  if (K == 4 && reinterpret_cast<uintptr_t>(w) % 16 == 0)
    return conv_tiled_k<T, 4, true>(hbc, rs, w, bias, x, Bo, Co, ctx, lengths, b, L, inner, gn, s);
  switch (K) {
#define SSM_CONV_TK(KK) \
  case KK:              \
    return conv_tiled_k<T, KK, false>(hbc, rs, w, bias, x, Bo, Co, ctx, lengths, b, L, inner, gn, s);
    SSM_CONV_TK(1) SSM_CONV_TK(2) SSM_CONV_TK(3) SSM_CONV_TK(4) SSM_CONV_TK(5) SSM_CONV_TK(6) SSM_CONV_TK(7)
    SSM_CONV_TK(8)
#undef SSM_CONV_TK
  }
  return cudaErrorInvalidValue;
}

template <typename T, int VEC>
static cudaError_t conv_launch_k(const T* hbc, long long rs, const float* w, const float* bias, T* x, T* Bo, T* Co,
                                 int b, int L, int inner, int gn, int K, cudaStream_t s) {
  const int groups = (inner + 2 * gn) / VEC;
  dim3 grid((groups + kConvThreads - 1) / kConvThreads, (L + kConvTB - 1) / kConvTB, b);
  if (K == 4 && reinterpret_cast<uintptr_t>(w) % 16 == 0) {
    ssm_conv_prefill_kernel<T, VEC, 4, true><<<grid, kConvThreads, 0, s>>>(hbc, rs, w, bias, x, Bo, Co, L, inner, gn);
    return cudaGetLastError();
  }
  switch (K) {
#define SSM_CONV_K(KK)                                                                                        \
  case KK:                                                                                                    \
    ssm_conv_prefill_kernel<T, VEC, KK, false><<<grid, kConvThreads, 0, s>>>(hbc, rs, w, bias, x, Bo, Co, L, inner, \
                                                                          gn);                                  \
    break;
    SSM_CONV_K(1) SSM_CONV_K(2) SSM_CONV_K(3) SSM_CONV_K(4) SSM_CONV_K(5) SSM_CONV_K(6) SSM_CONV_K(7) SSM_CONV_K(8)
#undef SSM_CONV_K
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename T>
static cudaError_t conv_launch_t(const void* hbc, long long rs, const float* w, const float* bias, void* x, void* Bo,
                                 void* Co, void* ctx, const int64_t* lengths, int b, int L, int inner, int gn, int K,
                                 cudaStream_t s) {
  constexpr int V = Vec8<T>::N;
  // the 8-byte path needs 8-byte aligned rows and channel ranges that split on VEC
  const bool vec = (reinterpret_cast<uintptr_t>(hbc) % 8 == 0) && ((rs * (long long)sizeof(T)) % 8 == 0) &&
                   inner % V == 0 && gn % V == 0 && reinterpret_cast<uintptr_t>(x) % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(Bo) % 8 == 0 && reinterpret_cast<uintptr_t>(Co) % 8 == 0;
  // 16-byte aligned rows: the tiled kernel (cp.async copies in flight); else the direct one
  // (every 16-byte piece of a row then lies inside the row's conv_dim channels)
  const bool tiled = vec && reinterpret_cast<uintptr_t>(hbc) % 16 == 0 && (rs * (long long)sizeof(T)) % 16 == 0 &&
                     ((long long)(inner + 2 * gn) * sizeof(T)) % 16 == 0;
  if (tiled)  // writes the decode cache itself
    return conv_tiled<T>((const T*)hbc, rs, w, bias, (T*)x, (T*)Bo, (T*)Co, (T*)ctx, lengths, b, L, inner, gn, K, s);
  cudaError_t e = vec ? conv_launch_k<T, V>((const T*)hbc, rs, w, bias, (T*)x, (T*)Bo, (T*)Co, b, L, inner, gn, K, s)
                      : conv_launch_k<T, 1>((const T*)hbc, rs, w, bias, (T*)x, (T*)Bo, (T*)Co, b, L, inner, gn, K, s);
  if (e != cudaSuccess || ctx == nullptr) return e;
  const long long n = (long long)b * (inner + 2 * gn);
  ssm_conv_ctx_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const T*)hbc, rs, lengths, (T*)ctx, b, L,
                                                                      inner + 2 * gn, K);
  return cudaGetLastError();
}

// Decode step (modules/ssm.py:173-186 with inference/ssm_cache.py:38-43): per channel the
// cache window is shifted left by one and the new input appended (in place), then
//   out = round(round(sum_k round(w[c,k] silu(ctx[c,k]))) + bias[c])
// with every round() to the activation type, as the reference's torch ops on tensors of
// that type round (silu, the product, the sum, the bias add; identities for fp32), and
// out split into x (b, inner), B, C (b, gn). One thread per (row, channel).
template <typename T>
__global__ void ssm_conv_decode_kernel(const T* __restrict__ hnew, long long row_stride, T* __restrict__ ctx,
                                       const float* __restrict__ w, const float* __restrict__ bias,
                                       T* __restrict__ x, T* __restrict__ Bo, T* __restrict__ Co, int B, int inner,
                                       int gn, int K) {
  const int conv_dim = inner + 2 * gn;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * conv_dim) return;
  const int b = (int)(i / conv_dim), c = (int)(i % conv_dim);
  T* cp = ctx + i * K;
  T win[8];
  const T xn = hnew[(long long)b * row_stride + c];
  float acc = 0.f;
  if (sizeof(T) == 2 && K == 4 && (reinterpret_cast<uintptr_t>(ctx) & 7) == 0) {
    // the window of a channel is 8 bytes: one load, one store
    uint2 q = *reinterpret_cast<const uint2*>(cp);
    const T* o = reinterpret_cast<const T*>(&q);
    win[0] = o[1]; win[1] = o[2]; win[2] = o[3]; win[3] = xn;
    *reinterpret_cast<uint2*>(cp) = *reinterpret_cast<const uint2*>(win);
  } else {
    for (int k = 0; k + 1 < K; ++k) win[k] = cp[k + 1];
    win[K - 1] = xn;
    for (int k = 0; k < K; ++k) cp[k] = win[k];
  }
  for (int k = 0; k < K; ++k) {
    const float v = to_f32(win[k]);
    acc += round_to<T>(w[(long long)c * K + k] * silu_t<T>(v));
  }
  float o = round_to<T>(acc);
  if (bias) o = o + round_to<T>(bias[c]);
  const T ov = from_f32<T>(o);
  if (c < inner) x[(long long)b * inner + c] = ov;
  else if (c < inner + gn) Bo[(long long)b * gn + (c - inner)] = ov;
  else Co[(long long)b * gn + (c - inner - gn)] = ov;
}

cudaError_t launch_ssm_conv_decode(const void* hnew, long long row_stride, void* ctx, const float* w,
                                   const float* bias, void* x, void* Bo, void* Co, int b, int inner, int gn, int K,
                                   int dtype, cudaStream_t s) {
  const long long n = (long long)b * (inner + 2 * gn);
  const unsigned grid = (unsigned)((n + 255) / 256);
  switch (dtype) {
    case SSD_F32:
      ssm_conv_decode_kernel<float><<<grid, 256, 0, s>>>((const float*)hnew, row_stride, (float*)ctx, w, bias,
                                                         (float*)x, (float*)Bo, (float*)Co, b, inner, gn, K);
      break;
    case SSD_BF16:
      ssm_conv_decode_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          (const __nv_bfloat16*)hnew, row_stride, (__nv_bfloat16*)ctx, w, bias, (__nv_bfloat16*)x,
          (__nv_bfloat16*)Bo, (__nv_bfloat16*)Co, b, inner, gn, K);
      break;
    case SSD_F16:
      ssm_conv_decode_kernel<__half><<<grid, 256, 0, s>>>((const __half*)hnew, row_stride, (__half*)ctx, w, bias,
                                                          (__half*)x, (__half*)Bo, (__half*)Co, b, inner, gn, K);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_ssm_conv_prefill(const void* hbc, long long row_stride, const float* w, const float* bias,
                                    void* x, void* Bo, void* Co, void* ctx, const int64_t* lengths, int b, int L,
                                    int inner, int gn, int K, int dtype, cudaStream_t s) {
  switch (dtype) {
    case SSD_F32:
      return conv_launch_t<float>(hbc, row_stride, w, bias, x, Bo, Co, ctx, lengths, b, L, inner, gn, K, s);
    case SSD_BF16:
      return conv_launch_t<__nv_bfloat16>(hbc, row_stride, w, bias, x, Bo, Co, ctx, lengths, b, L, inner, gn, K, s);
    case SSD_F16:
      return conv_launch_t<__half>(hbc, row_stride, w, bias, x, Bo, Co, ctx, lengths, b, L, inner, gn, K, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ssdb200
