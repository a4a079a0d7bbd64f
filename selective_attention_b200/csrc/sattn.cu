// sattn.cu - selective-attention decode step: the cache update and the pos-mode gated
// softmax attention of SelectiveMHA.step (modules/selective_attention.py:394-405,
// inference/selective_attn_cache.py:27-42) in one kernel.
//
// One CTA per (batch row, head). Its threads first write the new key, value and
// log-gate at slot write_idx, then stream the first write_idx + 1 cached keys and
// values once: a group of D/8 lanes owns one key (8 elements per lane, 16-byte loads),
// the score q.k*scale (+ the key's log-gate, except for the newest key, the token
// itself) goes through an online softmax per lane group, and the groups and warps are
// merged at the end. The step is bound by reading the cache from HBM.
#include <math.h>

#include "common.cuh"
#include "kernels.h"

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

// Merge the online-softmax state (m2, l2, a2) into (m, l, a).
__device__ __forceinline__ void merge(float& m, float& l, float (&a)[8], float m2, float l2, const float (&a2)[8]) {
  const float mn = fmaxf(m, m2);
  const float s1 = m == -INFINITY ? 0.f : expf(m - mn);
  const float s2 = m2 == -INFINITY ? 0.f : expf(m2 - mn);
  l = l * s1 + l2 * s2;
#pragma unroll
  for (int e = 0; e < 8; ++e) a[e] = a[e] * s1 + a2[e] * s2;
  m = mn;
}

constexpr int kWarps = 8;

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) sattn_decode_kernel(
    const T* __restrict__ q, const T* __restrict__ k_new, const T* __restrict__ v_new,
    const float* __restrict__ lg_new, T* kc, T* vc, float* lgc, long long widx, long long cap, T* __restrict__ out,
    int D, float scale) {
  __shared__ float sm_m[kWarps], sm_l[kWarps];
  __shared__ __align__(16) float sm_acc[kWarps][256];
  const long long bh = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  T* kb = kc + bh * cap * D;
  T* vb = vc + bh * cap * D;
  float* lgb = lgc + bh * cap;
  // SelectiveAttnCache.update_kv (selective_attn_cache.py:39-41)
  for (int d = tid; d < D; d += kWarps * 32) {
    kb[widx * D + d] = k_new[bh * D + d];
    vb[widx * D + d] = v_new[bh * D + d];
  }
  if (tid == 0) lgb[widx] = lg_new[bh];
  __syncthreads();  // the new slot is visible to the whole CTA

  const int W = (int)widx + 1;               // keys attended (write_idx after the update)
  const int L = D >> 3;                      // lanes per key
  const int KPW = 32 / L;                    // keys per warp per pass
  const int grp = lane / L, sl = lane - grp * L;
  float qv[8];
  load8<T>(q + bh * D + sl * 8, qv);
  float m = -INFINITY, l = 0.f, acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  const int stride = kWarps * KPW;
  // two passes per iteration: four 16-byte loads per lane in flight
  for (int j0 = warp * KPW; j0 < W; j0 += 2 * stride) {
    float kv[2][8], vv[2][8], g[2];
    int jj[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int j = j0 + u * stride + grp;
      jj[u] = j;
      if (j < W) {
        load8<T>(kb + (long long)j * D + sl * 8, kv[u]);
        load8<T>(vb + (long long)j * D + sl * 8, vv[u]);
        g[u] = j < W - 1 ? lgb[j] : 0.f;  // the token's own key is not gated (:127)
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) kv[u][e] = vv[u][e] = 0.f;
        g[u] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) d = fmaf(qv[e], kv[u][e], d);
      for (int off = 1; off < L; off <<= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      const float s = jj[u] < W ? d * scale + g[u] : -INFINITY;
      if (s != -INFINITY) {
        const float mn = fmaxf(m, s);
        const float a = m == -INFINITY ? 0.f : expf(m - mn);
        const float p = expf(s - mn);
        l = l * a + p;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(p, vv[u][e], acc[e] * a);
        m = mn;
      }
    }
  }
  // merge the key groups of the warp (lanes with the same slice)
  for (int off = L; off < 32; off <<= 1) {
    float a2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) a2[e] = __shfl_xor_sync(0xffffffffu, acc[e], off);
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
    merge(m, l, acc, m2, l2, a2);
  }
  if (grp == 0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) sm_acc[warp][sl * 8 + e] = acc[e];
    if (sl == 0) {
      sm_m[warp] = m;
      sm_l[warp] = l;
    }
  }
  __syncthreads();
  // merge the warps; thread d writes out[d]
  for (int d = tid; d < D; d += kWarps * 32) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w]);
    float Ls = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = sm_m[w] == -INFINITY ? 0.f : expf(sm_m[w] - M);
      Ls = fmaf(sm_l[w], f, Ls);
      O = fmaf(sm_acc[w][d], f, O);
    }
    out[bh * D + d] = from_f32<T>(O / Ls);
  }
}

template <typename T>
cudaError_t launch_t(const void* q, const void* k, const void* v, const float* lg, void* kc, void* vc, float* lgc,
                     long long widx, long long cap, void* out, long long bh, int D, float scale, cudaStream_t s) {
  sattn_decode_kernel<T><<<(unsigned)bh, kWarps * 32, 0, s>>>(
      (const T*)q, (const T*)k, (const T*)v, lg, (T*)kc, (T*)vc, lgc, widx, cap, (T*)out, D, scale);
  return cudaGetLastError();
}

}  // namespace

bool sattn_decode_supported(int D) { return D == 8 || D == 16 || D == 32 || D == 64 || D == 128 || D == 256; }

cudaError_t launch_sattn_decode(const void* q, const void* k, const void* v, const float* lg, void* kc, void* vc,
                                float* lgc, long long widx, long long cap, void* out, long long bh, int D,
                                float scale, int dtype, cudaStream_t s) {
  switch (dtype) {
    case SSD_F32: return launch_t<float>(q, k, v, lg, kc, vc, lgc, widx, cap, out, bh, D, scale, s);
    case SSD_BF16: return launch_t<__nv_bfloat16>(q, k, v, lg, kc, vc, lgc, widx, cap, out, bh, D, scale, s);
    case SSD_F16: return launch_t<__half>(q, k, v, lg, kc, vc, lgc, widx, cap, out, bh, D, scale, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ssdb200
