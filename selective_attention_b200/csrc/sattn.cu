// sattn.cu - selective-attention decode step: the cache update and the pos-mode gated
// softmax attention of SelectiveMHA.step (modules/selective_attention.py:390-404,
// inference/selective_attn_cache.py:27-42) in one kernel.
//
// One CTA per (batch row, head). Its threads first write the new key, value and
// log-gate at slot write_idx, then stream the first write_idx + 1 cached keys and
// values once: a group of D/8 lanes owns one key (8 elements per lane, 16-byte loads),
// the score q.k*scale (+ the key's log-gate, except for the newest key, the token
// itself) goes through an online softmax per lane group, and the groups and warps are
// merged at the end. The step is bound by reading the cache from HBM.
//
// The prefill kernel computes the same gated attention for a whole sequence
// (_build_attn_matrix + the seq-mode _gated_softmax + @ v, :27-144 and :270-280 of
// SelectiveMHA.forward in inference): causal softmax of q.k*scale where every key adds
// its log-gate except on the diagonal. The reference's compressed path (keys whose gate
// is zero removed, the token's own score appended ungated) is the same function with
// those keys' log-gates at -inf, which is how this kernel runs it.
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
        g[u] = j < W - 1 ? lgb[j] : 0.f;  // the token's own key is not gated (:122)
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

// ===========================================================================
// Prefill: CTA = (64-query tile, head, row); 64-key tiles of K and V staged in shared
// memory; thread (tr, tc) owns rows tr + 16 i (i < 4), score columns tc + 16 j, output
// columns 4 tc + 64 g (g < 2). Online softmax per row across the half warp of the row.
// ===========================================================================
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

template <typename T>
__global__ void __launch_bounds__(256) sattn_prefill_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                            const T* __restrict__ v, const float* __restrict__ lg,
                                                            T* __restrict__ out, int H, int L, int D, float scale) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int LD = D + 4, LDP = kPT + 4;
  float* Qs = sm;              // [64][LD]
  float* Ks = Qs + kPT * LD;   // [64][LD]
  float* Vs = Ks + kPT * LD;   // [64][LD]
  float* Ps = Vs + kPT * LD;   // [64][LDP]
  float* gs = Ps + kPT * LDP;  // [64] log-gates of the key tile
  const int qt = (int)gridDim.x - 1 - (int)blockIdx.x;  // the longest (last) query tiles start first
  const long long bh = (long long)blockIdx.z * H + blockIdx.y;
  const int q0 = qt * kPT, tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  const T* qb = q + bh * L * D;
  const T* kb = k + bh * L * D;
  const T* vb = v + bh * L * D;
  const float* gb = lg + bh * L;
  stage_rows64<T>(Qs, LD, qb, q0, L, D);
  float o[4][8], m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[i][e] = 0.f;
  }
  int dcol[2];
#pragma unroll
  for (int g = 0; g < 2; ++g) dcol[g] = min(4 * tc + 64 * g, D - 4);
  for (int kt = 0; kt <= qt; ++kt) {
    const int k0 = kt * kPT;
    __syncthreads();  // previous tile's K, V, P consumed
    stage_rows64<T>(Ks, LD, kb, k0, L, D);
    stage_rows64<T>(Vs, LD, vb, k0, L, D);
    if (tid < kPT) gs[tid] = k0 + tid < L ? gb[k0 + tid] : 0.f;
    __syncthreads();
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
    for (int d = 0; d < D; d += 4) {
      float4 a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(Qs + (tr + 16 * i) * LD + d);
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(Ks + (tc + 16 * j) * LD + d);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float t = sc[i][j];
          t = fmaf(a[i].x, b[j].x, t);
          t = fmaf(a[i].y, b[j].y, t);
          t = fmaf(a[i].z, b[j].z, t);
          sc[i][j] = fmaf(a[i].w, b[j].w, t);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = q0 + tr + 16 * i;
      float rmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kj = k0 + tc + 16 * j;
        float s = -INFINITY;
        if (kj <= qi && kj < L) s = sc[i][j] * scale + (kj < qi ? gs[tc + 16 * j] : 0.f);
        sc[i][j] = s;
        rmax = fmaxf(rmax, s);
      }
      rmax = hw_max(rmax);
      const float mn = fmaxf(m[i], rmax);
      const float corr = m[i] == -INFINITY ? 0.f : expf(m[i] - mn);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = sc[i][j] == -INFINITY ? 0.f : expf(sc[i][j] - mn);
        rs += p;
        Ps[(tr + 16 * i) * LDP + tc + 16 * j] = p;
      }
      l[i] = l[i] * corr + hw_sum(rs);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[i][e] *= corr;
      m[i] = mn;
    }
    __syncthreads();
#pragma unroll 2
    for (int j = 0; j < kPT; j += 4) {
      float4 pa[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pa[i] = *reinterpret_cast<const float4*>(Ps + (tr + 16 * i) * LDP + j);
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
        float4 vv[2];
#pragma unroll
        for (int g = 0; g < 2; ++g) vv[g] = *reinterpret_cast<const float4*>(Vs + (j + qq) * LD + dcol[g]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p = qq == 0 ? pa[i].x : (qq == 1 ? pa[i].y : (qq == 2 ? pa[i].z : pa[i].w));
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            o[i][4 * g] = fmaf(p, vv[g].x, o[i][4 * g]);
            o[i][4 * g + 1] = fmaf(p, vv[g].y, o[i][4 * g + 1]);
            o[i][4 * g + 2] = fmaf(p, vv[g].z, o[i][4 * g + 2]);
            o[i][4 * g + 3] = fmaf(p, vv[g].w, o[i][4 * g + 3]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = q0 + tr + 16 * i;
    if (qi >= L) continue;
    const float inv = 1.0f / l[i];
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int d = 4 * tc + 64 * g;
      if (d >= D) continue;
      T* op = out + (bh * L + qi) * D + d;
#pragma unroll
      for (int e = 0; e < 4; ++e) op[e] = from_f32<T>(o[i][4 * g + e] * inv);
    }
  }
}

template <typename T>
cudaError_t prefill_t(const void* q, const void* k, const void* v, const float* lg, void* out, int b, int H, int L,
                      int D, float scale, cudaStream_t s) {
  const size_t smem = (size_t)(3 * kPT * (D + 4) + kPT * (kPT + 4) + kPT) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(sattn_prefill_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((L + kPT - 1) / kPT), (unsigned)H, (unsigned)b);
  sattn_prefill_kernel<T><<<grid, 256, smem, s>>>((const T*)q, (const T*)k, (const T*)v, lg, (T*)out, H, L, D, scale);
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

namespace ssdb200 {

bool sattn_prefill_supported(int D) { return D == 16 || D == 32 || D == 64 || D == 128; }

cudaError_t launch_sattn_prefill(const void* q, const void* k, const void* v, const float* lg, void* out, int b, int H,
                                 int L, int D, float scale, int dtype, cudaStream_t s) {
  switch (dtype) {
    case SSD_F32: return prefill_t<float>(q, k, v, lg, out, b, H, L, D, scale, s);
    case SSD_BF16: return prefill_t<__nv_bfloat16>(q, k, v, lg, out, b, H, L, D, scale, s);
    case SSD_F16: return prefill_t<__half>(q, k, v, lg, out, b, H, L, D, scale, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ssdb200
