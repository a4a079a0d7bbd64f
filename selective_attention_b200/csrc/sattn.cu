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
// those keys' log-gates at -inf, which is how this kernel runs it. For 16-bit inputs with
// head_dim 64 or 128 a tensor-core version runs the two products on tcgen05 with the
// scores, the probabilities and the output accumulator in tensor memory.
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "sattn_tiles.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace ssdb200 {
namespace {

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

// ===========================================================================
// Tensor-core prefill (16-bit inputs, head_dim 64 or 128). CTA = 128 queries of one
// (row, head), 8 warps: threads t and t + 128 share query row q0 + t = TMEM lane t
// (each takes 32 of a tile's keys and half of O's columns). Per 64-key tile:
//   S = Q K^T          tcgen05 (A = Q, B = K, both K-major SW128 in shared memory) -> TMEM
//   softmax            thread reads its S row, adds the log-gates (not on the diagonal),
//                      masks keys past the query, keeps a running reference max and sum
//   P -> TMEM          16-bit probabilities, two per 32-bit column
//   O += P V           tcgen05 TS form (A = P from TMEM, B = V MN-major), 64 columns a block
// O is rescaled (TMEM load / store of the row) only when a row's max grows by more than 8
// (e^8 bounds the unnormalised probabilities). Every wait is bounded; on a timeout the
// kernel records an error code and releases its tensor memory.
// TMEM columns: S [0, 64), P [64, 96), O [128, 128 + D).
// ===========================================================================
using namespace sm100;
constexpr unsigned int kSiteAttnMma = 0x301;
constexpr int kTQ = 128;           // queries per CTA
constexpr int kTK = 64;            // keys per tile
constexpr int kQBlk = kTQ * 128;   // bytes of one 64-column block of the Q tile
constexpr int kKBlk = kTK * 128;   // bytes of one 64-column block of a K or V tile
constexpr size_t kTcSmem = 104 * 1024;  // at most two CTAs (2 x 256 TMEM columns) per SM
constexpr int kTcThreads = 256;          // two threads per query row
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.0f * kLog2e;  // rescale O when a row max grows by more than e^8

// rows x D 16-bit tile -> shared memory, 64-column blocks of 128-byte swizzled rows.
template <int ROWS, int D>
__device__ __forceinline__ void load_tile_sw128(uint8_t* dst, int blk_bytes, const uint16_t* src, int valid) {
  constexpr int CPR = D / 8, N = ROWS * CPR / kTcThreads;  // 16-byte chunks per row, per thread
  uint4 v[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int ci = threadIdx.x + kTcThreads * i, r = ci / CPR, c = ci % CPR;
    v[i] = r < valid ? __ldg(reinterpret_cast<const uint4*>(src + (long long)r * D + c * 8)) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int ci = threadIdx.x + kTcThreads * i, r = ci / CPR, c = ci % CPR;
    *reinterpret_cast<uint4*>(dst + (c >> 3) * blk_bytes + sw128_off((uint32_t)r, (uint32_t)(c & 7))) = v[i];
  }
}

// The same tile through cp.async (16-byte copies straight into shared memory; rows past
// `valid` are zero-filled), committed as one group.
template <int ROWS, int D>
__device__ __forceinline__ void load_tile_sw128_async(uint8_t* dst, int blk_bytes, const uint16_t* src, int valid) {
  constexpr int CPR = D / 8, N = ROWS * CPR / kTcThreads;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int ci = threadIdx.x + kTcThreads * i, r = ci / CPR, c = ci % CPR;
    const uint32_t d = smem_u32(dst + (c >> 3) * blk_bytes + sw128_off((uint32_t)r, (uint32_t)(c & 7)));
    const uint16_t* g = r < valid ? src + (long long)r * D + c * 8 : src;
    const uint32_t n = r < valid ? 16u : 0u;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(g), "r"(n) : "memory");
  }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// 2^x on the special-function unit (PTX ex2.approx; 2^-inf = +0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T, int D>
__global__ void __launch_bounds__(kTcThreads, 1) sattn_prefill_tc_kernel(const T* __restrict__ q,
                                                                         const T* __restrict__ k,
                                                                         const T* __restrict__ v,
                                                                         const float* __restrict__ lg,
                                                                         T* __restrict__ out, int H, int L,
                                                                         float scale) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int NB = D / 64;
  extern __shared__ uint8_t smraw[];
  uint8_t* base = align1024_shared(smraw);
  uint8_t* sQ = base;
  uint8_t* sKV = sQ + NB * kQBlk;                              // two buffers of (K, V)
  float* sg = reinterpret_cast<float*>(sKV + 4 * NB * kKBlk);  // two buffers of 64 log-gates
  float* xmax = sg + 2 * kTK;                                  // [2][128] row max of each half
  float* xsum = xmax + 2 * kTQ;                                // [2][128] row sum of each half
  uint64_t* bar = reinterpret_cast<uint64_t*>(xsum + 2 * kTQ);
  auto bufK = [&](int i) { return sKV + (2 * i) * NB * kKBlk; };
  auto bufV = [&](int i) { return sKV + (2 * i + 1) * NB * kKBlk; };
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  // threads 0-127 own the first 32 keys of each tile and the first half of O's columns for
  // query row tid; threads 128-255 the second halves of the same rows
  const int tid = threadIdx.x, warp = tid >> 5, half = tid >> 7, row = tid & 127;
  const int qt = (int)gridDim.x - 1 - (int)blockIdx.x;  // longest query tiles first
  const long long bh = (long long)blockIdx.z * H + blockIdx.y;
  const int q0 = qt * kTQ, qi = q0 + row;
  const uint16_t* qb = reinterpret_cast<const uint16_t*>(q) + bh * L * D;
  const uint16_t* kb = reinterpret_cast<const uint16_t*>(k) + bh * L * D;
  const uint16_t* vb = reinterpret_cast<const uint16_t*>(v) + bh * L * D;
  const float* gb = lg + bh * L;
  const uint32_t b_addr = smem_u32(bar);
  if (tid == 0) {
    mbar_init(b_addr, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 256);
  load_tile_sw128<kTQ, D>(sQ, kQBlk, qb + (long long)q0 * D, L - q0);
  load_tile_sw128_async<kTK, D>(bufK(0), kKBlk, kb, L);
  load_tile_sw128_async<kTK, D>(bufV(0), kKBlk, vb, L);
  cp_async_commit();
  if (tid < kTK) sg[tid] = tid < L ? gb[tid] * kLog2e : 0.f;
  cp_async_wait_all();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tl = (uint32_t)((warp & 3) * 32) << 16;  // TMEM lanes of this warp's rows
  constexpr uint32_t T_S = 0, T_P = 64, T_O = 128;
  constexpr uint32_t ID_S = idesc_f16(128, 64, BF16, false, false);
  constexpr uint32_t ID_O = idesc_f16(128, 64, BF16, false, true);
  const int jh = 32 * half;          // this thread's first key of a tile
  const int ch = (D / 2) * half;     // this thread's first O column
  // scores in the log2 domain (scale and gates times log2(e)): p = 2^(s - m)
  const float scale2 = scale * kLog2e;
  float m_used = -INFINITY, lsum = 0.f;
  uint32_t uses = 0;
  bool ok = true;
  const int nkt = min((q0 + kTQ + kTK - 1) / kTK, (L + kTK - 1) / kTK);
  for (int kt = 0; kt < nkt; ++kt) {
    const int k0 = kt * kTK, cur = kt & 1;
    uint8_t* sK = bufK(cur);
    uint8_t* sV = bufV(cur);
    const float* gcur = sg + cur * kTK;
    // tile kt is resident (previous iteration); its other buffer was last read by the
    // MMAs of tile kt-1, which have completed: prefetch tile kt+1 there
    if (kt + 1 < nkt) {
      const int k1 = k0 + kTK;
      load_tile_sw128_async<kTK, D>(bufK(cur ^ 1), kKBlk, kb + (long long)k1 * D, L - k1);
      load_tile_sw128_async<kTK, D>(bufV(cur ^ 1), kKBlk, vb + (long long)k1 * D, L - k1);
      cp_async_commit();
    }
    float gnext = 0.f;
    if (tid < kTK && k0 + kTK + tid < L) gnext = gb[k0 + kTK + tid] * kLog2e;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const uint32_t hf = ks >> 2, kk = (ks & 3) * 32;
        umma_f16(tmem + T_S, sdesc_sw128(smem_u32(sQ) + hf * kQBlk + kk, 16, 1024),
                 sdesc_sw128(smem_u32(sK) + hf * kKBlk + kk, 16, 1024), ID_S, ks > 0 ? 1u : 0u);
      }
      umma_commit(b_addr);
    }
    ok = mbar_wait(b_addr, uses & 1, kSiteAttnMma);
    ++uses;
    if (!__syncthreads_and(ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    uint32_t sr[32];
    tmem_ld32(tmem + tl + T_S + jh, sr);
    tmem_wait_ld();
    float mt = -INFINITY;
    if (k0 + kTK <= q0 && k0 + kTK <= L) {  // whole tile before every query of the CTA: all gated
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 g4 = *reinterpret_cast<const float4*>(gcur + jh + j);
        const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float s = fmaf(__uint_as_float(sr[j + e]), scale2, gg[e]);
          sr[j + e] = __float_as_uint(s);
          mt = fmaxf(mt, s);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int kj = k0 + jh + j;
        float s = -INFINITY;
        if (kj <= qi && kj < L)
          s = kj < qi ? fmaf(__uint_as_float(sr[j]), scale2, gcur[jh + j]) : __uint_as_float(sr[j]) * scale2;
        sr[j] = __float_as_uint(s);
        mt = fmaxf(mt, s);
      }
    }
    xmax[half * kTQ + row] = mt;
    __syncthreads();
    mt = fmaxf(xmax[row], xmax[kTQ + row]);  // both threads of the row see the same max
    float f = 1.f;
    bool rescale = false;
    if (mt != -INFINITY && (m_used == -INFINITY || mt > m_used + kRescaleLog2)) {
      if (kt > 0 && m_used != -INFINITY) {  // O and the sum hold earlier tiles: rescale them
        f = ex2(m_used - mt);
        lsum *= f;
        rescale = true;
      }
      m_used = mt;
    }
    // TMEM loads / stores are warp-collective: the whole warp runs them when any lane
    // rescales (the others with f = 1).
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
      for (int c = 0; c < D / 2; c += 32) {
        uint32_t o[32];
        tmem_ld32(tmem + tl + T_O + ch + c, o);
        tmem_wait_ld();
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          lo[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          hi[e] = __float_as_uint(__uint_as_float(o[16 + e]) * f);
        }
        tmem_st16(tmem + tl + T_O + ch + c, lo);
        tmem_st16(tmem + tl + T_O + ch + c + 16, hi);
      }
    }
    // while a row has no finite score yet, every s of the tile is -inf and 2^-inf = 0
    const float mb = m_used == -INFINITY ? 0.f : m_used;
    uint32_t pk[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float s0 = __uint_as_float(sr[2 * j]), s1 = __uint_as_float(sr[2 * j + 1]);
      const float p0 = ex2(s0 - mb), p1 = ex2(s1 - mb);
      pk[j] = pack2<T>(p0, p1);
      const float2 r = unpack2<T>(pk[j]);  // the sum uses the probabilities the MMA sees
      lsum += r.x + r.y;
    }
    tmem_st16(tmem + tl + T_P + 16 * half, pk);
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_f16_ts(tmem + T_O + 64 * nb, tmem + T_P + 8 * ks,
                      sdesc_sw128(smem_u32(sV) + nb * kKBlk + ks * 2048, 16, 1024), ID_O,
                      (kt > 0 || ks > 0) ? 1u : 0u);
      umma_commit(b_addr);
    }
    ok = mbar_wait(b_addr, uses & 1, kSiteAttnMma);
    ++uses;
    // the prefetched tile lands before the next iteration reads it
    if (tid < kTK) sg[(cur ^ 1) * kTK + tid] = gnext;
    cp_async_wait_all();
    fence_proxy_async_smem();
    if (!__syncthreads_and(ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
  }
  if (ok) {  // uniform across the CTA: every lane loads its row (warp-collective); rows past L store nothing
    xsum[half * kTQ + row] = lsum;
    __syncthreads();
    const float inv = 1.0f / (xsum[row] + xsum[kTQ + row]);
    T* op = out + (bh * L + qi) * D + ch;
#pragma unroll
    for (int c = 0; c < D / 2; c += 32) {
      uint32_t o[32];
      tmem_ld32(tmem + tl + T_O + ch + c, o);
      tmem_wait_ld();
      if (qi < L) {
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 w;
          w.x = pack2<T>(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
          w.y = pack2<T>(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
          w.z = pack2<T>(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
          w.w = pack2<T>(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
          *reinterpret_cast<uint4*>(op + c + e) = w;
        }
      }
    }
  }
  if (!ok && tid == 0) mbar_wait(b_addr, (uses - 1) & 1, kSiteAttnMma);  // drain the pending MMA (bounded)
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

template <typename T>
cudaError_t prefill_tc_t(const void* q, const void* k, const void* v, const float* lg, void* out, int b, int H, int L,
                         int D, float scale, cudaStream_t s) {
  dim3 grid((unsigned)((L + kTQ - 1) / kTQ), (unsigned)H, (unsigned)b);
  cudaError_t e;
  if (D == 64) {
    if ((e = cudaFuncSetAttribute(sattn_prefill_tc_kernel<T, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kTcSmem)))
      return e;
    sattn_prefill_tc_kernel<T, 64><<<grid, kTcThreads, kTcSmem, s>>>((const T*)q, (const T*)k, (const T*)v, lg, (T*)out, H,
                                                              L, scale);
  } else {
    if ((e = cudaFuncSetAttribute(sattn_prefill_tc_kernel<T, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kTcSmem)))
      return e;
    sattn_prefill_tc_kernel<T, 128><<<grid, kTcThreads, kTcSmem, s>>>((const T*)q, (const T*)k, (const T*)v, lg, (T*)out, H,
                                                               L, scale);
  }
  return cudaGetLastError();
}


// ---------------------------------------------------------------------------
// Pipelined tensor-core prefill, head_dim 64 (16-bit inputs)
// ---------------------------------------------------------------------------
// One CTA per (batch row x head, pair of 128-query tiles A = 2t and B = 2t + 1), the
// pairs with the most key tiles first. Warp roles (12 warps):
//   warp 0            loads: Q_A and Q_B once, then per 128-key tile K and V (TMA,
//                     128-byte swizzle) and its log-gates times log2(e), in a ring of
//                     kFaStages;
//   warp 1 (lane 0)   MMA issuer: S_w = Q_w K_j^T into TMEM; once softmax w has written
//                     P_w(j): O_w += P_w V_j (A from TMEM) and at once S_w(j + 1). The
//                     two tiles alternate, so the tensor core works on one tile while
//                     the other tile's softmax runs;
//   warps 4-7, 8-11   softmax of tile A, B: thread = query row = TMEM lane. A key tile's
//                     128 scores sit in registers: gate (every earlier key adds its
//                     log-gate, the token's own score is ungated), causal and length
//                     masks on the diagonal and tail tiles only, running max in the
//                     log2 domain (O and the sum are rescaled only when it grows by more
//                     than e^8), P = 2^(s - m) in 16 bits to TMEM, the row sum; at the
//                     end out = O / sum;
//   warps 2-3         no work (they keep the softmax warpgroups aligned to TMEM lanes).
// TMEM (512 columns): S_A [0,128) S_B [128,256) P_A [256,320) P_B [320,384)
//                     O_A [384,448) O_B [448,512). Every wait is bounded; a role that
// gives up records a site code, raises the CTA's abort flag and leaves its loop.
constexpr int kFaThreads = 384;
// Every kFaPolyEvery-th pair of probabilities is computed on the FMA pipes instead of the
// special-function unit (0: none), which the rest share with the 16-bit packing.
#ifndef SSD_FA_POLY_EVERY
#define SSD_FA_POLY_EVERY 0
#endif

// Packed fp32 pairs (Blackwell f32x2 arithmetic on 64-bit register pairs).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// 2^d for a pair, on the FMA pipes: d = n + f with n = round(d) (adding and subtracting
// 1.5 * 2^23 rounds to an integer, which then sits in the low mantissa bits) and
// f in [-0.5, 0.5]; 2^f by a cubic least-squares fit on Chebyshev nodes (relative error
// below 8e-5, far inside the 16-bit rounding of P); n goes into the exponent field. d is
// clamped at -125 so the exponent stays normal (2^-125 in place of 0 for masked scores).
__device__ __forceinline__ void exp2_pair_fma(float d0, float d1, float& p0, float& p1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const uint64_t d = f2_pack(fmaxf(d0, -125.f), fmaxf(d1, -125.f));
  const uint64_t r = f2_add(d, f2_pack(kMagic, kMagic));
  const uint64_t f = f2_add(d, f2_add(f2_pack(kMagic, kMagic), r ^ 0x8000000080000000ull));  // d - (r - M)
  uint64_t p = f2_fma(f, f2_pack(0.055171605f, 0.055171605f), f2_pack(0.24261111f, 0.24261111f));
  p = f2_fma(p, f, f2_pack(0.69326097f, 0.69326097f));
  p = f2_fma(p, f, f2_pack(0.99992806f, 0.99992806f));
  p0 = __uint_as_float((uint32_t)p + ((uint32_t)r << 23));
  p1 = __uint_as_float((uint32_t)(p >> 32) + ((uint32_t)(r >> 32) << 23));
}
constexpr int kFaStages = 3;
constexpr int kFaTile = 128 * 128;                 // 128 rows x 64 16-bit elements
constexpr int kFaStageBytes = 2 * kFaTile + 1024;  // K | V | 128 log-gates (1 KB keeps the alignment)
constexpr size_t kFaSmem = 1024 + 2 * kFaTile + kFaStages * kFaStageBytes + 256;
constexpr unsigned int kSiteFaLoad = 0x311, kSiteFaMma = 0x312, kSiteFaSoft = 0x313;

template <typename T>
__global__ void __launch_bounds__(kFaThreads, 1) sattn_prefill_fa_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                                          const __grid_constant__ CUtensorMap tm_k,
                                                                          const __grid_constant__ CUtensorMap tm_v,
                                                                          const float* __restrict__ lg,
                                                                          T* __restrict__ out, int L, float scale,
                                                                          float* __restrict__ lse, int causal) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int NS = kFaStages;
  extern __shared__ uint8_t smraw[];
  uint8_t* base = align1024_shared(smraw);
  uint8_t* sQ = base;  // Q_A | Q_B
  auto sK = [&](int s) { return base + 2 * kFaTile + s * kFaStageBytes; };
  auto sV = [&](int s) { return sK(s) + kFaTile; };
  auto sG = [&](int s) { return reinterpret_cast<float*>(sK(s) + 2 * kFaTile); };
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 2 * kFaTile + NS * kFaStageBytes);
  enum {
    Q_FULL = 0, K_FULL = 1, V_FULL = K_FULL + NS, KV_EMPTY = V_FULL + NS, S_FULL = KV_EMPTY + NS,
    S_FREE = S_FULL + 2, P_FULL = S_FREE + 2, O_DONE = P_FULL + 2, DRAIN = O_DONE + 2, NBARS = DRAIN + 1
  };
  static_assert(NBARS * 8 + 8 <= 256, "barrier area");
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tslot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int bh = blockIdx.x;
  const int t = (int)gridDim.y - 1 - (int)blockIdx.y;  // pairs with the most key tiles first
  const int q0A = 256 * t, q0B = q0A + 128;
  const int nkv = (L + 127) / 128;  // every key tile (bidirectional attention)
  const int nkA = q0A < L ? (causal ? min(q0A + 127, L - 1) / 128 + 1 : nkv) : 0;
  const int nkB = q0B < L ? (causal ? min(q0B + 127, L - 1) / 128 + 1 : nkv) : 0;
  const int nk = max(nkA, nkB);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    mbar_init(bar(Q_FULL), 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(K_FULL + s), 1);
      mbar_init(bar(V_FULL + s), 1);
      mbar_init(bar(KV_EMPTY + s), 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(bar(S_FULL + w), 1);
      mbar_init(bar(S_FREE + w), 4);
      mbar_init(bar(P_FULL + w), 4);
      mbar_init(bar(O_DONE + w), 1);
    }
    mbar_init(bar(DRAIN), 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tslot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  constexpr uint32_t T_S = 0, T_P = 256, T_O = 384;
  // Registers: launched with 168 a thread (384 x 168 = 64512, 16128 per SM sub-partition);
  // warpgroup 0 (loads, MMA) keeps 56 and the two softmax warpgroups take 208 each, which
  // holds a row's 128 scores without spilling: 128 x 56 + 256 x 208 = 60416 <= 64512, and
  // per sub-partition (one warp of each warpgroup) 32 x (56 + 2 x 208) = 15104 <= 16128.
  // (each role branch below starts with its warpgroup's share)
  static_assert(kFaThreads == 384, "register split assumes three warpgroups");

  if (warp == 0) {
    // ------------------------------------------------------------ loads
    regs_dec<56>();
    if (lane == 0) {
      mbar_expect_tx(bar(Q_FULL), (nkB > 0 ? 2u : 1u) * (uint32_t)kFaTile);
      tma_load_3d(smem_u32(sQ), &tm_q, 0, q0A, bh, bar(Q_FULL));
      if (nkB > 0) tma_load_3d(smem_u32(sQ + kFaTile), &tm_q, 0, q0B, bh, bar(Q_FULL));
    }
    const float* gb = lg + (long long)bh * L;
    bool fail = false;
    int j = 0;
    for (; j < nk; ++j) {
      const int s = j % NS;
      // the stage's gates are rewritten below: every lane waits for its release
      if (j >= NS && (!__all_sync(0xffffffffu, mbar_wait(bar(KV_EMPTY + s), ((j / NS) - 1) & 1, kSiteFaLoad)) ||
                      *s_abort)) {
        fail = true;
        break;
      }
      const int k = 128 * j + 4 * lane;
      float4 g4;
      g4.x = k < L ? gb[k] * kLog2e : -INFINITY;
      g4.y = k + 1 < L ? gb[k + 1] * kLog2e : -INFINITY;
      g4.z = k + 2 < L ? gb[k + 2] * kLog2e : -INFINITY;
      g4.w = k + 3 < L ? gb[k + 3] * kLog2e : -INFINITY;
      reinterpret_cast<float4*>(sG(s))[lane] = g4;
      __syncwarp();
      if (lane == 0) {
        mbar_expect_tx(bar(K_FULL + s), (uint32_t)kFaTile);
        tma_load_3d(smem_u32(sK(s)), &tm_k, 0, 128 * j, bh, bar(K_FULL + s));
        mbar_expect_tx(bar(V_FULL + s), (uint32_t)kFaTile);
        tma_load_3d(smem_u32(sV(s)), &tm_v, 0, 128 * j, bh, bar(V_FULL + s));
      }
    }
    if (fail && lane == 0) *s_abort = 1;
    if (lane == 0) {
      // no copy may still be in flight when the CTA exits
      mbar_wait(bar(Q_FULL), 0, kSiteFaLoad);
      for (int d = 1; d <= NS && d <= j; ++d) {
        const int jj = j - d;
        mbar_wait(bar(K_FULL + jj % NS), (jj / NS) & 1, kSiteFaLoad);
        mbar_wait(bar(V_FULL + jj % NS), (jj / NS) & 1, kSiteFaLoad);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    regs_dec<56>();
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_f16(128, 128, BF16, false, false);
      constexpr uint32_t ID_O = idesc_f16(128, 64, BF16, false, true);
      const uint32_t qa = smem_u32(sQ);
      const int nkw[2] = {nkA, nkB};
      bool issued = false;
      auto issue_s = [&](int w, int jj) -> bool {
        const int s = jj % NS;
        if (!mbar_wait(bar(K_FULL + s), (jj / NS) & 1, kSiteFaMma)) return false;
        tc_fence_after();
        const uint32_t qb = qa + (uint32_t)(w * kFaTile), kb = smem_u32(sK(s));
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_f16(tmem + T_S + 128 * w, sdesc_sw128(qb + 32 * ks, 16, 1024), sdesc_sw128(kb + 32 * ks, 16, 1024),
                   ID_S, ks > 0 ? 1u : 0u);
        umma_commit(bar(S_FULL + w));
        issued = true;
        return true;
      };
      bool fail = !mbar_wait(bar(Q_FULL), 0, kSiteFaMma);
      if (!fail) fail = !issue_s(0, 0);
      if (!fail && nkB > 0) fail = !issue_s(1, 0);
      for (int j = 0; j < nk && !fail && !*s_abort; ++j) {
        const int s = j % NS;
        // S_w(j + 1) as soon as softmax w holds S_w(j) in registers: it runs on the tensor
        // core while that softmax computes the probabilities of step j
        for (int w = 0; w < 2 && !fail; ++w) {
          if (j + 1 >= nkw[w]) continue;
          if (!mbar_wait(bar(S_FREE + w), j & 1, kSiteFaMma) || !issue_s(w, j + 1)) fail = true;
        }
        if (fail || !mbar_wait(bar(V_FULL + s), (j / NS) & 1, kSiteFaMma)) {
          fail = true;
          break;
        }
        const uint32_t vb = smem_u32(sV(s));
        for (int w = 0; w < 2; ++w) {
          if (j >= nkw[w]) continue;
          if (!mbar_wait(bar(P_FULL + w), j & 1, kSiteFaMma)) {
            fail = true;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_f16_ts(tmem + T_O + 64 * w, tmem + T_P + 64 * w + 8 * ks, sdesc_sw128(vb + 2048 * ks, 16, 1024),
                        ID_O, (j > 0 || ks > 0) ? 1u : 0u);
          umma_commit(bar(O_DONE + w));
        }
        if (fail) break;
        umma_commit(bar(KV_EMPTY + s));
      }
      if (fail) *s_abort = 1;
      // every MMA has completed before TMEM is released
      if (issued) {
        umma_commit(bar(DRAIN));
        mbar_wait(bar(DRAIN), 0, kSiteFaMma);
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    regs_dec<56>();  // warps 2-3: no work
  } else {
    // ------------------------------------------------------------ softmax of tile w
    regs_inc<208>();
    const int w = (warp - 4) >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t tl = (uint32_t)((warp & 3) * 32) << 16;
    const int nkw = w ? nkB : nkA;
    const int q0 = w ? q0B : q0A;
    const int qi = q0 + r;
    const float scale2 = scale * kLog2e;
    float m_used = -INFINITY, lsum = 0.f;
    bool wfail = false;
    auto warp_wait = [&](uint32_t b, uint32_t parity, unsigned int site) {
      if (!wfail) wfail = !__all_sync(0xffffffffu, mbar_wait(b, parity, site));
      return !wfail;
    };
    for (int j = 0; j < nkw; ++j) {
      const int s = j % NS;
      if (!warp_wait(bar(S_FULL + w), j & 1, kSiteFaSoft) || !warp_wait(bar(K_FULL + s), (j / NS) & 1, kSiteFaSoft))
        break;
      tc_fence_after();
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + tl + T_S + 128 * w + 32 * c, sv[c]);
      tmem_wait_ld();
      // S_w(j) is in registers: the MMA may overwrite it with S_w(j + 1)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(S_FREE + w));
      const float4* g4 = reinterpret_cast<const float4*>(sG(s));
      const int k0 = 128 * j;
      // eight partial maxima (columns e mod 8), so the reduction is not one long chain
      float mp[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) mp[q] = -INFINITY;
      // tiles are 128-aligned: a key tile holds none of the queries' own keys unless k0 == q0
      if ((causal ? k0 < q0 : k0 != q0) && k0 + 128 <= L) {  // every key of the tile is gated
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 g = g4[(32 * c + e) >> 2];
            const float x0 = fmaf(__uint_as_float(sv[c][e]), scale2, g.x);
            const float x1 = fmaf(__uint_as_float(sv[c][e + 1]), scale2, g.y);
            const float x2 = fmaf(__uint_as_float(sv[c][e + 2]), scale2, g.z);
            const float x3 = fmaf(__uint_as_float(sv[c][e + 3]), scale2, g.w);
            sv[c][e] = __float_as_uint(x0);
            sv[c][e + 1] = __float_as_uint(x1);
            sv[c][e + 2] = __float_as_uint(x2);
            sv[c][e + 3] = __float_as_uint(x3);
            const int q = e & 4;
            mp[q] = fmaxf(mp[q], x0);
            mp[q + 1] = fmaxf(mp[q + 1], x1);
            mp[q + 2] = fmaxf(mp[q + 2], x2);
            mp[q + 3] = fmaxf(mp[q + 3], x3);
          }
      } else {
        // diagonal or tail tile: keys past L (and, causal, past the query) drop out, the
        // query's own key is ungated
        const float* g = sG(s);
        const int gate_end = causal ? min(qi, L) : L;  // keys below this are gated (but qi)
        const bool own = qi < L && qi >= k0 && qi < k0 + 128;  // the query's own key is in this tile
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = k0 + 32 * c + e;
            const float sc = __uint_as_float(sv[c][e]);
            float x = key < gate_end ? fmaf(sc, scale2, g[32 * c + e]) : -INFINITY;
            if (own && key == qi) x = sc * scale2;
            sv[c][e] = __float_as_uint(x);
            mp[e & 7] = fmaxf(mp[e & 7], x);
          }
      }
      const float mt = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      float f = 1.f;
      bool resc = false;
      if (mt != -INFINITY && (m_used == -INFINITY || mt > m_used + kRescaleLog2)) {
        if (j > 0 && m_used != -INFINITY) {  // O and the sum hold earlier tiles: rescale them
          f = ex2(m_used - mt);
          lsum *= f;
          resc = true;
        }
        m_used = mt;
      }
      // the probabilities first, into registers: computing them overlaps PV_w(j - 1),
      // which must complete before P_w is rewritten and before O_w is rescaled
      // (while a row has no finite score yet, every score of the tile is -inf and 2^-inf = 0)
      const float mb = m_used == -INFINITY ? 0.f : m_used;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};  // four partial sums
      uint32_t pk[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          float p0, p1;
          if (SSD_FA_POLY_EVERY > 0 && q % (SSD_FA_POLY_EVERY > 0 ? SSD_FA_POLY_EVERY : 1) == 0) {
            exp2_pair_fma(__uint_as_float(sv[c][2 * q]) - mb, __uint_as_float(sv[c][2 * q + 1]) - mb, p0, p1);
          } else {
            p0 = ex2(__uint_as_float(sv[c][2 * q]) - mb);
            p1 = ex2(__uint_as_float(sv[c][2 * q + 1]) - mb);
          }
          ls[q & 3] += p0 + p1;
          pk[c][q] = pack2<T>(p0, p1);
        }
      lsum += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      if (j > 0) {
        if (!warp_wait(bar(O_DONE + w), (j - 1) & 1, kSiteFaSoft)) break;
        tc_fence_after();
      }
      // TMEM loads / stores are warp-collective: the whole warp runs them when any lane
      // rescales (the others with f = 1)
      if (__any_sync(0xffffffffu, resc)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 16 columns at a time
          uint32_t o[16];
          tmem_ld16(tmem + tl + T_O + 64 * w + 16 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st16(tmem + tl + T_O + 64 * w + 16 * c, o);
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_st16(tmem + tl + T_P + 64 * w + 16 * c, pk[c]);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(P_FULL + w));
    }
    if (!wfail && nkw > 0 && warp_wait(bar(O_DONE + w), (nkw - 1) & 1, kSiteFaSoft)) {
      tc_fence_after();
      uint32_t o[2][32];
      tmem_ld32(tmem + tl + T_O + 64 * w, o[0]);
      tmem_ld32(tmem + tl + T_O + 64 * w + 32, o[1]);
      tmem_wait_ld();
      const float inv = 1.0f / lsum;
      if (lse && qi < L) lse[(long long)bh * L + qi] = (m_used + __log2f(lsum)) * kLn2;  // natural log-sum-exp
      if (qi < L) {
        uint4* op = reinterpret_cast<uint4*>(out + ((long long)bh * L + qi) * 64);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 v4;
            v4.x = pack2<T>(__uint_as_float(o[c][e]) * inv, __uint_as_float(o[c][e + 1]) * inv);
            v4.y = pack2<T>(__uint_as_float(o[c][e + 2]) * inv, __uint_as_float(o[c][e + 3]) * inv);
            v4.z = pack2<T>(__uint_as_float(o[c][e + 4]) * inv, __uint_as_float(o[c][e + 5]) * inv);
            v4.w = pack2<T>(__uint_as_float(o[c][e + 6]) * inv, __uint_as_float(o[c][e + 7]) * inv);
            op[(32 * c + e) >> 3] = v4;
          }
      }
    }
    if (wfail) *s_abort = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

template <typename T>
cudaError_t prefill_fa_t(const void* q, const void* k, const void* v, const float* lg, void* out, int b, int H, int L,
                         float scale, cudaStream_t s, float* lse = nullptr, int causal = 1) {
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const long long bhn = (long long)b * H, npairs = ((long long)L + 255) / 256;
  if (bhn > 0x7fffffffll || npairs > 65535) return cudaErrorInvalidValue;
  CUtensorMap mq, mk, mv;
  if (!make_map_3d(&mq, q, bf16, 64, (uint64_t)L, (uint64_t)bhn, 64, 128, 1) ||
      !make_map_3d(&mk, k, bf16, 64, (uint64_t)L, (uint64_t)bhn, 64, 128, 1) ||
      !make_map_3d(&mv, v, bf16, 64, (uint64_t)L, (uint64_t)bhn, 64, 128, 1))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(sattn_prefill_fa_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kFaSmem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)bhn, (unsigned)npairs);
  sattn_prefill_fa_kernel<T><<<grid, kFaThreads, kFaSmem, s>>>(mq, mk, mv, lg, (T*)out, L, scale, lse, causal);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_sattn_attn_fa(const void* q, const void* k, const void* v, const float* lg, void* out, float* lse,
                                 int b, int H, int L, float scale, int dtype, int causal, cudaStream_t s) {
  if (dtype == SSD_BF16) return prefill_fa_t<__nv_bfloat16>(q, k, v, lg, out, b, H, L, scale, s, lse, causal);
  if (dtype == SSD_F16) return prefill_fa_t<__half>(q, k, v, lg, out, b, H, L, scale, s, lse, causal);
  return cudaErrorInvalidValue;
}

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

bool sattn_prefill_tc_supported(int D, int dtype) { return (D == 64 || D == 128) && dtype != SSD_F32; }

cudaError_t launch_sattn_prefill(const void* q, const void* k, const void* v, const float* lg, void* out, int b, int H,
                                 int L, int D, float scale, int dtype, int use_tc, cudaStream_t s) {
  if (use_tc) {
    if (!sattn_prefill_tc_supported(D, dtype)) return cudaErrorInvalidValue;
    if (D == 64) {  // the pipelined kernel; head_dim 128 keeps the single-tile one
      if (dtype == SSD_BF16) return prefill_fa_t<__nv_bfloat16>(q, k, v, lg, out, b, H, L, scale, s);
      return prefill_fa_t<__half>(q, k, v, lg, out, b, H, L, scale, s);
    }
    if (dtype == SSD_BF16) return prefill_tc_t<__nv_bfloat16>(q, k, v, lg, out, b, H, L, D, scale, s);
    return prefill_tc_t<__half>(q, k, v, lg, out, b, H, L, D, scale, s);
  }
  switch (dtype) {
    case SSD_F32: return prefill_t<float>(q, k, v, lg, out, b, H, L, D, scale, s);
    case SSD_BF16: return prefill_t<__nv_bfloat16>(q, k, v, lg, out, b, H, L, D, scale, s);
    case SSD_F16: return prefill_t<__half>(q, k, v, lg, out, b, H, L, D, scale, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ssdb200

namespace ssdb200 {
SSDB200_DEFINE_ERROR_FETCH(fetch_error_sattn)
}  // namespace ssdb200
