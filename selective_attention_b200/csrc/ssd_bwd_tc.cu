// ssd_bwd_tc.cu - the SSD backward's contractions on tcgen05 tensor cores (16-bit u / B / C,
// headdim 64, dstate 128, chunk 256): the chunk-state recompute, the state-side products and
// the intra-chunk products; the CUDA-core kernels in ssd_bwd.cu do the scans and the rest.
// Operands arrive by TMA (128-byte swizzle) or are rounded to 16 bits in shared memory,
// products accumulate in fp32 in TMEM, and the epilogues read rows with thread = row = TMEM
// lane. Every mbarrier wait is bounded; a CTA that gives up records a site code, lets what it
// has in flight land (bounded) and skips its remaining work.
#include <cudaTypedefs.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.cuh"

namespace ssdb200 {

using namespace sm100;

namespace {

constexpr unsigned int kSiteBwdTcTma = 0x121, kSiteBwdTcMma = 0x122;
// 8 elements of a 16-byte chunk times w (fp32 products, one rounding to 16 bits).
template <typename T16>
__device__ __forceinline__ uint4 scaled8(uint4 a, float w) {
  float2 f;
  uint4 v;
  f = unpack2<T16>(a.x); v.x = pack2<T16>(f.x * w, f.y * w);
  f = unpack2<T16>(a.y); v.y = pack2<T16>(f.x * w, f.y * w);
  f = unpack2<T16>(a.z); v.z = pack2<T16>(f.x * w, f.y * w);
  f = unpack2<T16>(a.w); v.w = pack2<T16>(f.x * w, f.y * w);
  return v;
}

// ---------------------------------------------------------------------------
// Chunk states and intra-chunk state gradients (ssd_bwd.cu bwd_chunk_states_kernel's
// two products) on tcgen05, per (chunk, head, product):
//   product 0: S[p,n]  = sum_l u[l,p] w_l B[l,n],         w_l = exp(min(cum_last - cum_l, 0)) dt_l
//   product 1: HG[p,n] = sum_l y_grad[l,p] e_l C[l,n],    e_l = exp(cum_l)
// (backward.py:487, backward_kernel.py:23-93), both zero past the row's length. As in the
// forward's chunk_state: two 128-token phases, the token rows of u (TMA) or y_grad (TMA, or
// fp32 rounded here) scaled by their weight in shared memory, then M = 128 (dstate) x
// N = 64 (headdim) x K = 128 MMAs with both operands MN-major; thread = n = TMEM lane
// writes S / HG as [p][n] fp32.
// ---------------------------------------------------------------------------
constexpr int kCsThreads = 128;
constexpr size_t kCsSmem = 1024 + 32768 + 16384 + 1024 + 64;

template <bool BF16, typename YT>
__global__ void __launch_bounds__(kCsThreads) bwd_chunk_states_tc_kernel(
    const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_b,
    const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_c, const YT* __restrict__ yg,
    const float* __restrict__ dt, const float* __restrict__ cum, float* __restrict__ states, float* __restrict__ hg,
    ChunkMap cm, int H, int G, uint16_t* __restrict__ y16out) {
  using T16 = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr bool kY16 = sizeof(YT) == 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  uint8_t* sB = sm;           // 2 x (128 tokens x 128 B): dstate halves
  uint8_t* sX = sm + 32768;   // 128 tokens x 128 B
  float* sW = reinterpret_cast<float*>(sm + 49152);  // [256] token weights
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 49152 + 1024);  // TMA, MMA
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  const uint32_t bar_tma = smem_u32(&bars[0]), bar_mma = smem_u32(&bars[1]);
  const int h = blockIdx.x, k = blockIdx.y, which = blockIdx.z;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int g = h / (H / G), tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long kh = (long long)k * H + h;
  const int vl = ci.vlim;
  const bool from_y = which == 1;
  if (tid == 0) {
    prefetch_tmap(from_y ? &tm_c : &tm_b);
    if (!from_y) prefetch_tmap(&tm_u);
    else if (kY16) prefetch_tmap(&tm_y);
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 64);
  {
    const float clast = cum[kh * 256 + 255];
    for (int i = tid; i < 256; i += kCsThreads) {
      const float c = cum[kh * 256 + i];
      sW[i] = i < vl ? (from_y ? __expf(c) : __expf(fminf(clast - c, 0.f)) * dt[kh * 256 + i]) : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  constexpr uint32_t ID = idesc_f16(128, 64, BF16, /*a_mn=*/true, /*b_mn=*/true);
  bool ok = true;
  int uses = 0;
  for (int ph = 0; ph < 2 && ok; ++ph) {
    if (128 * ph >= vl) break;  // weights past the length are 0: nothing to add
    const int t0 = (int)(ci.tok0 + 128 * ph);
    if (tid == 0) {
      const CUtensorMap* mbc = from_y ? &tm_c : &tm_b;
      const bool x_tma = !from_y || kY16;
      mbar_expect_tx(bar_tma, 32768u + (x_tma ? 16384u : 0u));
      tma_load_3d(smem_u32(sB), mbc, 0, g, t0, bar_tma);
      tma_load_3d(smem_u32(sB + 16384), mbc, 64, g, t0, bar_tma);
      if (x_tma) tma_load_3d(smem_u32(sX), from_y ? &tm_y : &tm_u, 0, h, t0, bar_tma);
    }
    if (from_y && !kY16) {
      // fp32 y_grad rows times e_l, rounded to 16 bits into the swizzled tile. Every row below
      // the length is read (the 16-bit copy needs it even where e_l = 0); the 16 loads are
      // issued before any is used, rows at or past the length reading the last valid row.
      float4 ya[8], yb[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = tid + kCsThreads * i, row = q >> 3, c8 = q & 7, l = 128 * ph + row;
        const int lr = l < vl ? l : vl - 1;  // vl > 128 ph here
        const float* src = reinterpret_cast<const float*>(yg) + ((ci.tok0 + lr) * H + h) * 64 + c8 * 8;
        ya[i] = __ldg(reinterpret_cast<const float4*>(src));
        yb[i] = __ldg(reinterpret_cast<const float4*>(src + 4));
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = tid + kCsThreads * i, row = q >> 3, c8 = q & 7, l = 128 * ph + row;
        const float w = sW[l];
        const float4 a = ya[i], b = yb[i];
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (w != 0.f)
          v = make_uint4(pack2<T16>(a.x * w, a.y * w), pack2<T16>(a.z * w, a.w * w), pack2<T16>(b.x * w, b.y * w),
                         pack2<T16>(b.z * w, b.w * w));
        if (y16out && l < vl)  // the rows rounded, unscaled, for the later kernels' TMA loads
          *reinterpret_cast<uint4*>(y16out + ((ci.tok0 + l) * H + h) * 64 + c8 * 8) =
              make_uint4(pack2<T16>(a.x, a.y), pack2<T16>(a.z, a.w), pack2<T16>(b.x, b.y), pack2<T16>(b.z, b.w));
        *reinterpret_cast<uint4*>(sX + sw128_off((uint32_t)row, (uint32_t)c8)) = v;
      }
    }
    const bool landed = mbar_wait(bar_tma, uses & 1, kSiteBwdTcTma);
    if (landed && (!from_y || kY16)) {
      // token rows scaled in place by their weight (rows with weight 0 become exact zeros)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = tid + kCsThreads * i;
        uint4* pch = reinterpret_cast<uint4*>(sX + q * 16);
        const float w = sW[128 * ph + (q >> 3)];
        *pch = (w == 0.f) ? make_uint4(0u, 0u, 0u, 0u) : scaled8<T16>(*pch, w);
      }
    }
    fence_proxy_async_smem();
    ok = __syncthreads_and(landed) != 0;
    if (!ok) break;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_f16(tmem, sdesc_sw128(smem_u32(sB) + ks * 2048, 16384, 1024), sdesc_sw128(smem_u32(sX) + ks * 2048, 16, 1024),
                 ID, (ph > 0 || ks > 0) ? 1u : 0u);
      umma_commit(bar_mma);
    }
    // the next phase reuses both tiles, the epilogue reads the accumulator
    ok = __syncthreads_and(mbar_wait(bar_mma, uses & 1, kSiteBwdTcMma)) != 0;
    ++uses;
    tc_fence_after();
  }
  if (ok) {
    const int n = warp * 32 + lane;
    float* out = (from_y ? hg : states) + kh * 8192;
    if (uses == 0) {  // no valid token: the state is zero
      for (int p = 0; p < 64; ++p) out[p * 128 + n] = 0.f;
    } else {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + half * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) out[(half * 32 + j) * 128 + n] = __uint_as_float(v[j]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

template <bool BF16, typename YT>
cudaError_t launch_states_typed(const LaunchCtx& c, const BwdArgs& a) {
  CUtensorMap mu, mb, my, mc;
  if (!make_map_3d(&mu, a.u, BF16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mb, a.B, BF16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&my, sizeof(YT) == 2 ? a.y_grad : a.u, BF16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mc, a.C, BF16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128))
    return cudaErrorInvalidValue;
  auto kern = bwd_chunk_states_tc_kernel<BF16, YT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kCsSmem);
  if (e != cudaSuccess) return e;
  kern<<<dim3((unsigned)c.H, (unsigned)c.nchunks_max, 2u), kCsThreads, kCsSmem, c.stream>>>(
      mu, mb, my, mc, reinterpret_cast<const YT*>(a.y_grad), a.dt, a.cum, a.states, a.hg, c.cm, c.H, c.G,
      sizeof(YT) == 2 ? nullptr : a.y16);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Intra-chunk products of the backward (ssd_bwd.cu bwd_intra_kernel's contractions and
// its per-row work) on tcgen05, per (chunk, head); the dt backward (scans) stays on CUDA
// cores (bwd_dt_kernel). For each 128-row half of the chunk (rows l = query tokens):
//   accY[l,p] = sum_{s >= l} CB[s,l] exp(min(cum_s - cum_l, 0)) y_grad[s,p]        (:272-293)
//     A operand = the decay-weighted CB rows s, l contiguous (MN-major), 16 bits, B = y_grad
//   G[l,s]    = y_grad[l] . u[s]  (s <= l), computed as G^T: lane s, column l    (:632-659)
//   CB_grad[l,s] += G dt_s exp(min(cum_l - cum_s, 0));  w = CB_grad_h[l,s] CB[l,s] (s < l)
//   rows[l] = sum_s w,  cols[s] = sum_l w                                         (:847-895)
//   acc = accS + accY:  u_grad = acc dt_l,  ddt[l] = sum_p acc u,  gB[l] = dt_l sum_p accS u
// accY: TMEM lane = row l. G^T: lane = source token s, so a warp's 32 lanes read CB and add
// into CB_grad along contiguous rows. Two warps per lane quadrant split each accumulator's
// columns. TMEM: accY [0, 64), G^T (one 128 x 128 block) [128, 256).
// ---------------------------------------------------------------------------
constexpr int kInThreads = 256;
// dynamic: u [256][128 B] | y_grad [256][128 B] | A: one 128-s block [2 l-blocks][128 s][128 B];
// static: dt, cum, cols, rows [4][256], ddt / gB partials of the two column halves [2][2][128],
// barriers
constexpr int kInOffU = 0, kInOffY = 32768, kInOffA = 65536;
constexpr size_t kInSmem = 1024 + 98304;  // + 6 KB of static shared arrays

// Sums of 32 values over the warp's lanes, transposed: lane i returns sum over lanes of
// v[i] (31 shuffles in five halving steps; v is overwritten).
__device__ __forceinline__ float warp_transpose_sum32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 16; k >= 1; k >>= 1) {
    const bool upper = (lane & k) != 0;
#pragma unroll
    for (int i = 0; i < k; ++i) {
      const float send = upper ? v[i] : v[i + k];
      const float keep = upper ? v[i + k] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, k);
    }
  }
  return v[0];
}

// 8 warps: warp w reads TMEM lane quadrant w % 4 (rows l0 + 32 (w % 4) + lane) and the
// column half w / 4 of each accumulator; two CTAs per SM.
template <bool BF16, typename YT>
__global__ void __launch_bounds__(kInThreads, 2) bwd_intra_tc_kernel(
    const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_y, const void* __restrict__ u,
    const YT* __restrict__ yg, const float* __restrict__ dt, const float* __restrict__ cum,
    const float* __restrict__ CB, const float* __restrict__ accS, float* __restrict__ CBg, void* __restrict__ u_grad,
    float* __restrict__ rows4, ChunkMap cm, int H, int G, long long plane) {
  using T16 = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr bool kY16 = sizeof(YT) == 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  uint8_t* sU = sm + kInOffU;
  uint8_t* sY = sm + kInOffY;
  uint8_t* sA = sm + kInOffA;
  __shared__ float dts[256], cms[256], cols[256], rws[256];
  __shared__ float dpp[256], bpp[256];  // [2][128] each
  __shared__ uint64_t bars[2];
  __shared__ uint32_t tslot[1];
  const uint32_t bar_tma = smem_u32(&bars[0]), bar_mma = smem_u32(&bars[1]);
  const int h = blockIdx.x, k = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int g = h / (H / G), tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hc = warp >> 2;
  const long long kh = (long long)k * H + h;
  const long long kg = ((long long)k * G + g) * 65536;
  const int vl = ci.vlim, lim = ci.lim;
  if (tid == 0) {
    prefetch_tmap(&tm_u);
    if (kY16) prefetch_tmap(&tm_y);
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 256);
  {
    const int i = tid;  // kInThreads == 256
    dts[i] = dt[kh * 256 + i];
    cms[i] = cum[kh * 256 + i];
    cols[i] = 0.f;
    rws[i] = 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tl = (uint32_t)(qd * 32) << 16;
  constexpr uint32_t T_Y = 0, T_G = 128;
  constexpr uint32_t ID_Y = idesc_f16(128, 64, BF16, /*a_mn=*/true, /*b_mn=*/true);
  constexpr uint32_t ID_G = idesc_f16(128, 128, BF16, false, false);
  int uses = 0;
  if (tid == 0) {
    mbar_expect_tx(bar_tma, 32768u + (kY16 ? 32768u : 0u));
    for (int b = 0; b < 2; ++b) {
      tma_load_3d(smem_u32(sU + 16384 * b), &tm_u, 0, h, (int)(ci.tok0 + 128 * b), bar_tma);
      if (kY16) tma_load_3d(smem_u32(sY + 16384 * b), &tm_y, 0, h, (int)(ci.tok0 + 128 * b), bar_tma);
    }
  }
  if (!kY16) {
    // fp32 y_grad rows rounded to 16 bits, K-major over p; rows past the length are 0. All
    // loads are issued before any is used (rows past the length read the last valid row).
    float4 ya[8], yb[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = tid + kInThreads * i, row = q >> 3, c8 = q & 7;
      const int rr = row < vl ? row : max(vl - 1, 0);
      const float* src = reinterpret_cast<const float*>(yg) + ((ci.tok0 + rr) * H + h) * 64 + c8 * 8;
      ya[i] = __ldg(reinterpret_cast<const float4*>(src));
      yb[i] = __ldg(reinterpret_cast<const float4*>(src + 4));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = tid + kInThreads * i, row = q >> 3, c8 = q & 7;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row < vl)
        v = make_uint4(pack2<T16>(ya[i].x, ya[i].y), pack2<T16>(ya[i].z, ya[i].w), pack2<T16>(yb[i].x, yb[i].y),
                       pack2<T16>(yb[i].z, yb[i].w));
      *reinterpret_cast<uint4*>(sY + sw128_off((uint32_t)row, (uint32_t)c8)) = v;
    }
  }
  bool ok = mbar_wait(bar_tma, 0, kSiteBwdTcTma);
  if (ok && vl < 256) {
    // token rows at or past the length: zeros (their y_grad is ignored, their u unused)
    for (int q = tid; q < (256 - vl) * 8; q += kInThreads) {
      const uint32_t off = (uint32_t)(vl + (q >> 3)) * 128u + (uint32_t)(q & 7) * 16u;
      *reinterpret_cast<uint4*>(sU + off) = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(sY + off) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  fence_proxy_async_smem();
  ok = __syncthreads_and(ok) != 0;

  for (int m = 0; m < 2 && ok; ++m) {
    const int l0 = 128 * m;
    const int r = 32 * qd + lane, l = l0 + r;
    if (l0 >= lim) {  // no row of this half is produced: its per-row sums are 0
      if (hc == 0) {
        rows4[kh * 256 + l] = 0.f;
        rows4[plane + kh * 256 + l] = 0.f;
      }
      continue;
    }
    const bool lv = l < vl;
    // ---- accY over source blocks j = m .. 1 (s >= l); none when l0 >= vl (then no row is valid)
    for (int j = m; j < 2 && ok; ++j) {
      if (128 * j >= vl) break;
      // A block: rows s = 128 j + sl, columns l = l0 + ll, the decay-weighted CB, 16 bits.
      // Two passes of four chunks: the eight 16-byte loads of a pass are issued together
      // (the whole tile is inside the chunk's CB; entries outside s >= l, s, l < len are
      // loaded and dropped).
#pragma unroll
      for (int i0 = 0; i0 < 8; i0 += 4) {
        float4 ca[4], cb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int q = tid + kInThreads * (i0 + i), sl = q >> 4, l8 = (q & 15) * 8;
          const float* src = CB + kg + (long long)(128 * j + sl) * 256 + l0 + l8;
          ca[i] = __ldg(reinterpret_cast<const float4*>(src));
          cb[i] = __ldg(reinterpret_cast<const float4*>(src + 4));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int q = tid + kInThreads * (i0 + i), sl = q >> 4, l8 = (q & 15) * 8;
          const int s_ = 128 * j + sl, lb = l0 + l8;
          const float cb8[8] = {ca[i].x, ca[i].y, ca[i].z, ca[i].w, cb[i].x, cb[i].y, cb[i].z, cb[i].w};
          const float cs_ = cms[s_];
          const bool srow = s_ < vl;
          float x[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int le = lb + e;
            x[e] = (srow && le <= s_) ? cb8[e] * __expf(fminf(cs_ - cms[le], 0.f)) : 0.f;
          }
          const uint4 v = make_uint4(pack2<T16>(x[0], x[1]), pack2<T16>(x[2], x[3]), pack2<T16>(x[4], x[5]),
                                     pack2<T16>(x[6], x[7]));
          *reinterpret_cast<uint4*>(sA + (l8 >> 6) * 16384 + sw128_off((uint32_t)sl, (uint32_t)((l8 & 63) >> 3))) = v;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_f16(tmem + T_Y, sdesc_sw128(smem_u32(sA) + ks * 2048, 16384, 1024),
                   sdesc_sw128(smem_u32(sY) + (128 * j + 16 * ks) * 128, 16, 1024), ID_Y,
                   (j > m || ks > 0) ? 1u : 0u);
        umma_commit(bar_mma);
      }
      ok = __syncthreads_and(mbar_wait(bar_mma, uses & 1, kSiteBwdTcMma)) != 0;  // sA is reused
      ++uses;
      tc_fence_after();
    }
    if (!ok) break;
    // ---- G^T[s, l] = u[s] . y_grad[l] over source blocks j = 0 .. m (s <= l), one block at a
    // time; TMEM lane = source token s, so CB / CB_grad rows are read and added coalesced
    for (int j = 0; j <= m && ok; ++j) {
      if (128 * j >= vl) break;
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_f16(tmem + T_G, sdesc_sw128(smem_u32(sU) + 128 * j * 128 + ks * 32, 16, 1024),
                   sdesc_sw128(smem_u32(sY) + l0 * 128 + ks * 32, 16, 1024), ID_G, ks > 0 ? 1u : 0u);
        umma_commit(bar_mma);
      }
      ok = __syncthreads_and(mbar_wait(bar_mma, uses & 1, kSiteBwdTcMma)) != 0;
      ++uses;
      tc_fence_after();
      if (!ok) break;
      const int ws0 = 128 * j + 32 * qd;  // first source token of this warp
      const int sj = ws0 + lane;
      const bool sv = sj < vl;
      const float dsj = dts[sj], csj = cms[sj];
      float cacc = 0.f;
#pragma unroll 1
      for (int c = 2 * hc; c < 2 * hc + 2; ++c) {
        const int lb = l0 + 32 * c;  // columns l = lb + i
        if (lb + 31 < ws0 || ws0 >= vl || lb >= vl) continue;  // warp-uniform: no pair s <= l < len
        const float cml = cms[lb + lane];  // lane i: cum of column l = lb + i (shuffled below)
        // CB[l, s] for the 32 columns (inside the chunk's tile; pairs outside s <= l < len dropped)
        float w[32];
        const float* cbcol = CB + kg + (long long)lb * 256 + sj;
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = __ldg(cbcol + i * 256);
        uint32_t v[32];
        tmem_ld32(tmem + tl + T_G + 32 * c, v);
        tmem_wait_ld();
        float* cbgcol = CBg + kg + (long long)lb * 256 + sj;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int l_ = lb + i;
          const bool pv = sv && sj <= l_ && l_ < vl;
          const float cl = __shfl_sync(0xffffffffu, cml, i);  // every lane takes part
          const float cbg = pv ? __uint_as_float(v[i]) * dsj * __expf(fminf(cl - csj, 0.f)) : 0.f;
          if (pv) atomicAdd(cbgcol + i * 256, cbg);
          w[i] = (pv && sj < l_) ? cbg * w[i] : 0.f;
          cacc += w[i];
        }
        // row sums over the warp's 32 source tokens: lane i ends with the sum for l = lb + i
        atomicAdd(&rws[lb + lane], warp_transpose_sum32(w));
      }
      atomicAdd(&cols[sj], cacc);
      tc_fence_before();
      __syncthreads();  // every thread has read G before the next block overwrites it
    }
    if (!ok) break;
    // ---- per-row work on this warp's 32 columns p: u_grad, and the ddt / gB partials
    {
      uint32_t yv[32];
      tmem_ld32(tmem + tl + T_Y + 32 * hc, yv);
      tmem_wait_ld();
      float dpart = 0.f, bpart = 0.f;
      uint4* grow = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(u_grad) + ((ci.tok0 + l) * H + h) * 64 + 32 * hc);
      if (!lv) {  // rows at or past the length: u_grad 0
        if (l < lim) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) grow[c8] = make_uint4(0u, 0u, 0u, 0u);
        }
      } else {
        const float d = dts[l];
        // accS [p / 4][l][4]: lanes read consecutive 16-byte pieces
        const float4* srow = reinterpret_cast<const float4*>(accS) + (kh * 16 + 8 * hc) * 256 + l;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          const float4 s0 = srow[(2 * c8) * 256];
          const float4 s1 = srow[(2 * c8 + 1) * 256];
          const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
          const uint4 u8 = *reinterpret_cast<const uint4*>(sU + sw128_off((uint32_t)l, (uint32_t)(4 * hc + c8)));
          const uint32_t uw[4] = {u8.x, u8.y, u8.z, u8.w};
          uint32_t og[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 uf = unpack2<T16>(uw[q]);
            const float a0 = sv[2 * q] + __uint_as_float(yv[8 * c8 + 2 * q]);
            const float a1 = sv[2 * q + 1] + __uint_as_float(yv[8 * c8 + 2 * q + 1]);
            dpart = fmaf(a0, uf.x, fmaf(a1, uf.y, dpart));
            bpart = fmaf(sv[2 * q], uf.x, fmaf(sv[2 * q + 1], uf.y, bpart));
            og[q] = pack2<T16>(a0 * d, a1 * d);
          }
          grow[c8] = make_uint4(og[0], og[1], og[2], og[3]);
        }
      }
      dpp[hc * 128 + r] = dpart;
      bpp[hc * 128 + r] = bpart;
    }
    tc_fence_before();
    __syncthreads();
    if (hc == 0) {
      // rows4: [0] ddt, [1] gB, [2] rows, [3] cols, each (chunk, head, 256)
      rows4[kh * 256 + l] = dpp[r] + dpp[128 + r];
      rows4[plane + kh * 256 + l] = lv ? (bpp[r] + bpp[128 + r]) * dts[l] : 0.f;
    }
    __syncthreads();  // partials read before the next half writes them
  }
  if (ok) {
    rows4[2 * plane + kh * 256 + tid] = rws[tid];
    rows4[3 * plane + kh * 256 + tid] = cols[tid];
  } else if (tid == 0 && uses > 0) {
    mbar_wait(bar_mma, (uses - 1) & 1, kSiteBwdTcMma);  // let an MMA in flight land (bounded)
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

template <bool BF16, typename YT>
cudaError_t launch_intra_typed(const LaunchCtx& c, const BwdArgs& a) {
  CUtensorMap mu, my;
  if (!make_map_3d(&mu, a.u, BF16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&my, sizeof(YT) == 2 ? a.y_grad : a.u, BF16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128))
    return cudaErrorInvalidValue;
  auto kern = bwd_intra_tc_kernel<BF16, YT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kInSmem);
  if (e != cudaSuccess) return e;
  const long long plane = (long long)c.nchunks_max * c.H * 256;
  kern<<<dim3((unsigned)c.H, (unsigned)c.nchunks_max), kInThreads, kInSmem, c.stream>>>(
      mu, my, a.u, reinterpret_cast<const YT*>(a.y_grad), a.dt, a.cum, a.CB, a.accS, a.CBg, a.u_grad, a.rows4,
      c.cm, c.H, c.G, plane);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// State-side products per (chunk, group, 128-row half), looping over the group's heads, so
// that B_grad and C_grad sum over the heads inside TMEM (no atomics):
//   accS_h[l,p] = scale_l sum_n B[l,n] hg_h[p,n]              (stored per head, blocked)
//   Q_h[l,p]    = sum_n C[l,n] prev_h[p,n];  gC_h[l] = sum_p (e_l y_h[l,p]) Q_h[l,p]
//   B_grad[l,:] = sum_h sum_p (w_l u_h[l,p]) hg_h[p,:]       (TMEM, over the heads)
//   C_grad[l,:] = sum_h sum_p (e_l y_h[l,p]) prev_h[p,:]
// with w_l = scale_l dt_l and e_l = exp(cum_l) of head h (0 at or past the length). The
// 16-bit prev / hg (from the state pass) and u, y_grad rows arrive by TMA in a two-stage ring
// over the heads; u and y_grad rows are scaled in place (16-bit products), B and C rows stay.
// 8 warps: warps w and w + 4 share TMEM lane quadrant w % 4 and split the columns.
// ---------------------------------------------------------------------------
constexpr int kSgThreads = 256;
constexpr int kSgStage = 65536;  // hg16 | prev16 (2 n-blocks x 64 p x 128 B each) | u | y (128 rows x 128 B)
constexpr size_t kSgSmem = 1024 + 65536 + 2 * kSgStage;

template <bool BF16>
__global__ void __launch_bounds__(kSgThreads, 1) bwd_state_grad_grp_tc_kernel(
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_c,
    const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_y,
    const __grid_constant__ CUtensorMap tm_hg, const __grid_constant__ CUtensorMap tm_pv, const float* __restrict__ dt,
    const float* __restrict__ cum, float* __restrict__ accS_out, float* __restrict__ Bgrad,
    float* __restrict__ Cgrad, float* __restrict__ gC_out, ChunkMap cm, int H, int G) {
  using T16 = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  uint8_t* sB = sm;          // [2 n-blocks][128 rows][128 B]
  uint8_t* sC = sm + 32768;  // same
  auto sHg = [&](int st) { return sm + 65536 + kSgStage * st; };
  auto sPv = [&](int st) { return sHg(st) + 16384; };
  auto sU = [&](int st) { return sHg(st) + 32768; };
  auto sY = [&](int st) { return sHg(st) + 49152; };
  __shared__ float sS[2][128], wS[2][128], eS[2][128], gcp[2][128];
  __shared__ uint64_t bars[4];  // B / C, stage[2], mma
  __shared__ uint32_t tslot[1];
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int m = blockIdx.x, g = blockIdx.y, k = blockIdx.z;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int l0 = 128 * m;
  if (l0 >= ci.lim) return;
  const int HG = H / G, vl = ci.vlim;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = (warp & 3) * 32 + lane, hc = warp >> 2, l = l0 + r;
  const uint32_t tl = (uint32_t)((warp & 3) * 32) << 16;
  const int t0 = (int)(ci.tok0 + l0);
  auto factors = [&](int st, int j) {  // row factors of head g HG + j (threads < 128)
    if (tid < 128) {
      const long long kh = (long long)k * H + g * HG + j;
      const int li = l0 + tid;
      const float c = cum[kh * 256 + li], clast = cum[kh * 256 + 255];
      const float sc = li < vl ? __expf(fminf(clast - c, 0.f)) : 0.f;
      sS[st][tid] = sc;
      wS[st][tid] = sc * dt[kh * 256 + li];
      eS[st][tid] = li < vl ? __expf(c) : 0.f;
    }
  };
  int ld_iss[2] = {0, 0}, ld_wt[2] = {0, 0}, mma_iss = 0, mma_wt = 0;  // thread 0's books
  auto load_stage = [&](int st, int j) {  // thread 0
    const int h = g * HG + j, kh = k * H + h;
    mbar_expect_tx(bar(1 + st), (uint32_t)kSgStage);
    tma_load_3d(smem_u32(sHg(st)), &tm_hg, 0, 0, kh, bar(1 + st));
    tma_load_3d(smem_u32(sHg(st)) + 8192, &tm_hg, 64, 0, kh, bar(1 + st));
    tma_load_3d(smem_u32(sPv(st)), &tm_pv, 0, 0, kh, bar(1 + st));
    tma_load_3d(smem_u32(sPv(st)) + 8192, &tm_pv, 64, 0, kh, bar(1 + st));
    tma_load_3d(smem_u32(sU(st)), &tm_u, 0, h, t0, bar(1 + st));
    tma_load_3d(smem_u32(sY(st)), &tm_y, 0, h, t0, bar(1 + st));
    ++ld_iss[st];
  };
  if (tid == 0) {
    prefetch_tmap(&tm_b);
    prefetch_tmap(&tm_c);
    prefetch_tmap(&tm_u);
    prefetch_tmap(&tm_y);
    prefetch_tmap(&tm_hg);
    prefetch_tmap(&tm_pv);
    for (int i = 0; i < 4; ++i) mbar_init(bar(i), 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 512);
  factors(0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  constexpr uint32_t T_S = 0, T_Q = 64, T_BG = 128, T_CG = 256;
  constexpr uint32_t ID_S = idesc_f16(128, 64, BF16, false, false);  // K = n
  constexpr uint32_t ID_G = idesc_f16(128, 128, BF16, false, true);  // K = p, N = n MN-major
  if (tid == 0) {
    mbar_expect_tx(bar(0), 65536u);
    tma_load_3d(smem_u32(sB), &tm_b, 0, g, t0, bar(0));
    tma_load_3d(smem_u32(sB) + 16384, &tm_b, 64, g, t0, bar(0));
    tma_load_3d(smem_u32(sC), &tm_c, 0, g, t0, bar(0));
    tma_load_3d(smem_u32(sC) + 16384, &tm_c, 64, g, t0, bar(0));
    load_stage(0, 0);
  }
  bool ok = mbar_wait(bar(0), 0, kSiteBwdTcTma);
  if (ok && vl - l0 < 128) {  // B / C rows at or past the length: zeros
    for (int q = tid; q < (128 - max(vl - l0, 0)) * 8; q += kSgThreads) {
      const uint32_t off = (uint32_t)(max(vl - l0, 0) + (q >> 3)) * 128u + (uint32_t)(q & 7) * 16u;
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(sB + off) = z;
      *reinterpret_cast<uint4*>(sB + 16384 + off) = z;
      *reinterpret_cast<uint4*>(sC + off) = z;
      *reinterpret_cast<uint4*>(sC + 16384 + off) = z;
    }
  }
  ok = __syncthreads_and(ok) != 0;
  for (int j = 0; j < HG && ok; ++j) {
    const int st = j & 1;
    const long long kh = (long long)k * H + g * HG + j;
    if (j + 1 < HG) {  // the next head's stage: its previous user's MMAs completed last iteration
      if (tid == 0) load_stage(st ^ 1, j + 1);
      factors(st ^ 1, j + 1);
    }
    bool got = mbar_wait(bar(1 + st), (j >> 1) & 1, kSiteBwdTcTma);
    if (tid == 0 && got) ++ld_wt[st];
    ok = __syncthreads_and(got) != 0;
    if (!ok) break;
    // u rows times w_l and y_grad rows times e_l, in place (rows past the length become 0)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSgThreads * i, row = q >> 3;
      uint4* pu = reinterpret_cast<uint4*>(sU(st) + q * 16);
      uint4* py = reinterpret_cast<uint4*>(sY(st) + q * 16);
      const float w = wS[st][row], e = eS[st][row];
      *pu = w == 0.f ? make_uint4(0u, 0u, 0u, 0u) : scaled8<T16>(*pu, w);
      *py = e == 0.f ? make_uint4(0u, 0u, 0u, 0u) : scaled8<T16>(*py, e);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t hf = ks >> 2, kk = (ks & 3) * 32;
        umma_f16(tmem + T_S, sdesc_sw128(smem_u32(sB) + hf * 16384 + kk, 16, 1024),
                 sdesc_sw128(smem_u32(sHg(st)) + hf * 8192 + kk, 16, 1024), ID_S, ks > 0 ? 1u : 0u);
        umma_f16(tmem + T_Q, sdesc_sw128(smem_u32(sC) + hf * 16384 + kk, 16, 1024),
                 sdesc_sw128(smem_u32(sPv(st)) + hf * 8192 + kk, 16, 1024), ID_S, ks > 0 ? 1u : 0u);
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint32_t acc = (j > 0 || ks > 0) ? 1u : 0u;
        umma_f16(tmem + T_BG, sdesc_sw128(smem_u32(sU(st)) + ks * 32, 16, 1024),
                 sdesc_sw128(smem_u32(sHg(st)) + ks * 2048, 8192, 1024), ID_G, acc);
        umma_f16(tmem + T_CG, sdesc_sw128(smem_u32(sY(st)) + ks * 32, 16, 1024),
                 sdesc_sw128(smem_u32(sPv(st)) + ks * 2048, 8192, 1024), ID_G, acc);
      }
      umma_commit(bar(3));
      ++mma_iss;
    }
    got = mbar_wait(bar(3), mma_wt & 1, kSiteBwdTcMma);
    if (got) ++mma_wt;
    ok = __syncthreads_and(got) != 0;
    if (!ok) break;
    tc_fence_after();
    {
      // accS row l, this thread's 32 columns p, times scale_l, stored blocked [p / 4][l][4]
      uint32_t v[32];
      tmem_ld32(tmem + tl + T_S + 32 * hc, v);
      tmem_wait_ld();
      const float sc = sS[st][r];
      float4* o = reinterpret_cast<float4*>(accS_out) + (kh * 16 + 8 * hc) * 256 + l;
#pragma unroll
      for (int e = 0; e < 32; e += 4)
        o[(e >> 2) * 256] = make_float4(__uint_as_float(v[e]) * sc, __uint_as_float(v[e + 1]) * sc,
                                        __uint_as_float(v[e + 2]) * sc, __uint_as_float(v[e + 3]) * sc);
      // gC partial: the scaled y_grad row (shared memory) against Q's row
      tmem_ld32(tmem + tl + T_Q + 32 * hc, v);
      tmem_wait_ld();
      float acc = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        const uint4 y8 = *reinterpret_cast<const uint4*>(sY(st) + sw128_off((uint32_t)r, (uint32_t)(4 * hc + c8)));
        const uint32_t yw[4] = {y8.x, y8.y, y8.z, y8.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 yf = unpack2<T16>(yw[q]);
          acc = fmaf(yf.x, __uint_as_float(v[8 * c8 + 2 * q]), fmaf(yf.y, __uint_as_float(v[8 * c8 + 2 * q + 1]), acc));
        }
      }
      gcp[hc][r] = acc;
    }
    tc_fence_before();
    __syncthreads();  // T_S / T_Q read before the next head's products, partials complete
    if (hc == 0) gC_out[kh * 256 + l] = l < vl ? gcp[0][r] + gcp[1][r] : 0.f;
  }
  if (ok) {
    // B_grad / C_grad rows of this half: 64 of the 128 columns per thread, plain stores
    tc_fence_after();
#pragma unroll 1
    for (int part = 0; part < 2; ++part) {
      float* dst = (part ? Cgrad : Bgrad) + ((ci.tok0 + l) * G + g) * 128 + 64 * hc;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + tl + (part ? T_CG : T_BG) + 64 * hc + 32 * c, v);
        tmem_wait_ld();
        if (l < ci.lim) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(dst + 32 * c + e) =
                make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]), __uint_as_float(v[e + 2]),
                            __uint_as_float(v[e + 3]));
        }
      }
    }
  } else if (tid == 0) {  // let what is in flight land before TMEM and the CTA go away (bounded)
    while (mma_wt < mma_iss && mbar_wait(bar(3), mma_wt & 1, kSiteBwdTcMma)) ++mma_wt;
    for (int st = 0; st < 2; ++st)
      while (ld_wt[st] < ld_iss[st] && mbar_wait(bar(1 + st), ld_wt[st] & 1, kSiteBwdTcTma)) ++ld_wt[st];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <bool BF16>
cudaError_t launch_grp_typed(const LaunchCtx& c, const BwdArgs& a, const void* y16) {
  CUtensorMap mb, mc, mu, my, mh, mp;
  const uint64_t nkh = (uint64_t)c.nchunks_max * (uint64_t)c.H;
  if (!make_map_3d(&mb, a.B, BF16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mc, a.C, BF16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mu, a.u, BF16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&my, y16, BF16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mh, a.hg16, BF16, 128, 64, nkh, 64, 64, 1) ||
      !make_map_3d(&mp, a.prev16, BF16, 128, 64, nkh, 64, 64, 1))
    return cudaErrorInvalidValue;
  auto kern = bwd_state_grad_grp_tc_kernel<BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSgSmem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(2u, (unsigned)c.G, (unsigned)c.nchunks_max), kSgThreads, kSgSmem, c.stream>>>(
      mb, mc, mu, my, mh, mp, a.dt, a.cum, a.accS, a.B_grad, a.C_grad, a.gC, c.cm, c.H, c.G);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// CB = C B^T and the bmm backward on tcgen05 (ssd_bwd.cu bwd_cb_kernel / bwd_bmm_kernel;
// forward_kernel.py:270-328, backward_kernel.py:686-780), per (chunk, group, 128-row block m):
//   cb:  CB[l,s] = sum_n C[l,n] B[s,n] for l in block m, s in blocks 0..m      (K = n)
//   bmm product 0: C_grad[l,:] += sum_{s <= l} CB_grad[l,s] B[s,:]           (K = s)
//   bmm product 1: B_grad[s,:] += sum_{l >= s} CB_grad[l,s] C[l,:]           (K = l)
// B / C rows arrive by TMA (rows at or past the length zeroed in shared memory); CB_grad
// (fp32, the group's heads summed) is rounded to 16 bits into the A operand, K-major for
// product 0 and MN-major (rows read as columns) for product 1. The bmm rows are added to the
// gradients read-modify-write (each row belongs to one CTA).
// ---------------------------------------------------------------------------
constexpr int kBmThreads = 256;
constexpr size_t kBmSmem = 1024 + 65536;
constexpr size_t kCbSmem = 1024 + 3 * 32768;

// Zeros rows [from, 128) of a [2 n-blocks][128 rows][128 B] tile.
__device__ __forceinline__ void zero_rows_tile(uint8_t* t, int from) {
  from = max(from, 0);
  for (int q = threadIdx.x; q < (128 - from) * 8; q += blockDim.x) {
    const uint32_t off = (uint32_t)(from + (q >> 3)) * 128u + (uint32_t)(q & 7) * 16u;
    *reinterpret_cast<uint4*>(t + off) = make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(t + 16384 + off) = make_uint4(0u, 0u, 0u, 0u);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(kBmThreads) bwd_cb_tc_kernel(const __grid_constant__ CUtensorMap tm_b,
                                                               const __grid_constant__ CUtensorMap tm_c,
                                                               float* __restrict__ CB, ChunkMap cm, int G) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  uint8_t* sC = sm;  // C rows of block m; then B rows of blocks 0 and 1
  auto sBr = [&](int j) { return sm + 32768 * (1 + j); };
  __shared__ uint64_t bars[2];
  __shared__ uint32_t tslot[1];
  const uint32_t bar_tma = smem_u32(&bars[0]), bar_mma = smem_u32(&bars[1]);
  const int m = blockIdx.x, g = blockIdx.y, k = blockIdx.z;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int vl = ci.vlim, r0 = 128 * m;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = (warp & 3) * 32 + lane, hc = warp >> 2;
  const uint32_t tl = (uint32_t)((warp & 3) * 32) << 16;
  if (tid == 0) {
    prefetch_tmap(&tm_b);
    prefetch_tmap(&tm_c);
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    mbar_expect_tx(bar_tma, 32768u * (uint32_t)(m + 2));
    const int t0 = (int)ci.tok0;
    tma_load_3d(smem_u32(sC), &tm_c, 0, g, t0 + r0, bar_tma);
    tma_load_3d(smem_u32(sC) + 16384, &tm_c, 64, g, t0 + r0, bar_tma);
    for (int j = 0; j <= m; ++j) {
      tma_load_3d(smem_u32(sBr(j)), &tm_b, 0, g, t0 + 128 * j, bar_tma);
      tma_load_3d(smem_u32(sBr(j)) + 16384, &tm_b, 64, g, t0 + 128 * j, bar_tma);
    }
  }
  bool ok = mbar_wait(bar_tma, 0, kSiteBwdTcTma);
  if (ok) {
    zero_rows_tile(sC, vl - r0);
    for (int j = 0; j <= m; ++j) zero_rows_tile(sBr(j), vl - 128 * j);
  }
  fence_proxy_async_smem();
  tc_fence_before();
  ok = __syncthreads_and(ok) != 0;
  if (ok && tid == 0) {
    tc_fence_after();
    constexpr uint32_t ID = idesc_f16(128, 128, BF16, false, false);
    for (int j = 0; j <= m; ++j)
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t off = (uint32_t)(ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u;
        umma_f16(tmem + 128 * j, sdesc_sw128(smem_u32(sC) + off, 16, 1024), sdesc_sw128(smem_u32(sBr(j)) + off, 16, 1024),
                 ID, ks > 0 ? 1u : 0u);
      }
    umma_commit(bar_mma);
  }
  if (ok) ok = __syncthreads_and(mbar_wait(bar_mma, 0, kSiteBwdTcMma)) != 0;
  if (ok) {
    tc_fence_after();
    // row l = r0 + r: this thread's half of the 128 (m + 1) columns, fp32
    const int ncol = 64 * (m + 1);
    float* dst = CB + ((long long)k * G + g) * 65536 + (long long)(r0 + r) * 256 + ncol * hc;
#pragma unroll 1
    for (int c = 0; c < ncol; c += 32) {
      uint32_t v[32];
      tmem_ld32(tmem + tl + (uint32_t)(ncol * hc + c), v);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; e += 4)
        *reinterpret_cast<float4*>(dst + c + e) = make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]),
                                                              __uint_as_float(v[e + 2]), __uint_as_float(v[e + 3]));
    }
  } else if (tid == 0) {
    mbar_wait(bar_mma, 0, kSiteBwdTcMma);  // an MMA that was issued lands before TMEM goes (bounded)
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

template <bool BF16>
__global__ void __launch_bounds__(kBmThreads) bwd_bmm_tc_kernel(const __grid_constant__ CUtensorMap tm_b,
                                                                const __grid_constant__ CUtensorMap tm_c,
                                                                const float* __restrict__ CBg, float* __restrict__ Bgrad,
                                                                float* __restrict__ Cgrad, ChunkMap cm, int G) {
  using T16 = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  uint8_t* sA = sm;          // 16-bit CB_grad block [2 64-blocks][128 rows][128 B]
  uint8_t* sX = sm + 32768;  // B or C rows [2 n-blocks][128 rows][128 B]
  __shared__ uint64_t bars[2];
  __shared__ uint32_t tslot[1];
  const uint32_t bar_tma = smem_u32(&bars[0]), bar_mma = smem_u32(&bars[1]);
  const int prod = blockIdx.x >> 1, m = blockIdx.x & 1, g = blockIdx.y, k = blockIdx.z;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int vl = ci.vlim, r0 = 128 * m;
  if (r0 >= vl) return;  // rows at or past the length receive nothing
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = (warp & 3) * 32 + lane, hc = warp >> 2;
  const uint32_t tl = (uint32_t)((warp & 3) * 32) << 16;
  const CUtensorMap* mx = prod == 0 ? &tm_b : &tm_c;
  const float* cbg = CBg + ((long long)k * G + g) * 65536;
  if (tid == 0) {
    prefetch_tmap(mx);
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t ID = prod == 0 ? idesc_f16(128, 128, BF16, false, true) : idesc_f16(128, 128, BF16, true, true);
  // source blocks: product 0 s-blocks 0..m, product 1 l-blocks m..1 (below the length)
  const int jb = prod == 0 ? 0 : m, je = prod == 0 ? m : 1;
  bool ok = true;
  int uses = 0;
  for (int j = jb; j <= je && ok; ++j) {
    if (128 * j >= vl) break;
    if (tid == 0) {
      mbar_expect_tx(bar_tma, 32768u);
      tma_load_3d(smem_u32(sX), mx, 0, g, (int)ci.tok0 + 128 * j, bar_tma);
      tma_load_3d(smem_u32(sX) + 16384, mx, 64, g, (int)ci.tok0 + 128 * j, bar_tma);
    }
    // A: product 0 rows l = r0 + i, columns s = 128 j + c (K-major); product 1 CB_grad rows
    // l = 128 j + i read as the K index, columns s = r0 + c as M (MN-major): one layout,
    // [c / 64][i][c % 64], swizzled
#pragma unroll 2
    for (int i0 = 0; i0 < 8; i0 += 4) {
      float4 va[4], vb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int q = tid + kBmThreads * (i0 + i), row = q >> 4, c8 = q & 15;
        const float* src = prod == 0 ? cbg + (long long)(r0 + row) * 256 + 128 * j + 8 * c8
                                     : cbg + (long long)(128 * j + row) * 256 + r0 + 8 * c8;
        va[i] = __ldg(reinterpret_cast<const float4*>(src));
        vb[i] = __ldg(reinterpret_cast<const float4*>(src + 4));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int q = tid + kBmThreads * (i0 + i), row = q >> 4, c8 = q & 15;
        *reinterpret_cast<uint4*>(sA + (c8 >> 3) * 16384 + sw128_off((uint32_t)row, (uint32_t)(c8 & 7))) =
            make_uint4(pack2<T16>(va[i].x, va[i].y), pack2<T16>(va[i].z, va[i].w), pack2<T16>(vb[i].x, vb[i].y),
                       pack2<T16>(vb[i].z, vb[i].w));
      }
    }
    bool got = mbar_wait(bar_tma, uses & 1, kSiteBwdTcTma);
    if (got) zero_rows_tile(sX, vl - 128 * j);
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(got) != 0;
    if (!ok) break;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t ad = prod == 0
                                ? sdesc_sw128(smem_u32(sA) + (uint32_t)(ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u, 16, 1024)
                                : sdesc_sw128(smem_u32(sA) + (uint32_t)ks * 2048u, 16384, 1024);
        umma_f16(tmem, ad, sdesc_sw128(smem_u32(sX) + (uint32_t)ks * 2048u, 16384, 1024), ID,
                 (j > jb || ks > 0) ? 1u : 0u);
      }
      umma_commit(bar_mma);
    }
    ok = __syncthreads_and(mbar_wait(bar_mma, uses & 1, kSiteBwdTcMma)) != 0;  // sA, sX reused
    ++uses;
    tc_fence_after();
  }
  if (ok && uses > 0) {
    const int row = r0 + r;
    float* out = (prod == 0 ? Cgrad : Bgrad) + ((ci.tok0 + row) * G + g) * 128 + 64 * hc;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint32_t v[32];
      tmem_ld32(tmem + tl + (uint32_t)(64 * hc + 32 * c), v);
      tmem_wait_ld();
      if (row < ci.lim) {
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          float4 o = *reinterpret_cast<float4*>(out + 32 * c + e);
          o.x += __uint_as_float(v[e]);
          o.y += __uint_as_float(v[e + 1]);
          o.z += __uint_as_float(v[e + 2]);
          o.w += __uint_as_float(v[e + 3]);
          *reinterpret_cast<float4*>(out + 32 * c + e) = o;
        }
      }
    }
  } else if (!ok && tid == 0 && uses > 0) {
    mbar_wait(bar_mma, (uses - 1) & 1, kSiteBwdTcMma);  // bounded
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

template <bool BF16>
cudaError_t launch_cb_bmm_typed(const LaunchCtx& c, const BwdArgs& a, bool bmm) {
  CUtensorMap mb, mc;
  if (!make_map_3d(&mb, a.B, BF16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mc, a.C, BF16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128))
    return cudaErrorInvalidValue;
  cudaError_t e;
  if (bmm) {
    if ((e = cudaFuncSetAttribute(bwd_bmm_tc_kernel<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBmSmem)))
      return e;
    bwd_bmm_tc_kernel<BF16><<<dim3(4u, (unsigned)c.G, (unsigned)c.nchunks_max), kBmThreads, kBmSmem, c.stream>>>(
        mb, mc, a.CBg, a.B_grad, a.C_grad, c.cm, c.G);
  } else {
    if ((e = cudaFuncSetAttribute(bwd_cb_tc_kernel<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kCbSmem)))
      return e;
    bwd_cb_tc_kernel<BF16><<<dim3(2u, (unsigned)c.G, (unsigned)c.nchunks_max), kBmThreads, kCbSmem, c.stream>>>(
        mb, mc, a.CB, c.cm, c.G);
  }
  return cudaGetLastError();
}
}  // namespace

bool bwd_state_grad_tc_supported(int x_dtype, int y_dtype, int P, int N, int cs) {
  const bool x16 = x_dtype == SSD_BF16 || x_dtype == SSD_F16;
  return x16 && (y_dtype == SSD_F32 || y_dtype == x_dtype) && P == 64 && N == 128 && cs == 256;
}


cudaError_t launch_bwd_chunk_states_tc(const LaunchCtx& c, const BwdArgs& a) {
  if (c.nchunks_max > 65535 || c.H > 65535) return cudaErrorInvalidValue;
  if (a.x_dtype == SSD_BF16) {
    if (a.y_dtype == SSD_F32) return launch_states_typed<true, float>(c, a);
    return launch_states_typed<true, __nv_bfloat16>(c, a);
  }
  if (a.y_dtype == SSD_F32) return launch_states_typed<false, float>(c, a);
  return launch_states_typed<false, __half>(c, a);
}

cudaError_t launch_bwd_state_grad_grp_tc(const LaunchCtx& c, const BwdArgs& a) {
  if (c.nchunks_max > 65535 || c.G > 65535) return cudaErrorInvalidValue;
  const void* y16 = a.y_dtype == SSD_F32 ? (const void*)a.y16 : a.y_grad;  // y16: written by the recompute
  return a.x_dtype == SSD_BF16 ? launch_grp_typed<true>(c, a, y16) : launch_grp_typed<false>(c, a, y16);
}

cudaError_t launch_bwd_cb_tc(const LaunchCtx& c, const BwdArgs& a) {
  if (c.nchunks_max > 65535 || c.G > 65535) return cudaErrorInvalidValue;
  return a.x_dtype == SSD_BF16 ? launch_cb_bmm_typed<true>(c, a, false) : launch_cb_bmm_typed<false>(c, a, false);
}

cudaError_t launch_bwd_bmm_tc(const LaunchCtx& c, const BwdArgs& a) {
  if (c.nchunks_max > 65535 || c.G > 65535) return cudaErrorInvalidValue;
  return a.x_dtype == SSD_BF16 ? launch_cb_bmm_typed<true>(c, a, true) : launch_cb_bmm_typed<false>(c, a, true);
}

cudaError_t launch_bwd_intra_tc(const LaunchCtx& c, const BwdArgs& a) {
  if (c.nchunks_max > 65535 || c.H > 65535) return cudaErrorInvalidValue;
  BwdArgs b = a;
  if (a.y_dtype == SSD_F32) b.y_grad = a.y16;  // the 16-bit copy the recompute wrote
  if (a.x_dtype == SSD_BF16) return launch_intra_typed<true, __nv_bfloat16>(c, b);
  return launch_intra_typed<false, __half>(c, b);
}

SSDB200_DEFINE_ERROR_FETCH(fetch_error_bwd_tc)

}  // namespace ssdb200
