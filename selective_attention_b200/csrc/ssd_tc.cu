// ssd_tc.cu - tensor-core (tcgen05 + TMA) SSD stages for 16-bit inputs with
// headdim 64, dstate 128, chunk 256.
//
// chunk_state (ssd_scan/forward_kernel.py:19-87 chunk_cumsum fused with :107-185),
// one CTA (4 warps) per (head, chunk), ~52 KB of shared memory (4 CTAs per SM):
//   dt, cum for the chunk's 256 tokens (shuffle scan), written for chunk_scan and
//   state_passing; then in two 128-token phases
//   S^T[n, p] += sum_l B[l, n] * (x[l, p] * w_l),  w_l = exp(min(cum_last - cum_l, 0)) * dt_l
//   M = 128 (dstate), N = 64 (headdim), K = 128 tokens per phase; both operands
//   MN-major (token rows of 128 B as TMA lands them); x is scaled by w_l in place.
//
// chunk_scan (ssd_scan/forward_kernel.py:350-455 with bmm_chunk :270-328 fused):
// persistent and warp-specialised (one CTA per SM, see tc_chunk_scan_kernel). For
// the 128 rows l of half m of a chunk and 128-token source blocks j = 0..m:
//   MMA1  CB_j[l, s]  = C[l, :] . B[s, :]          M 128, N 128, K 128 (K-major)
//   CB_j -> M_j[l, s] = CB * decay(l, s) * dt_s  (bf16/fp16, K-major, over the B tile)
//   MMA2  Yin[l, p]  += sum_s M_j[l, s] x[s, p]    M 128, N 64, K 128 (x MN-major)
//   MMA3  Yoff[l, p]  = C[l, :] . prev[:, p]        M 128, N 64, K 128 (prev16 stored
//                                                    [n][p], read MN-major)
//   y = exp(cum_l) * Yoff + Yin (+ D x) (* silu z)
// decay(l, s) = exp(min(cum_l - cum_s, 0)) with s <= l. Per 32x32 tile it is
// evaluated as exp(cum_l - cum_r) * exp(cum_r - cum_s), r the tile's last column,
// whenever cum is non-increasing (A <= 0 and dt >= 0, so min(., 0) is the identity)
// and, on diagonal tiles, the tile's own decay is below 80 (no overflow); otherwise
// element by element.
//
// All tiles use the 128-byte swizzle; accumulators are fp32 in TMEM. Every mbarrier
// wait is bounded: a CTA that gives up records a site code in the error flag and
// returns after its copies/MMAs get a last bounded wait and TMEM is released.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.cuh"

namespace ssdb200 {

using namespace sm100;

enum : unsigned int {
  kSiteStateTma = 0x101,
  kSiteStateMma = 0x102,
  kSiteScanTma = 0x201,
  kSiteScanMma1 = 0x202,
  kSiteScanMma2 = 0x203,
  kSiteScanConv = 0x204,
  kSiteScanEpi = 0x205,
};

template <bool BF16> struct T16Of;
template <> struct T16Of<true> { using type = __nv_bfloat16; };
template <> struct T16Of<false> { using type = __half; };

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) { return align1024_shared(p); }

// Scale the 16-byte chunk (8 elements of T16) by w (fp32 products, one rounding).
template <typename T16>
__device__ __forceinline__ uint4 scale8(uint4 a, float w) {
  float2 f;
  uint4 v;
  f = unpack2<T16>(a.x); v.x = pack2<T16>(f.x * w, f.y * w);
  f = unpack2<T16>(a.y); v.y = pack2<T16>(f.x * w, f.y * w);
  f = unpack2<T16>(a.z); v.z = pack2<T16>(f.x * w, f.y * w);
  f = unpack2<T16>(a.w); v.w = pack2<T16>(f.x * w, f.y * w);
  return v;
}

// Scale 8 elements by w2 = (w, w) in the 16-bit type itself (bf16x2 / f16x2
// multiplies: w and each product are rounded to the 16-bit type).
template <typename T16> __device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t w2);
template <> __device__ __forceinline__ uint32_t mul2<__nv_bfloat16>(uint32_t a, uint32_t w2) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&w2));
  return *reinterpret_cast<uint32_t*>(&r);
}
template <> __device__ __forceinline__ uint32_t mul2<__half>(uint32_t a, uint32_t w2) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&w2));
  return *reinterpret_cast<uint32_t*>(&r);
}
template <typename T16>
__device__ __forceinline__ uint4 scale8_packed(uint4 a, uint32_t w2) {
  return make_uint4(mul2<T16>(a.x, w2), mul2<T16>(a.y, w2), mul2<T16>(a.z, w2), mul2<T16>(a.w, w2));
}

// Transpose NP x NP 16-byte pieces across each group of NP lanes: lane li of a
// group enters with pieces 0..NP-1 of "its" row and leaves with piece li of the
// group's rows 0..NP-1. Rows held one per lane become whole-row stores: store j
// of the group then writes row j contiguously.
template <int NP>
__device__ __forceinline__ void lane_transpose(uint4 (&d)[NP], int li) {
#pragma unroll
  for (int msk = NP / 2; msk >= 1; msk >>= 1) {
    const bool upper = (li & msk) != 0;
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      if (q & msk) continue;
      const uint4 snd = upper ? d[q] : d[q | msk];
      uint4 rcv;
      rcv.x = __shfl_xor_sync(0xffffffffu, snd.x, msk);
      rcv.y = __shfl_xor_sync(0xffffffffu, snd.y, msk);
      rcv.z = __shfl_xor_sync(0xffffffffu, snd.z, msk);
      rcv.w = __shfl_xor_sync(0xffffffffu, snd.w, msk);
      if (upper) d[q] = rcv; else d[q | msk] = rcv;
    }
  }
}

// ===========================================================================
// chunk_state (+ chunk_cumsum)
// ===========================================================================
constexpr int kStateSmem = 32768 + 16384 + 1024 + 1024 + 64 + 64 + 1024;

// FUSE: compute dt / cum from delta_raw and write them; otherwise read them.
template <bool BF16, typename DT, bool FUSE>
__global__ void __launch_bounds__(128) tc_chunk_state_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_b,
    const float* __restrict__ A, const DT* __restrict__ delta_raw, const float* __restrict__ delta_bias,
    float* __restrict__ dt_io, float* __restrict__ cum_io, float* __restrict__ states, ChunkMap cm, int H,
    int hpg, int use_sp, float dmin, float dmax) {
  using T16 = typename T16Of<BF16>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB = smem;            // 2 x (128 rows x 128 B): dstate halves, one 128-token phase
  uint8_t* sX = smem + 32768;    // 128 rows x 128 B
  float* sW = reinterpret_cast<float*>(smem + 49152);
  float* sCum = sW + 256;
  float* sWarp = sCum + 256;     // 4 warp totals
  uint64_t* bars = reinterpret_cast<uint64_t*>(sWarp + 16);  // tma0, tma1, mma0, mma1
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 4);

  const int h = blockIdx.x, k = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int g = h / hpg;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t bar[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) bar[i] = smem_u32(&bars[i]);
  const bool two_phases = ci.lim > 128;

  if (tid == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_b);
#pragma unroll
    for (int i = 0; i < 4; ++i) mbar_init(bar[i], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const int t0 = (int)ci.tok0;

  if (tid == 0) {
    mbar_expect_tx(bar[0], 49152u);
    tma_load_3d(smem_u32(sX), &tm_x, 0, h, t0, bar[0]);
    tma_load_3d(smem_u32(sB), &tm_b, 0, g, t0, bar[0]);
    tma_load_3d(smem_u32(sB + 16384), &tm_b, 64, g, t0, bar[0]);
  }

  // ---- chunk_cumsum for (k, h): tokens 2*tid, 2*tid+1 ----
  const long long io = ((long long)k * H + h) * 256 + 2 * tid;
  float d[2], cum0, cum1;
  if constexpr (FUSE) {
    const float a = A[h];
    const float bias = delta_bias ? delta_bias[h] : 0.f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int l = 2 * tid + e;
      d[e] = 0.f;
      if (l < ci.vlim)
        d[e] = dt_transform(Ld<DT>::f(delta_raw + (ci.tok0 + l) * (long long)H + h) + bias, use_sp, dmin, dmax);
    }
    const float c0 = d[0] * a;
    const float tot = c0 + d[1] * a;
    float incl = tot;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    if (lane == 31) sWarp[warp] = incl;
    __syncthreads();
    float wbase = 0.f;
    for (int w = 0; w < warp; ++w) wbase += sWarp[w];
    const float excl = wbase + incl - tot;
    cum0 = excl + c0;
    cum1 = excl + tot;
    *reinterpret_cast<float2*>(dt_io + io) = make_float2(d[0], d[1]);
    *reinterpret_cast<float2*>(cum_io + io) = make_float2(cum0, cum1);
  } else {
    const float2 dv = *reinterpret_cast<const float2*>(dt_io + io);
    const float2 cv = *reinterpret_cast<const float2*>(cum_io + io);
    d[0] = dv.x;
    d[1] = dv.y;
    cum0 = cv.x;
    cum1 = cv.y;
  }
  sCum[2 * tid] = cum0;
  sCum[2 * tid + 1] = cum1;
  __syncthreads();
  {
    const float clast = sCum[255];
    sW[2 * tid] = (2 * tid < ci.lim) ? __expf(fminf(clast - cum0, 0.f)) * d[0] : 0.f;
    sW[2 * tid + 1] = (2 * tid + 1 < ci.lim) ? __expf(fminf(clast - cum1, 0.f)) * d[1] : 0.f;
  }
  __syncthreads();

  const uint32_t idesc = idesc_f16(128, 64, BF16, /*a_mn=*/true, /*b_mn=*/true);
  bool ok = true;
  bool pend_tma = true, pend_mma = false;
  int cur_mma_bar = 2;
  for (int ph = 0; ph < (two_phases ? 2 : 1); ++ph) {
    bool w_ok = mbar_wait_sleep(bar[ph], 0, kSiteStateTma);
    if (w_ok) {
      // x rows scaled by w_l in place (rows past `lim` have w = 0 and become exact zeros).
      for (int q = tid; q < 1024; q += 128) {
        uint4* pch = reinterpret_cast<uint4*>(sX + q * 16);
        const int l = ph * 128 + (q >> 3);
        const float w = sW[l];
        *pch = (w == 0.f) ? make_uint4(0u, 0u, 0u, 0u) : scale8<T16>(*pch, w);
      }
    }
    fence_proxy_async_smem();
    ok = __syncthreads_and(w_ok) != 0;
    if (!ok) break;
    pend_tma = false;
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a0 = smem_u32(sB), b0 = smem_u32(sX);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t ad = sdesc_sw128(a0 + ks * 2048, 16384, 1024);
        const uint64_t bd = sdesc_sw128(b0 + ks * 2048, 16, 1024);
        umma_f16(tmem, ad, bd, idesc, (ph > 0 || ks > 0) ? 1u : 0u);
      }
      umma_commit(bar[2 + ph]);
    }
    pend_mma = true;
    cur_mma_bar = 2 + ph;
    if (ph == 0 && two_phases) {
      // The second phase reuses the buffers: wait for this phase's MMAs first.
      if (tid == 0) {
        if (mbar_wait_sleep(bar[2], 0, kSiteStateMma)) {
          mbar_expect_tx(bar[1], 49152u);
          tma_load_3d(smem_u32(sX), &tm_x, 0, h, t0 + 128, bar[1]);
          tma_load_3d(smem_u32(sB), &tm_b, 0, g, t0 + 128, bar[1]);
          tma_load_3d(smem_u32(sB + 16384), &tm_b, 64, g, t0 + 128, bar[1]);
        }
      }
      pend_tma = true;
    }
  }
  bool mma_ok = false;
  if (ok) mma_ok = mbar_wait_sleep(bar[cur_mma_bar], 0, kSiteStateMma);
  tc_fence_after();
  if (ok && __syncthreads_and(mma_ok)) {
    const int n = warp * 32 + lane;
    float* out = states + ((long long)k * H + h) * (64 * 128);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + half * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) out[(half * 32 + j) * 128 + n] = __uint_as_float(r[j]);
    }
  } else if (tid == 0) {
    // Let in-flight copies / MMAs land (bounded) before the CTA exits.
    if (pend_tma) mbar_wait_sleep(bar[two_phases ? 1 : 0], 0, kSiteStateTma);
    if (pend_mma) mbar_wait_sleep(bar[cur_mma_bar], 0, kSiteStateMma);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

// ===========================================================================
// chunk_state + state_passing: one (row, head pair) chain per CTA
// ===========================================================================
// The CTA walks the row's chunks in order for two heads of one group. Per chunk
// it computes dt / cum (forward_kernel.py:20-105), the chunk states
// S_k = sum_l B_l^T (x_l w_l) of both heads with one N = 128 MMA per 16 tokens
// (:108-200; the B tile is loaded once for the pair) and folds S_k into the
// running states, which live in TMEM in fp32 (:203-258):
//   prev_0 = h_init (or 0),  prev_{k+1} = exp(cum_last_k) prev_k + S_k,  h_last = prev_count.
// prev_k is written in the input's 16-bit type for chunk_scan; the fp32 chunk
// states never reach memory.
// Roles (22 warps):
//   warp 0 (one lane)   TMA producer of 128-token stages (B: two dstate halves, x of
//                       each head) in a kSpStages-deep ring;
//   warp 1 (one lane)   MMA issuer: chunk k accumulates in TMEM columns
//                       [128 (k % 3), +128) (head i at +64 i); three accumulators let
//                       the MMAs run up to three chunks ahead of the fold;
//   warps 2..5          dt, cum and token weights w, up to kSpWBufs chunks ahead:
//                       warp 2 + 2 i + e serves head i on the chunks of parity e (a chunk's
//                       dt does not depend on the previous chunk, so two warps a head
//                       double the rate of this step);
//   warps 6..13         scale the x rows of each stage by w in place (4 warps a head);
//   warps 14..21        fold: prev (TMEM columns [384 + 64 i, +64)) = exp(cum_last) prev
//                       + S_k, then store prev in 16 bits; thread = dstate row n (its
//                       TMEM lane), 4 warps a head.
// Scaling the next chunk overlaps the fold of the previous one. With an odd number
// of heads per group the last CTA has one head; the second head's scale and fold
// warps then only keep the barrier phases.
constexpr int kSpStages = 3;
constexpr int kSpStageBytes = 32768 + 2 * 16384;  // B [128 tokens x 2 halves x 128 B] | x head 0 | x head 1
constexpr int kSpThreads = 704;                    // 22 warps
constexpr int kSpWBufs = 3;
constexpr int kSpAccs = 3;  // chunk-state accumulators in TMEM  // w / exp(cum_last) buffers: the prep warps run up to two chunks ahead
// ring | w [buffer][2 heads][256] | exp(cum_last) [buffer][2] | barriers, TMEM slot, abort flag
constexpr int kSpSmem = kSpStages * kSpStageBytes + kSpWBufs * 2048 + 32 + 256 + 1024;

enum : unsigned int {
  kSiteSpTma = 0x111,
  kSiteSpScaled = 0x112,
  kSiteSpMma = 0x113,
  kSiteSpPrep = 0x114,
  kSiteSpFold = 0x115,
};

template <bool BF16, typename DT>
__global__ void __launch_bounds__(kSpThreads, 1) tc_state_pass_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_b,
    const float* __restrict__ A, const DT* __restrict__ delta_raw, const float* __restrict__ delta_bias,
    float* __restrict__ dt_out, float* __restrict__ cum_out, typename T16Of<BF16>::type* __restrict__ prev16,
    const float* __restrict__ h_init, float* __restrict__ h_last, ChunkMap cm, int H, int hpg, int use_sp,
    float dmin, float dmax) {
  // the chunk_scan launched after this kernel may start its set-up on the free SMs now;
  // it waits for this grid's completion before it reads dt, cum or prev16
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  using T16 = typename T16Of<BF16>::type;
  constexpr int NST = kSpStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  auto sBst = [&](int s) { return smem + s * kSpStageBytes; };
  auto sXst = [&](int s, int i) { return smem + s * kSpStageBytes + 32768 + 16384 * i; };
  constexpr int NW = kSpWBufs;
  float* sW = reinterpret_cast<float*>(smem + NST * kSpStageBytes);  // [buffer][head][256] token weights
  float* sEl = sW + 512 * NW;                                          // [buffer][head] exp(cum_last)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sEl + 8);
  // FULL[NST] SCALED[NST] EMPTY[NST] ACC_FULL[NA] ACC_FREE[NA] W_READY[NW] W_FREE[NW]
  constexpr int NA = kSpAccs;
  constexpr int FULL = 0, SCALED = NST, EMPTY = 2 * NST, ACC_FULL = 3 * NST, ACC_FREE = ACC_FULL + NA,
                W_READY = ACC_FREE + NA, W_FREE = W_READY + NW, NBARS = W_FREE + NW;
  static_assert(NBARS * 8 + 8 <= 256, "barrier area");
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tslot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  constexpr uint32_t T_PREV = 128 * NA;  // running states: TMEM columns [384, 512)
  static_assert(128 * NA + 128 <= 512, "TMEM columns");

  // blockIdx.x -> (row, group, head pair of the group)
  const int npairs = (hpg + 1) >> 1;
  const int G = H / hpg;
  int rem = blockIdx.x;
  const int pair = rem % npairs;
  rem /= npairs;
  const int g = rem % G;
  const int row = rem / G;
  const int h0 = g * hpg + 2 * pair;
  const int nh = min(2, hpg - 2 * pair);
  int first, count;
  if (cm.packed) {
    const int2 r = cm.rows[row];
    first = r.x;
    count = r.y;
  } else {
    first = row * cm.nc;
    count = cm.nc;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_b);
    for (int s = 0; s < NST; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(SCALED + s), 8);
      mbar_init(bar(EMPTY + s), 1);
    }
    for (int b = 0; b < NA; ++b) {
      mbar_init(bar(ACC_FULL + b), 1);
      mbar_init(bar(ACC_FREE + b), 8);
    }
    for (int b = 0; b < NW; ++b) {
      mbar_init(bar(W_READY + b), 2);
      mbar_init(bar(W_FREE + b), 16);  // 8 scale + 8 fold warps
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tslot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  // Warps wait independently; a warp that gives up stops releasing work and raises
  // the abort flag, so the others leave at their next check or bounded wait.
  bool wfail = false;
  auto warp_wait = [&](uint32_t b, uint32_t parity, unsigned int site) {
    if (!wfail) wfail = !__all_sync(0xffffffffu, mbar_wait_sleep(b, parity, site));
    return !wfail;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int r = 0;
      bool fail = false;
      const uint32_t bytes = 32768u + 16384u * (uint32_t)nh;
      for (int k = 0; k < count && !fail && !*s_abort; ++k) {
        ChunkInfo ci;
        chunk_info(cm, first + k, ci);
        const int nst = (ci.lim + 127) >> 7, t0 = (int)ci.tok0;
        for (int s = 0; s < nst; ++s, ++r) {
          const int slot = r % NST;
          if (r >= NST && !mbar_wait_sleep(bar(EMPTY + slot), ((r / NST) - 1) & 1, kSiteSpMma)) {
            fail = true;
            break;
          }
          const uint32_t fb = bar(FULL + slot);
          mbar_expect_tx(fb, bytes);
          tma_load_3d(smem_u32(sBst(slot)), &tm_b, 0, g, t0 + 128 * s, fb);
          tma_load_3d(smem_u32(sBst(slot) + 16384), &tm_b, 64, g, t0 + 128 * s, fb);
          for (int i = 0; i < nh; ++i) tma_load_3d(smem_u32(sXst(slot, i)), &tm_x, 0, h0 + i, t0 + 128 * s, fb);
        }
      }
      if (fail) *s_abort = 1;
      // No copy may still be in flight when the CTA exits.
      for (int d = 1; d <= NST && d <= r; ++d) {
        const int rr = r - d;
        mbar_wait_sleep(bar(FULL + rr % NST), (rr / NST) & 1, kSiteSpTma);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, 64 * nh, BF16, /*a_mn=*/true, /*b_mn=*/true);
      int r = 0, last_bar = -1, last_par = 0;
      bool fail = false;
      for (int k = 0; k < count && !fail && !*s_abort; ++k) {
        ChunkInfo ci;
        chunk_info(cm, first + k, ci);
        const int nst = (ci.lim + 127) >> 7;
        const uint32_t acc = tmem + 128 * (k % NA);
        // the fold of chunk k - 2 must have read this accumulator
        if (k >= NA && !mbar_wait_sleep(bar(ACC_FREE + k % NA), ((k - NA) / NA) & 1, kSiteSpFold)) {
          fail = true;
          break;
        }
        for (int s = 0; s < nst; ++s, ++r) {
          const int slot = r % NST;
          if (!mbar_wait_sleep(bar(SCALED + slot), (r / NST) & 1, kSiteSpScaled)) {
            fail = true;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sBst(slot)), b0 = smem_u32(sXst(slot, 0));
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_f16(acc, sdesc_sw128(a0 + ks * 2048, 16384, 1024), sdesc_sw128(b0 + ks * 2048, 16384, 1024),
                     idesc, (s > 0 || ks > 0) ? 1u : 0u);
          umma_commit(bar(EMPTY + slot));
          last_bar = EMPTY + slot;
          last_par = (r / NST) & 1;
        }
        if (fail) break;
        umma_commit(bar(ACC_FULL + k % NA));
      }
      if (fail) *s_abort = 1;
      // All MMAs must be complete before TMEM is released.
      if (last_bar >= 0) mbar_wait_sleep(bar(last_bar), last_par, kSiteSpMma);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ------------------------------------------------------------ dt / cum / w, ahead of the chain
    // warp 2 + 2 hl + par serves head hl on chunks par, par + 2, ...; lane: tokens
    // [8 lane, 8 lane + 8) of the chunk. Raw dt is loaded two chunks (of this warp)
    // ahead, in two register sets used in turn, so the latency of these strided loads
    // stays off the chain.
    const int hl = (warp - 2) >> 1, par = (warp - 2) & 1, tb = 8 * lane;
    const bool act = hl < nh;
    const int h = h0 + (act ? hl : 0);
    const float a = A[h];
    const float bias = delta_bias ? delta_bias[h] : 0.f;
    auto load_raw = [&](int k, float (&rv)[8]) {
#pragma unroll
      for (int e = 0; e < 8; ++e) rv[e] = 0.f;
      if (k >= count || !act) return;
      ChunkInfo ci;
      chunk_info(cm, first + k, ci);
      const DT* dr = delta_raw + (ci.tok0 + tb) * (long long)H + h;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (tb + e < ci.vlim) rv[e] = Ld<DT>::f(dr + (long long)e * H);
    };
    // One chunk: dt / cum to global memory, w / exp(cum_last) into buffer k % NW.
    auto prep = [&](int k, float (&raw)[8]) -> bool {
      const int buf = k % NW;
      ChunkInfo ci;
      chunk_info(cm, first + k, ci);
      float d[8], c[8];
      float run = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        d[e] = (act && tb + e < ci.vlim) ? dt_transform(raw[e] + bias, use_sp, dmin, dmax) : 0.f;
        run += d[e] * a;
        c[e] = run;
      }
      load_raw(k + 4, raw);
      float incl = run;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const float base = incl - run;
      const float cl = __shfl_sync(0xffffffffu, incl, 31);
      if (k >= NW && !warp_wait(bar(W_FREE + buf), ((k - NW) / NW) & 1, kSiteSpPrep)) return false;
      if (act) {
        const long long io = ((first + k) * (long long)H + h) * 256 + tb;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          *reinterpret_cast<float4*>(dt_out + io + 4 * q) =
              make_float4(d[4 * q], d[4 * q + 1], d[4 * q + 2], d[4 * q + 3]);
          *reinterpret_cast<float4*>(cum_out + io + 4 * q) =
              make_float4(base + c[4 * q], base + c[4 * q + 1], base + c[4 * q + 2], base + c[4 * q + 3]);
        }
        float* w = sW + 512 * buf + 256 * hl + tb;
        float wv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) wv[e] = tb + e < ci.lim ? __expf(fminf(cl - (base + c[e]), 0.f)) * d[e] : 0.f;
        reinterpret_cast<float4*>(w)[0] = make_float4(wv[0], wv[1], wv[2], wv[3]);
        reinterpret_cast<float4*>(w)[1] = make_float4(wv[4], wv[5], wv[6], wv[7]);
        if (lane == 0) sEl[2 * buf + hl] = expf(cl);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(W_READY + buf));
      return true;
    };
    float rawA[8], rawB[8];
    load_raw(par, rawA);
    load_raw(par + 2, rawB);
    for (int k = par; k < count && !*s_abort; k += 4) {
      if (!prep(k, rawA) || (k + 2 < count && !prep(k + 2, rawB))) break;
    }
    if (wfail) *s_abort = 1;
  } else if (warp < 14) {
    // ------------------------------------------------------------ scale x by w (in place)
    const int hg = (warp - 6) >> 2, cw = (warp - 6) & 3;
    const bool active = hg < nh;
    int r = 0;
    for (int k = 0; k < count && !wfail && !*s_abort; ++k) {
      ChunkInfo ci;
      chunk_info(cm, first + k, ci);
      const int nst = (ci.lim + 127) >> 7, buf = k % NW;
      if (!warp_wait(bar(W_READY + buf), (k / NW) & 1, kSiteSpPrep)) break;
      const float* wh = sW + 512 * buf + 256 * hg;
      // rows past `lim` become exact zeros (their w is 0)
      for (int s = 0; s < nst; ++s, ++r) {
        const int slot = r % NST;
        if (!warp_wait(bar(FULL + slot), (r / NST) & 1, kSiteSpTma)) break;
        if (active) {
          uint4* sx = reinterpret_cast<uint4*>(sXst(slot, hg)) + cw * 32 + lane;
          // All loads first: stores through the same shared-memory pointers would
          // otherwise order each chunk's load behind the previous chunk's store.
          uint4 xv[8];
          float wv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            xv[i] = sx[128 * i];
            wv[i] = wh[128 * s + ((cw * 32 + lane + 128 * i) >> 3)];
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            uint4 o4;
            if constexpr (BF16) {
              const __nv_bfloat162 w2 = __float2bfloat162_rn(wv[i]);
              o4 = scale8_packed<T16>(xv[i], *reinterpret_cast<const uint32_t*>(&w2));
            } else {
              o4 = scale8<T16>(xv[i], wv[i]);
            }
            sx[128 * i] = (wv[i] == 0.f) ? make_uint4(0u, 0u, 0u, 0u) : o4;
          }
          fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(SCALED + slot));
      }
      if (wfail) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(W_FREE + buf));  // w of chunk k no longer read
    }
    if (wfail) *s_abort = 1;
  } else {
    // ------------------------------------------------------------ fold into the running states
    const int hg = (warp - 14) >> 2;  // head of the pair
    const bool active = hg < nh;
    const int quad = warp & 3, n = quad * 32 + lane;
    const uint32_t tlane = (uint32_t)(quad * 32) << 16;
    const uint32_t tprev = tmem + tlane + T_PREV + 64 * hg;
    const int h = h0 + (active ? hg : 0);
    const long long PN = 64 * 128;
    const int li = lane & 7, rbase = quad * 32 + (lane & ~7);
    // prev16 row n of a chunk = 64 contiguous p values (128 bytes), transposed across
    // each group of 8 lanes so that every store instruction writes four whole rows.
    auto store_prev16 = [&](uint4 (&d)[8], T16* chunk_base) {
      lane_transpose<8>(d, li);
      uint4* d4 = reinterpret_cast<uint4*>(chunk_base) + rbase * 8 + li;
#pragma unroll
      for (int j = 0; j < 8; ++j) d4[8 * j] = d[j];
    };
    auto pack8 = [&](const uint32_t (&v)[16], int off) {
      return make_uint4(pack2<T16>(__uint_as_float(v[off]), __uint_as_float(v[off + 1])),
                        pack2<T16>(__uint_as_float(v[off + 2]), __uint_as_float(v[off + 3])),
                        pack2<T16>(__uint_as_float(v[off + 4]), __uint_as_float(v[off + 5])),
                        pack2<T16>(__uint_as_float(v[off + 6]), __uint_as_float(v[off + 7])));
    };
    // prev_0 = h_init (or 0) into TMEM and, as 16 bits, for the first chunk.
    if (active) {
      const float* hi = h_init ? h_init + ((long long)row * H + h) * PN + n : nullptr;
      uint4 d[8];
#pragma unroll
      for (int qt = 0; qt < 4; ++qt) {
        uint32_t v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(hi ? hi[(16 * qt + i) * 128] : 0.f);
        if (count == 0) {
          float* dst = h_last + ((long long)row * H + h) * PN + n;
#pragma unroll
          for (int i = 0; i < 16; ++i) dst[(16 * qt + i) * 128] = __uint_as_float(v[i]);
        } else {
          tmem_st16(tprev + 16 * qt, v);
          d[2 * qt] = pack8(v, 0);
          d[2 * qt + 1] = pack8(v, 8);
        }
      }
      if (count > 0) {
        tmem_wait_st();
        store_prev16(d, prev16 + ((long long)first * H + h) * PN);
      }
    }
    for (int j = 0; j < count && !*s_abort; ++j) {
      const int buf = j % NW;
      if (!warp_wait(bar(ACC_FULL + j % NA), (j / NA) & 1, kSiteSpMma) ||
          !warp_wait(bar(W_READY + buf), (j / NW) & 1, kSiteSpPrep))
        break;
      tc_fence_after();
      const float el = sEl[2 * buf + hg];
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(W_FREE + buf));  // exp(cum_last) of chunk j read
      const bool last = j + 1 == count;
      uint4 d[8];
      if (active) {
        const uint32_t acc = tmem + tlane + 128 * (j % NA) + 64 * hg;
        float* dst = h_last + ((long long)row * H + h) * PN + n;
#pragma unroll
        for (int qt = 0; qt < 4; ++qt) {
          uint32_t a[16], pv[16];
          tmem_ld16(acc + 16 * qt, a);
          tmem_ld16(tprev + 16 * qt, pv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i)
            a[i] = __float_as_uint(fmaf(el, __uint_as_float(pv[i]), __uint_as_float(a[i])));
          if (last) {
#pragma unroll
            for (int i = 0; i < 16; ++i) dst[(16 * qt + i) * 128] = __uint_as_float(a[i]);
          } else {
            tmem_st16(tprev + 16 * qt, a);
            d[2 * qt] = pack8(a, 0);
            d[2 * qt + 1] = pack8(a, 8);
          }
        }
      }
      // this chunk's accumulator is read: MMA(j + kSpAccs) may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(ACC_FREE + j % NA));
      if (active && !last) {
        tmem_wait_st();
        store_prev16(d, prev16 + ((long long)(first + j + 1) * H + h) * PN);
      }
    }
    if (wfail) *s_abort = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ===========================================================================
// chunk_scan (+ bmm_chunk): persistent, warp-specialised, CB shared across heads
// ===========================================================================
// Work items are (chunk k, half m, group g, block of up to HB heads of the group).
// Per item, C rows of the half and B rows [0, 128(m+1)) are loaded once,
// CB_j = C B_j^T (j = 0..m, 128 source tokens each) is computed once into TMEM
// and rounded there to the input's 16-bit type; then, head by head, only x, prev,
// z, dt and cum are loaded (the epilogue reads D from global memory).
// The decay is factored per 32-row block R (rows [32R, 32R+32) of the chunk):
//   exp(cum_l - cum_s) = exp(cum_l - cum_{32R}) * exp(cum_{32R} - cum_s)
// Both factors are <= 1 for s < 32R when cum is non-increasing (A <= 0, dt >= 0);
// inside the diagonal 32x32 tile the second one is bounded by the tile's own decay,
// which must stay below kScanFacMaxDecay. For such "factored" row blocks
//   M'_j[l, s] = CB_j[l, s] * g_R[s],  g_R[s] = exp(cum_{32R} - cum_s) dt_s  (s <= l)
// is one packed 16-bit multiply per pair of elements, and the row factor
// exp(cum_l - cum_{32R}) is applied to Yin in the epilogue. Other row blocks get the
// exact M_j[l, s] = CB_j[l, s] exp(min(cum_l - cum_s, 0)) dt_s and row factor 1.
//   Yin  += M'_j x_j   (A from TMEM)    Yoff = C prev     (per head)
//   y = exp(cum_l) Yoff + rowf_l Yin (+ D x) (* silu z)
// Roles (one CTA per SM, items blockIdx.x, blockIdx.x + gridDim.x, ...):
//   warp 0 (one lane)  TMA producer: C per item, B one 128-token block at a time,
//                      head stages (x, prev, dt, cum) in a 3-deep ring; z of a
//                      first-half head comes with them (into the x rows [128, 256)
//                      that half does not use), z of a second-half head goes into its
//                      stage's prev tile once MMA3 has read prev;
//   warp 1 (one lane)  MMA issuer;
//   warps 2..9         conversion: CB_j landing (fp32) -> 16 bits per item, then per
//                      head the g table and CB_j -> M'_j (warp: two 32-column blocks
//                      of a 32-row quadrant);
//   warps 10..17       epilogue of the previous head (32 output columns per warp),
//                      so conversion of head i+1 overlaps the epilogue of head i.
// TMEM columns: 16-bit CB_0 [0,64) CB_1 [64,128); Y buffer 1 (Yin, Yoff) [128,256),
//               also MMA1's fp32 landing zone at an item's start; M buffers [256,320)
//               [320,384); Y buffer 0 [384,512). Heads alternate Y buffers.
// The epilogue warps copy a head's x, z and cum rows into registers first and release
// the stage; the stage is reloaded once that release and the head's MMAs are done.
// Barriers that a role may lag behind are kept per ring slot, so a waiter is never
// two phases behind the barrier it polls. Every wait is bounded; a role that gives
// up records the site, raises the CTA's abort flag and leaves its loop.
constexpr int kScanHeadStageBytes = 32768 + 16384;  // x rows [0, 256) (m = 0: [0, 128) | z) | prev (m = 1: later z)
constexpr int kScanStages = 3;                       // head stages in flight
constexpr int kScanSmallBytes = 4224;  // words: dt [0,256) cum [256,512) flags [512,516) g [520,1032)
constexpr int kScanThreads = 576;      // warp 0 TMA, warp 1 MMA, warps 2..9 conversion, 10..17 epilogue
constexpr int kScanMaxHeads = 1024;    // A[0:H) staged in shared memory
// C 32 KB | B (one 128-token block) 32 KB | head stages | small stages | barriers | A
constexpr int kScanSmallOff = 65536 + kScanStages * kScanHeadStageBytes;
constexpr int kScanBarOff = kScanSmallOff + kScanStages * kScanSmallBytes;
constexpr int kScanSmem = kScanBarOff + 256 + 4 * kScanMaxHeads + 1024;
// Largest decay inside a diagonal 32x32 tile for which the factored form is used:
// g_R reaches exp(decay) * dt, which must fit the 16-bit type with a wide margin.
__device__ __forceinline__ float scan_fac_max_decay(bool bf16) { return bf16 ? 60.f : 8.f; }

struct ScanItem {
  int k, m, g, h0, nh;  // chunk, half, group, first head, heads in the block
};

// Item `it` -> ScanItem; false if the half holds no token of the row.
__device__ __forceinline__ bool scan_item(const ChunkMap& cm, int it, int G, int hpg, int HB, ScanItem& si,
                                          ChunkInfo& ci) {
  const int nhb = (hpg + HB - 1) / HB;
  int rem = it;
  const int hbi = rem % nhb;
  rem /= nhb;
  si.g = rem % G;
  rem /= G;
  si.m = 1 - (rem & 1);  // the heavier half of a chunk first
  si.k = rem >> 1;
  si.h0 = si.g * hpg + hbi * HB;
  si.nh = min(HB, hpg - hbi * HB);
  if (!chunk_info(cm, si.k, ci)) return false;
  return 128 * si.m < ci.lim;
}

// The j-th item of CTA b: rows of gridDim.x items taken in snake order (b, then
// 2 grid - 1 - b, ...). Items alternate a chunk's heavier second half and its first
// half, so a plain grid stride with an even grid would hand every CTA the same kind.
__device__ __forceinline__ int scan_item_of(int j) {
  const int b = (j & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x;
  return j * (int)gridDim.x + b;
}

template <bool BF16, typename YT>
__global__ void __launch_bounds__(kScanThreads, 1) tc_chunk_scan_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_c,
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_h,
    const __grid_constant__ CUtensorMap tm_z, const float* __restrict__ A, const float* __restrict__ dt,
    const float* __restrict__ cum, const float* __restrict__ D, int has_z, YT* __restrict__ y, ChunkMap cm, int H,
    int G, int HB, int dt_nonneg, int n_items) {
  using T16 = typename T16Of<BF16>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  constexpr int NS = kScanStages;
  uint8_t* sC = smem;           // 2 x (128 rows x 128 B): dstate halves of the half's C rows
  uint8_t* sB = smem + 32768;   // B rows of one 128-token block j: 2 x (128 rows x 128 B)
  // head stage: x rows [0, 256) | prev, then the z rows of the half once MMA3 has read prev
  auto hstage = [&](int s) { return smem + 65536 + s * kScanHeadStageBytes; };
  auto small = [&](int s) { return reinterpret_cast<float*>(smem + kScanSmallOff + s * kScanSmallBytes); };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kScanBarOff);
  // per stage (NS each): HEAD_FULL, STAGE_FREE, STAGE_MMA, YOFF, Z_FULL
  enum {
    ITEM_FULL = 0, BJ_FULL, B_FREE, C_FREE, CBS_FULL, CBS_FREE, MFULL0, MFULL1, M2DONE0, M2DONE1, YFULL0, YFULL1,
    YFREE0, YFREE1, HEAD_FULL0, STAGE_FREE0 = HEAD_FULL0 + NS, STAGE_MMA0 = STAGE_FREE0 + NS,
    YOFF0 = STAGE_MMA0 + NS, Z_FULL0 = YOFF0 + NS, NBARS = Z_FULL0 + NS
  };
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tslot + 1);
  float* sA = reinterpret_cast<float*>(smem + kScanBarOff + 256);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int hpg = H / G;
  // TMEM: 16-bit CB_0 [0,64) CB_1 [64,128); Y buffer 1 [128,256) (Yin, Yoff), also the
  // fp32 landing zone of MMA1 at an item's start; M buffers [256,320) [320,384);
  // Y buffer 0 [384,512).
  const uint32_t T_SCR = 128, T_M = 256;
  auto t_yin = [&](int yb) { return yb ? 128u : 384u; };
  auto t_yoff = [&](int yb) { return yb ? 192u : 448u; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_c);
    prefetch_tmap(&tm_b);
    prefetch_tmap(&tm_h);
    if (has_z) prefetch_tmap(&tm_z);
    mbar_init(bar(ITEM_FULL), 1);
    mbar_init(bar(BJ_FULL), 1);
    mbar_init(bar(B_FREE), 1);
    mbar_init(bar(C_FREE), 1);
    mbar_init(bar(CBS_FULL), 1);
    mbar_init(bar(CBS_FREE), 8);
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(HEAD_FULL0 + s), 1);
      mbar_init(bar(STAGE_FREE0 + s), 8);
      mbar_init(bar(STAGE_MMA0 + s), 1);
      mbar_init(bar(YOFF0 + s), 1);
      mbar_init(bar(Z_FULL0 + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(MFULL0 + s), 8);
      mbar_init(bar(M2DONE0 + s), 1);
      mbar_init(bar(YFULL0 + s), 1);
      mbar_init(bar(YFREE0 + s), 8);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  for (int i = tid; i < H; i += kScanThreads) sA[i] = A[i];
  if (warp == 1) tmem_alloc(smem_u32(tslot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int I = 0, Hc = 0, zc = 0, Bc = 0, Bj = 0;  // items, heads, z phases started, MMA1 jobs, B_1 landings
      bool fail = false;
      int zpend = -1, zh = 0, zt = 0;  // head counter, head and first token of a pending z load
      // z rows of a second-half head go into its stage's prev tile once its MMA3 has
      // read prev. (A first-half head's z comes with its main loads, into the x rows
      // [128, 256) that the first half does not use.)
      auto load_z = [&]() -> bool {
        const int s = zpend % NS;
        if (!mbar_wait_sleep(bar(YOFF0 + s), (zpend / NS) & 1, kSiteScanMma2)) return false;
        mbar_expect_tx(bar(Z_FULL0 + s), 16384u);
        tma_load_3d(smem_u32(hstage(s) + 32768), &tm_z, 0, zh, zt, bar(Z_FULL0 + s));
        ++zc;
        zpend = -1;
        return true;
      };
      for (int jt = 0, it = scan_item_of(0); it < n_items && !fail && !*s_abort; it = scan_item_of(++jt)) {
        ScanItem si;
        ChunkInfo ci;
        if (!scan_item(cm, it, G, hpg, HB, si, ci)) continue;
        const int t0 = (int)ci.tok0, S = 128 * (si.m + 1);
        // C free once the previous item's last MMA3 completed; the B buffer once the
        // previous MMA1 did.
        if ((I > 0 && !mbar_wait_sleep(bar(C_FREE), (I - 1) & 1, kSiteScanMma1)) ||
            (Bc > 0 && !mbar_wait_sleep(bar(B_FREE), (Bc - 1) & 1, kSiteScanMma1))) {
          fail = true;
          break;
        }
        mbar_expect_tx(bar(ITEM_FULL), 65536u);
        tma_load_3d(smem_u32(sC), &tm_c, 0, si.g, t0 + 128 * si.m, bar(ITEM_FULL));
        tma_load_3d(smem_u32(sC + 16384), &tm_c, 64, si.g, t0 + 128 * si.m, bar(ITEM_FULL));
        tma_load_3d(smem_u32(sB), &tm_b, 0, si.g, t0, bar(ITEM_FULL));
        tma_load_3d(smem_u32(sB + 16384), &tm_b, 64, si.g, t0, bar(ITEM_FULL));
        ++Bc;
        // dt, cum and prev16 come from the state pass, which may still be running when
        // this kernel starts (programmatic dependent launch): this thread alone reads
        // them, so it alone waits for that grid's completion and its writes
        if (I == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int i = 0; i < si.nh; ++i) {
          const int h = si.h0 + i, hs = Hc % NS;
          // The stage is free once the epilogue of the head NS back copied what it
          // needs and that head's MMAs completed.
          if (Hc >= NS && (!mbar_wait_sleep(bar(STAGE_FREE0 + hs), ((Hc - NS) / NS) & 1, kSiteScanEpi) ||
                           !mbar_wait_sleep(bar(STAGE_MMA0 + hs), ((Hc - NS) / NS) & 1, kSiteScanMma2))) {
            fail = true;
            break;
          }
          uint8_t* st = hstage(hs);
          float* sm = small(hs);
          const uint32_t fb = bar(HEAD_FULL0 + hs);
          const bool z_now = has_z && si.m == 0;
          mbar_expect_tx(fb, (uint32_t)S * 128u + 16384u + 2048u + (z_now ? 16384u : 0u));
          for (int j = 0; j <= si.m; ++j) tma_load_3d(smem_u32(st + 16384 * j), &tm_x, 0, h, t0 + 128 * j, fb);
          tma_load_3d(smem_u32(st + 32768), &tm_h, 0, 0, si.k * H + h, fb);
          bulk_load(smem_u32(sm), dt + ((long long)si.k * H + h) * 256, 1024u, fb);
          bulk_load(smem_u32(sm + 256), cum + ((long long)si.k * H + h) * 256, 1024u, fb);
          if (z_now) tma_load_3d(smem_u32(st + 16384), &tm_z, 0, h, t0, fb);
          // z of the previous head first: MMA1 of this item may wait for that head's
          // epilogue, which needs its z, before B's block 1 can be loaded.
          if (zpend >= 0 && !load_z()) {
            fail = true;
            break;
          }
          if (z_now) {
            // the z tile arrives with HEAD_FULL; complete this head's Z_FULL phase
            mbar_arrive(bar(Z_FULL0 + hs));
            ++zc;
          } else if (has_z) {
            zpend = Hc;
            zh = h;
            zt = t0 + 128;
          }
          if (i == 0 && si.m == 1) {
            // B rows of block 1 once MMA1 of block 0 has read the buffer
            if (!mbar_wait_sleep(bar(B_FREE), (Bc - 1) & 1, kSiteScanMma1)) {
              fail = true;
              break;
            }
            mbar_expect_tx(bar(BJ_FULL), 32768u);
            tma_load_3d(smem_u32(sB), &tm_b, 0, si.g, t0 + 128, bar(BJ_FULL));
            tma_load_3d(smem_u32(sB + 16384), &tm_b, 64, si.g, t0 + 128, bar(BJ_FULL));
            ++Bc;
            ++Bj;
          }
          ++Hc;
        }
        ++I;
      }
      if (!fail && !*s_abort && zpend >= 0 && !load_z()) fail = true;
      if (fail) *s_abort = 1;
      // No copy may still be in flight when the CTA exits.
      if (I > 0) mbar_wait_sleep(bar(ITEM_FULL), (I - 1) & 1, kSiteScanTma);
      if (Bj > 0) mbar_wait_sleep(bar(BJ_FULL), (Bj - 1) & 1, kSiteScanTma);
      for (int d = 1; d <= NS && d <= Hc; ++d) {
        const int hc = Hc - d;
        mbar_wait_sleep(bar(HEAD_FULL0 + hc % NS), (hc / NS) & 1, kSiteScanTma);
      }
      for (int d = 1; d <= NS && d <= zc; ++d) {
        const int hc = zc - d;
        mbar_wait_sleep(bar(Z_FULL0 + hc % NS), (hc / NS) & 1, kSiteScanTma);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_cb = idesc_f16(128, 128, BF16, false, false);
      const uint32_t id_off = idesc_f16(128, 64, BF16, false, /*b_mn=*/true);
      const uint32_t id_in = idesc_f16(128, 64, BF16, false, true);
      int I = 0, Hc = 0, Jc = 0, Sc = 0, Bj = 0;  // items, heads, M-buffer jobs, CB landings, B_1 landings
      bool fail = false;
      int last_bar = -1, last_par = 0;
      for (int jt = 0, it = scan_item_of(0); it < n_items && !fail && !*s_abort; it = scan_item_of(++jt)) {
        ScanItem si;
        ChunkInfo ci;
        if (!scan_item(cm, it, G, hpg, HB, si, ci)) continue;
        if (!mbar_wait_sleep(bar(ITEM_FULL), I & 1, kSiteScanTma)) {
          fail = true;
          break;
        }
        const uint32_t c0 = smem_u32(sC);
        for (int j = 0; j <= si.m && !fail; ++j) {
          // The landing zone is Y buffer 1: free once the epilogue of the last head
          // that used it loaded it, and once the previous CB_j landing was converted.
          const int y1 = Hc / 2;  // heads so far that used Y buffer 1 (odd head counters)
          if ((y1 > 0 && !mbar_wait_sleep(bar(YFREE1), (y1 - 1) & 1, kSiteScanEpi)) ||
              (Sc > 0 && !mbar_wait_sleep(bar(CBS_FREE), (Sc - 1) & 1, kSiteScanConv)) ||
              (j == 1 && !mbar_wait_sleep(bar(BJ_FULL), Bj & 1, kSiteScanTma))) {
            fail = true;
            break;
          }
          if (j == 1) ++Bj;
          tc_fence_after();
          const uint32_t b0 = smem_u32(sB);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t hf = ks >> 2, kk = (ks & 3) * 32;
            umma_f16(tmem + T_SCR, sdesc_sw128(c0 + hf * 16384 + kk, 16, 1024),
                     sdesc_sw128(b0 + hf * 16384 + kk, 16, 1024), id_cb, ks > 0 ? 1u : 0u);
          }
          umma_commit(bar(CBS_FULL));
          umma_commit(bar(B_FREE));
          ++Sc;
        }
        if (fail) break;
        // Head MMAs may write Y buffer 1 only after the last landing was converted.
        if (!mbar_wait_sleep(bar(CBS_FREE), (Sc - 1) & 1, kSiteScanConv)) {
          fail = true;
          break;
        }
        for (int i = 0; i < si.nh && !fail; ++i) {
          const int hs = Hc % NS, yb = Hc & 1;
          if (!mbar_wait_sleep(bar(HEAD_FULL0 + hs), (Hc / NS) & 1, kSiteScanTma) ||
              (Hc >= 2 && !mbar_wait_sleep(bar(YFREE0 + yb), ((Hc - 2) >> 1) & 1, kSiteScanEpi))) {
            fail = true;
            break;
          }
          tc_fence_after();
          const uint32_t h0 = smem_u32(hstage(hs) + 32768), x0 = smem_u32(hstage(hs));
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t hf = ks >> 2, kk = (ks & 3) * 32;
            umma_f16(tmem + t_yoff(yb), sdesc_sw128(c0 + hf * 16384 + kk, 16, 1024),
                     sdesc_sw128(h0 + ks * 2048, 16, 1024), id_off, ks > 0 ? 1u : 0u);
          }
          umma_commit(bar(YOFF0 + hs));
          if (i == si.nh - 1) umma_commit(bar(C_FREE));
          for (int j = 0; j <= si.m; ++j) {
            const int mb = Jc & 1;
            if (!mbar_wait_sleep(bar(MFULL0 + mb), (Jc >> 1) & 1, kSiteScanConv)) {
              fail = true;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              umma_f16_ts(tmem + t_yin(yb), tmem + T_M + 64 * mb + 8 * ks,
                          sdesc_sw128(x0 + 16384 * j + ks * 2048, 16, 1024), id_in, (j > 0 || ks > 0) ? 1u : 0u);
            umma_commit(bar(M2DONE0 + mb));
            ++Jc;
          }
          if (fail) break;
          umma_commit(bar(YFULL0 + yb));
          umma_commit(bar(STAGE_MMA0 + hs));
          last_bar = STAGE_MMA0 + hs;
          last_par = (Hc / NS) & 1;
          ++Hc;
        }
        ++I;
      }
      if (fail) *s_abort = 1;
      // All MMAs must be complete before TMEM is released.
      if (last_bar >= 0) mbar_wait_sleep(bar(last_bar), last_par, kSiteScanMma2);
      else if (Sc > 0) mbar_wait_sleep(bar(CBS_FULL), (Sc - 1) & 1, kSiteScanMma1);
    }
    __syncwarp();
  } else if (warp < 10) {
    // ------------------------------------------------------------ conversion warps (2..9)
    // warp (quad, cc): rows of TMEM quadrant quad, column blocks cg = 2 cc, 2 cc + 1 (32 each)
    const int ct = tid - 64;  // 0..255
    const int quad = warp & 3, cc = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const uint32_t tlane = (uint32_t)(quad * 32) << 16;
    const float fac_max = scan_fac_max_decay(BF16);
    int I = 0, Hc = 0, Jc = 0, Sc = 0;
    bool fail = false, wfail = false;
    auto warp_wait = [&](uint32_t b, uint32_t parity, unsigned int site) {
      if (!wfail) wfail = !__all_sync(0xffffffffu, mbar_wait_sleep(b, parity, site));
      return !wfail;
    };
    for (int jt = 0, it = scan_item_of(0); it < n_items && !fail; it = scan_item_of(++jt)) {
      ScanItem si;
      ChunkInfo ci;
      if (!scan_item(cm, it, G, hpg, HB, si, ci)) continue;
      const int m = si.m, l = 128 * m + r, R = 4 * m + quad, S = 128 * (m + 1);
      // ---- CB_j (fp32, landing zone) -> 16-bit CB_j at [64 j, 64 j + 64) ----
      for (int j = 0; j <= m; ++j, ++Sc) {
        warp_wait(bar(CBS_FULL), Sc & 1, kSiteScanMma1);
        tc_fence_after();
        if (wfail) continue;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int cg = 2 * cc + t;
          uint32_t v[32], hv[16];
          tmem_ld32(tmem + tlane + T_SCR + 32 * cg, v);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 16; ++q) hv[q] = pack2<T16>(__uint_as_float(v[2 * q]), __uint_as_float(v[2 * q + 1]));
          tmem_st16(tmem + tlane + 64 * j + 16 * cg, hv);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(CBS_FREE));
      }
      for (int i = 0; i < si.nh; ++i) {
        const int h = si.h0 + i, hs = Hc % NS;
        uint8_t* sX = hstage(hs);
        float* sm = small(hs);
        const float* sDt = sm;
        const float* sCum = sm + 256;
        int* sFlag = reinterpret_cast<int*>(sm + 512);
        uint32_t* sG = reinterpret_cast<uint32_t*>(sm + 520);  // [row block of the half][pair of s]
        warp_wait(bar(HEAD_FULL0 + hs), (Hc / NS) & 1, kSiteScanTma);
        const bool mono = dt_nonneg && (sA[h] <= 0.f);
        if (!wfail) {
          // The two warps of a quadrant compute the g pairs of their own row block R
          // and meet at a barrier of their own, so the quadrants run decoupled.
          const int tq = cc * 32 + lane;
          const float cr = sCum[32 * R];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int pidx = tq + 64 * e, s2 = 2 * pidx;
            uint32_t gv = 0u;
            if (mono && s2 < 32 * (R + 1)) {
              const float g0 = s2 < ci.lim ? __expf(cr - sCum[s2]) * sDt[s2] : 0.f;
              const float g1 = s2 + 1 < ci.lim ? __expf(cr - sCum[s2 + 1]) * sDt[s2 + 1] : 0.f;
              gv = pack2<T16>(g0, g1);
            }
            sG[quad * 128 + pidx] = gv;
          }
          if (tq == 0) sFlag[quad] = mono && (cr - sCum[32 * R + 31] <= fac_max);
          if (S > ci.lim) {
            // x rows past `lim` -> exact zeros, so they cannot leak into Yin
            for (int q = ct; q < S * 8; q += 256)
              if ((q >> 3) >= ci.lim) *reinterpret_cast<uint4*>(sX + q * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        // publishes this quadrant's g pairs and flag
        if (!named_bar_and(2 + quad, 64, !wfail && !*s_abort)) { fail = true; break; }
        const float cl = sCum[l];
        const bool fR = sFlag[quad] != 0;
        for (int j = 0; j <= m; ++j) {
          const int mb = Jc & 1;
          if (Jc >= 2) {
            warp_wait(bar(M2DONE0 + mb), ((Jc - 2) >> 1) & 1, kSiteScanMma2);
            tc_fence_after();
          }
          if (wfail) {
            ++Jc;
            continue;
          }
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int cg = 2 * cc + t;
            // ---- 16-bit CB_j block cg, rows of this quadrant -> M'_j (TMEM) ----
            const int s0 = 128 * j + cg * 32;
            uint32_t pk[16];
            if (s0 > 32 * R + 31) {
#pragma unroll
              for (int q = 0; q < 16; ++q) pk[q] = 0u;
            } else {
              uint4 g4v[4];
              if (fR) {
                const uint4* gp = reinterpret_cast<const uint4*>(sG + quad * 128 + (s0 >> 1));
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) g4v[q4] = gp[q4];
              }
              uint32_t cb[16];
              tmem_ld16(tmem + tlane + 64 * j + 16 * cg, cb);
              tmem_wait_ld();
              if (fR) {
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                  const uint4 g4 = g4v[q4];
                  pk[4 * q4] = mul2<T16>(cb[4 * q4], g4.x);
                  pk[4 * q4 + 1] = mul2<T16>(cb[4 * q4 + 1], g4.y);
                  pk[4 * q4 + 2] = mul2<T16>(cb[4 * q4 + 2], g4.z);
                  pk[4 * q4 + 3] = mul2<T16>(cb[4 * q4 + 3], g4.w);
                }
                if (s0 == 32 * R) {
                  // diagonal tile: column c of the tile is kept when c <= lane
#pragma unroll
                  for (int q = 0; q < 16; ++q) {
                    const uint32_t keep = (2 * q + 1 <= lane) ? 0xffffffffu : ((2 * q <= lane) ? 0x0000ffffu : 0u);
                    pk[q] &= keep;
                  }
                }
              } else {
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                  const float2 c2 = unpack2<T16>(cb[q]);
                  const int sa = s0 + 2 * q, sb2 = sa + 1;
                  float x0 = 0.f, x1 = 0.f;
                  if (sa <= l && sa < ci.lim) x0 = c2.x * __expf(fminf(cl - sCum[sa], 0.f)) * sDt[sa];
                  if (sb2 <= l && sb2 < ci.lim) x1 = c2.y * __expf(fminf(cl - sCum[sb2], 0.f)) * sDt[sb2];
                  pk[q] = pack2<T16>(x0, x1);
                }
              }
            }
            tmem_st16(tmem + tlane + T_M + 64 * mb + 16 * cg, pk);
          }
          tmem_wait_st();
          fence_proxy_async_smem();  // sX zero-fill (first job) visible to MMA2
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(MFULL0 + mb));
          ++Jc;
        }
        ++Hc;
      }
      ++I;
    }
    if (fail || wfail) *s_abort = 1;
  } else {
    // ------------------------------------------------------------ epilogue warps (10..17)
    // warp (quad, ce): rows of TMEM quadrant quad, output columns [32 ce, 32 ce + 32).
    // y = (exp(cum_l) Yoff + rowf_l Yin + D x) * silu(z)
    const int quad = warp & 3, ce = (warp - 10) >> 2;
    const int r = quad * 32 + lane;
    const uint32_t tlane = (uint32_t)(quad * 32) << 16;
    const float fac_max = scan_fac_max_decay(BF16);
    int Hc = 0;
    bool fail = false, wfail = false;
    auto warp_wait = [&](uint32_t b, uint32_t parity, unsigned int site) {
      if (!wfail) wfail = !__all_sync(0xffffffffu, mbar_wait_sleep(b, parity, site));
      return !wfail;
    };
    for (int jt = 0, it = scan_item_of(0); it < n_items && !fail; it = scan_item_of(++jt)) {
      ScanItem si;
      ChunkInfo ci;
      if (!scan_item(cm, it, G, hpg, HB, si, ci)) continue;
      const int m = si.m, l = 128 * m + r, R = 4 * m + quad;
      for (int i = 0; i < si.nh; ++i, ++Hc) {
        const int h = si.h0 + i, hs = Hc % NS, yb = Hc & 1;
        const uint8_t* sX = hstage(hs);
        const float* sCum = small(hs) + 256;
        // Copy what this epilogue reads from the head stage, then release the stage.
        warp_wait(bar(HEAD_FULL0 + hs), (Hc / NS) & 1, kSiteScanTma);
        if (has_z) warp_wait(bar(Z_FULL0 + hs), (Hc / NS) & 1, kSiteScanTma);
        uint4 xv[4], zv[4];
        float cl = 0.f, rowf = 1.f;
        if (!wfail) {
          const bool mono = dt_nonneg && (sA[h] <= 0.f);
          cl = sCum[l];
          const bool fR = mono && (sCum[32 * R] - sCum[32 * R + 31] <= fac_max);
          rowf = fR ? __expf(cl - sCum[32 * R]) : 1.f;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            xv[q] = *reinterpret_cast<const uint4*>(sX + 16384 * m + sw128_off(r, 4 * ce + q));
            zv[q] = has_z ? *reinterpret_cast<const uint4*>(sX + (m ? 32768 : 16384) + sw128_off(r, 4 * ce + q))
                          : make_uint4(0u, 0u, 0u, 0u);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(STAGE_FREE0 + hs));
        }
        warp_wait(bar(YFULL0 + yb), (Hc >> 1) & 1, kSiteScanMma2);
        tc_fence_after();
        if (wfail) continue;
        const float el = __expf(cl);
        // y pieces of this lane's row: 32 columns in 16-byte pieces (4 for 16-bit y, 8 for fp32)
        constexpr int NPC = sizeof(YT) == 4 ? 8 : 4;
        uint4 pc[NPC];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t ri[16], ro[16];
          tmem_ld16(tmem + tlane + t_yin(yb) + 32 * ce + 16 * hf, ri);
          tmem_ld16(tmem + tlane + t_yoff(yb) + 32 * ce + 16 * hf, ro);
          tmem_wait_ld();
          if (hf == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(YFREE0 + yb));  // Y may be overwritten by head Hc + 2
          }
          float o[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj)
            o[jj] = fmaf(el, __uint_as_float(ro[jj]), rowf * __uint_as_float(ri[jj]));
          if (D) {
            const float4* d4 = reinterpret_cast<const float4*>(D + h * 64 + ce * 32 + 16 * hf);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const uint4 xq = xv[2 * hf + q];
              const float4 da = __ldg(d4 + 2 * q), db = __ldg(d4 + 2 * q + 1);
              const float dq[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
              const uint32_t w4[4] = {xq.x, xq.y, xq.z, xq.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack2<T16>(w4[e]);
                o[q * 8 + 2 * e] = fmaf(dq[2 * e], f.x, o[q * 8 + 2 * e]);
                o[q * 8 + 2 * e + 1] = fmaf(dq[2 * e + 1], f.y, o[q * 8 + 2 * e + 1]);
              }
            }
          }
          if (has_z) {
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const uint4 zq = zv[2 * hf + q];
              const uint32_t w4[4] = {zq.x, zq.y, zq.z, zq.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack2<T16>(w4[e]);
                const float h0 = 0.5f * f.x, h1 = 0.5f * f.y;
                // silu(z) = z * sigmoid(z) = h + h * tanh(h), h = z / 2
                o[q * 8 + 2 * e] *= fmaf(h0, tanh_approx(h0), h0);
                o[q * 8 + 2 * e + 1] *= fmaf(h1, tanh_approx(h1), h1);
              }
            }
          }
          if constexpr (sizeof(YT) == 4) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              pc[4 * hf + q] = make_uint4(__float_as_uint(o[4 * q]), __float_as_uint(o[4 * q + 1]),
                                          __float_as_uint(o[4 * q + 2]), __float_as_uint(o[4 * q + 3]));
          } else {
#pragma unroll
            for (int q = 0; q < 2; ++q)
              pc[2 * hf + q] = make_uint4(pack2<YT>(o[8 * q], o[8 * q + 1]), pack2<YT>(o[8 * q + 2], o[8 * q + 3]),
                                          pack2<YT>(o[8 * q + 4], o[8 * q + 5]), pack2<YT>(o[8 * q + 6], o[8 * q + 7]));
          }
        }
        // Rows are transposed across groups of NPC lanes: each store writes whole 64- or
        // 128-byte row segments instead of 32 scattered 16-byte pieces.
        const int li = lane & (NPC - 1), lr0 = 128 * m + quad * 32 + (lane & ~(NPC - 1));
        lane_transpose<NPC>(pc, li);
#pragma unroll
        for (int j = 0; j < NPC; ++j) {
          const int lj = lr0 + j;
          if (lj < ci.lim) {
            const long long yo = ((ci.tok0 + lj) * H + h) * 64 + ce * 32;
            reinterpret_cast<uint4*>(y + yo)[li] = pc[j];
          }
        }
      }
    }
    if (fail || wfail) *s_abort = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ===========================================================================
// Host side: tensor maps and launches
// ===========================================================================
bool tc_supported(int x_dtype, int P, int N, int cs) {
  return (x_dtype == SSD_BF16 || x_dtype == SSD_F16) && P == 64 && N == 128 && cs == 256;
}

template <bool BF16, typename DT, bool FUSE>
static cudaError_t tc_state_launch(const LaunchCtx& c, const CUtensorMap& mx, const CUtensorMap& mb, const float* A,
                                   const void* dr, const float* bias, float* dt, float* cum, float* states) {
  auto kern = tc_chunk_state_kernel<BF16, DT, FUSE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kStateSmem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)c.H, (unsigned)c.nchunks_max);
  kern<<<grid, 128, kStateSmem, c.stream>>>(mx, mb, A, (const DT*)dr, bias, dt, cum, states, c.cm, c.H, c.H / c.G,
                                            c.use_sp, c.dmin, c.dmax);
  return cudaGetLastError();
}

template <bool BF16>
static cudaError_t tc_state_dt(const LaunchCtx& c, int dt_dtype, const CUtensorMap& mx, const CUtensorMap& mb,
                               const float* A, const void* dr, const float* bias, float* dt, float* cum,
                               float* states) {
  if (!dr) return tc_state_launch<BF16, float, false>(c, mx, mb, A, dr, bias, dt, cum, states);
  switch (dt_dtype) {
    case SSD_F32: return tc_state_launch<BF16, float, true>(c, mx, mb, A, dr, bias, dt, cum, states);
    case SSD_BF16: return tc_state_launch<BF16, __nv_bfloat16, true>(c, mx, mb, A, dr, bias, dt, cum, states);
    case SSD_F16: return tc_state_launch<BF16, __half, true>(c, mx, mb, A, dr, bias, dt, cum, states);
  }
  return cudaErrorInvalidValue;
}

// delta_raw == NULL: dt / cum are inputs; otherwise they are computed (chunk_cumsum fused) and written.
cudaError_t launch_tc_chunk_state(const LaunchCtx& c, int x_dtype, int dt_dtype, const void* u, const void* B,
                                  const float* A, const void* delta_raw, const float* delta_bias, float* dt,
                                  float* cum, float* states, int* tmap_status) {
  const bool bf16 = x_dtype == SSD_BF16;
  CUtensorMap mx, mb;
  if (!make_map_3d(&mx, u, bf16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mb, B, bf16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128)) {
    *tmap_status = 1;
    return cudaErrorInvalidValue;
  }
  *tmap_status = 0;
  if (bf16) return tc_state_dt<true>(c, dt_dtype, mx, mb, A, delta_raw, delta_bias, dt, cum, states);
  return tc_state_dt<false>(c, dt_dtype, mx, mb, A, delta_raw, delta_bias, dt, cum, states);
}

template <bool BF16, typename DT>
static cudaError_t tc_state_pass_launch(const LaunchCtx& c, const CUtensorMap& mx, const CUtensorMap& mb,
                                        const float* A, const void* dr, const float* bias, float* dt, float* cum,
                                        void* prev16, const float* h_init, float* h_last) {
  auto kern = tc_state_pass_kernel<BF16, DT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSpSmem);
  if (e != cudaSuccess) return e;
  const int hpg = c.H / c.G;
  const long long chains = (long long)c.nrows * c.G * ((hpg + 1) / 2);  // (row, head pair)
  if (chains <= 0 || chains > 0x7fffffffll) return cudaErrorInvalidValue;
  kern<<<(unsigned)chains, kSpThreads, kSpSmem, c.stream>>>(
      mx, mb, A, (const DT*)dr, bias, dt, cum, reinterpret_cast<typename T16Of<BF16>::type*>(prev16), h_init,
      h_last, c.cm, c.H, c.H / c.G, c.use_sp, c.dmin, c.dmax);
  return cudaGetLastError();
}

template <bool BF16>
static cudaError_t tc_state_pass_dt(const LaunchCtx& c, int dt_dtype, const CUtensorMap& mx, const CUtensorMap& mb,
                                    const float* A, const void* dr, const float* bias, float* dt, float* cum,
                                    void* prev16, const float* h_init, float* h_last) {
  switch (dt_dtype) {
    case SSD_F32: return tc_state_pass_launch<BF16, float>(c, mx, mb, A, dr, bias, dt, cum, prev16, h_init, h_last);
    case SSD_BF16:
      return tc_state_pass_launch<BF16, __nv_bfloat16>(c, mx, mb, A, dr, bias, dt, cum, prev16, h_init, h_last);
    case SSD_F16: return tc_state_pass_launch<BF16, __half>(c, mx, mb, A, dr, bias, dt, cum, prev16, h_init, h_last);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_tc_state_pass(const LaunchCtx& c, int x_dtype, int dt_dtype, const void* u, const void* B,
                                 const float* A, const void* delta_raw, const float* delta_bias, float* dt,
                                 float* cum, void* prev16, const float* h_init, float* h_last, int* tmap_status) {
  const bool bf16 = x_dtype == SSD_BF16;
  CUtensorMap mx, mb;
  if (!make_map_3d(&mx, u, bf16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mb, B, bf16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128)) {
    *tmap_status = 1;
    return cudaErrorInvalidValue;
  }
  *tmap_status = 0;
  if (!delta_raw) return cudaErrorInvalidValue;
  if (bf16) return tc_state_pass_dt<true>(c, dt_dtype, mx, mb, A, delta_raw, delta_bias, dt, cum, prev16, h_init,
                                          h_last);
  return tc_state_pass_dt<false>(c, dt_dtype, mx, mb, A, delta_raw, delta_bias, dt, cum, prev16, h_init, h_last);
}

template <bool BF16, typename YT>
static cudaError_t tc_scan_launch(const LaunchCtx& c, const CUtensorMap& mx, const CUtensorMap& mc,
                                  const CUtensorMap& mb, const CUtensorMap& mh, const CUtensorMap& mz, int has_z,
                                  const float* A, const float* dt, const float* cum, const float* D, void* y) {
  if (c.H > kScanMaxHeads) return cudaErrorInvalidValue;
  auto kern = tc_chunk_scan_kernel<BF16, YT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kScanSmem);
  if (e != cudaSuccess) return e;
  const int dt_nonneg = (c.dmax >= 0.f) && (c.use_sp || c.dmin >= 0.f);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Heads per item: the heads of an item share one CB (its load, MMA and rounding).
  // Up to 8, fewer when that leaves under two items per CTA. An item's start costs about
  // two heads' time on the CTA; with many rounds of items per CTA the pipeline hides it,
  // but with few rounds (small batches) it does not, and then the block size with the
  // smallest estimated makespan, rounds x (2 + heads per item), is taken.
  const int hpg = c.H / c.G;
  auto n_items = [&](int b) { return 2ll * c.nchunks_max * c.G * ((hpg + b - 1) / b); };
  auto makespan = [&](int b) {
    const long long it = n_items(b), g = it < sms ? it : sms;
    return ((it + g - 1) / g) * (2ll + b);
  };
  int hb = hpg < 8 ? hpg : 8;
  while (hb > 1 && n_items(hb) < 2ll * sms) hb = (hb + 1) / 2;
  if ((n_items(hb) + sms - 1) / sms <= 4) {
    long long best = makespan(hb);
    const int b0 = hb;
    for (int b = b0 + 1; b <= hpg && b <= kScanMaxHeads; ++b) {
      if ((hpg + b - 1) / b == (hpg + b - 2) / (b - 1)) continue;  // same block count as b - 1
      const long long cost = makespan(b);
      if (cost <= best) {
        best = cost;
        hb = b;
      }
    }
  }
  const long long items = n_items(hb);
  if (items > 0x7fffffffll) return cudaErrorInvalidValue;
  const int grid = (int)(items < sms ? items : sms);  // persistent: one CTA per SM
  // Programmatic dependent launch: the kernel may begin while the preceding kernel on the
  // stream (the state pass) finishes; its producer waits for that grid before reading
  // dt, cum and prev16 (griddepcontrol.wait), so only the set-up and the first C / B
  // loads overlap. Used when the fused state pass runs in one wave (chains <= SMs: SMs
  // idle beside it, c1: 3.6 % faster); with several waves it made this kernel slower
  // (c2 -9 %, c4 -11 %), so there the launch is ordinary.
  const long long chains = (long long)c.nrows * c.G * ((hpg + 1) / 2);
  const bool pdl = chains <= sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kScanThreads);
  cfg.dynamicSmemBytes = kScanSmem;
  cfg.stream = c.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, mx, mc, mb, mh, mz, A, dt, cum, D, has_z, reinterpret_cast<YT*>(y), c.cm,
                            c.H, c.G, hb, dt_nonneg, (int)items);
}

cudaError_t launch_tc_chunk_scan(const LaunchCtx& c, int x_dtype, int y_dtype, const void* u, const float* A,
                                 const float* dt, const float* cum, const void* B, const void* C, const void* prev16,
                                 const float* D, const void* z, void* y, int* tmap_status) {
  const bool bf16 = x_dtype == SSD_BF16;
  CUtensorMap mx, mc, mb, mh, mz;
  // prev16 holds the previous-chunk states in the input's 16-bit type, [chunk][head][n][p]
  // (p contiguous: the MN-major B operand of MMA3), so every
  // MMA of the kernel has operands of one type.
  const uint64_t nch = (uint64_t)c.nchunks_max;
  if (!make_map_3d(&mx, u, bf16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mc, C, bf16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mb, B, bf16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mh, prev16, bf16, 64, 128, nch * (uint64_t)c.H, 64, 128, 1)) {
    *tmap_status = 1;
    return cudaErrorInvalidValue;
  }
  // z (same layout as u) is loaded one 128-row half at a time.
  const int has_z = z != nullptr;
  if (!make_map_3d(&mz, has_z ? z : u, bf16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128)) {
    *tmap_status = 1;
    return cudaErrorInvalidValue;
  }
  *tmap_status = 0;
  if (y_dtype == SSD_F32) {
    if (bf16) return tc_scan_launch<true, float>(c, mx, mc, mb, mh, mz, has_z, A, dt, cum, D, y);
    return tc_scan_launch<false, float>(c, mx, mc, mb, mh, mz, has_z, A, dt, cum, D, y);
  }
  if (y_dtype == x_dtype) {
    if (bf16) return tc_scan_launch<true, __nv_bfloat16>(c, mx, mc, mb, mh, mz, has_z, A, dt, cum, D, y);
    return tc_scan_launch<false, __half>(c, mx, mc, mb, mh, mz, has_z, A, dt, cum, D, y);
  }
  return cudaErrorInvalidValue;
}

SSDB200_DEFINE_ERROR_FETCH(fetch_error_tc)

}  // namespace ssdb200
