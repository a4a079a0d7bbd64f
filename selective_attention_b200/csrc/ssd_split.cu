// ssd_split.cu - the SSD forward for fp32 inputs on tcgen05 tensor cores with split-bf16
// products (headdim 64, dstate 128, chunk 256).
//
// Every fp32 operand x is split into two bf16 parts, hi = bf16(x) and lo = bf16(x - hi),
// which together carry 16 significant bits; a product a b is taken as
//   a_hi b_hi + a_hi b_lo + a_lo b_hi
// (three kind::f16 MMAs into one fp32 TMEM accumulator; the dropped a_lo b_lo term and the
// rounding of the parts are each about 2^-18 of |a b|). The reference's tl.dot runs fp32
// operands as TF32 (10-bit mantissas); the three-product split keeps the fp32 chain's
// rel 1e-4 agreement. The stages are those of the CUDA-core chain with its fp32 cumsum and
// state passing (ssd_scan/forward_kernel.py:107-185, :270-328, :350-455):
//   chunk_state  S[p,n]  = sum_l u[l,p] w_l B[l,n],  w_l = exp(min(cum_last - cum_l, 0)) dt_l
//   bmm_chunk    CB[l,s] = sum_n C[l,n] B[s,n]
//   chunk_scan   y[l,p]  = exp(cum_l) sum_n C[l,n] prev[p,n]
//                        + sum_{s <= l} CB[l,s] exp(min(cum_l - cum_s, 0)) dt_s u[s,p]  (+ D u, * silu z)
// Operands are staged by CUDA cores: fp32 loads (all of a step's loads issued before its
// stores), the split, and 16-byte stores into the 128-byte-swizzled layout
// [column / 64][row][column % 64], which one descriptor reads as a K-major operand and
// another as an MN-major one. Two stages alternate, so the staging of step i + 1 overlaps
// the MMAs of step i; one thread issues the MMAs. Every mbarrier wait is bounded; a CTA
// whose wait gives up records a site code and writes nothing.
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace ssdb200 {

using namespace sm100;

namespace {

constexpr unsigned int kSiteSplitState = 0x141;
constexpr unsigned int kSiteSplitBmm = 0x142;
constexpr unsigned int kSiteSplitScan = 0x143;
constexpr int kSplitThreads = 256;

// 8 consecutive fp32 values -> one 16-byte chunk of hi parts and one of lo parts.
__device__ __forceinline__ void store_split8(uint8_t* hi, uint8_t* lo, uint32_t off, const float (&v)[8]) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    h[q] = pack2<__nv_bfloat16>(v[2 * q], v[2 * q + 1]);
    const float2 hf = unpack2<__nv_bfloat16>(h[q]);
    l[q] = pack2<__nv_bfloat16>(v[2 * q] - hf.x, v[2 * q + 1] - hf.y);
  }
  *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void load8(const float* src, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(src));
  const float4 b = __ldg(reinterpret_cast<const float4*>(src + 4));
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

// The three split products of one 16-deep K step into `d`.
__device__ __forceinline__ void mma3(uint32_t d, uint64_t ah, uint64_t al, uint64_t bh, uint64_t bl, uint32_t id,
                                     uint32_t acc) {
  umma_f16(d, ah, bh, id, acc);
  umma_f16(d, ah, bl, id, 1u);
  umma_f16(d, al, bh, id, 1u);
}

// Commit books of the two stage barriers: commits issued per barrier, so a wait can name
// the phase it needs and the exit path can wait for the last one of each.
struct StageBooks {
  int n[2] = {0, 0};
};

// Wait (bounded, every thread) until stage b's MMAs of commit number `c` (1-based) are done.
__device__ __forceinline__ bool wait_commit(uint32_t bar, int c, unsigned int site) {
  return c <= 0 || mbar_wait(bar, (uint32_t)(c - 1) & 1u, site);
}

// Operand tiles written once per (chunk, group) and read with bulk copies: 32 KB each, the bf16
// hi parts (16 KB) then the lo parts (16 KB), in the 128-byte-swizzled layout.
//   Bs  per (chunk, group): 4 tiles, one per 64-token step of chunk_state: the step's B rows as
//       an MN-major operand, [dstate block (2)][64 tokens][64 states], split_b_kernel
//   CBs per (chunk, group): 6 tiles [128 rows][64 source tokens], K-major: half m = 0: source
//       blocks 0, 1; half m = 1: blocks 0..3 (masked CB), bmm_chunk
//   Cs  per (chunk, group): 2 halves x 2 dstate blocks [128 rows][64 states], K-major, bmm_chunk
constexpr int kSplitTile = 32768;

// ---------------------------------------------------------------------------- B tiles
// CTA = (64-token step, group, chunk): the step's B rows (rows at or past lim zero), split.
__global__ void __launch_bounds__(kSplitThreads) split_b_kernel(const float* __restrict__ Bm,
                                                                uint8_t* __restrict__ Bs, ChunkMap cm, int G) {
  const int st = blockIdx.x, g = blockIdx.y, k = blockIdx.z;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int lim = ci.lim, t0 = 64 * st;
  if (t0 >= lim) return;
  const int tid = threadIdx.x;
  uint8_t* dst = Bs + (((size_t)k * G + g) * 4 + st) * kSplitTile;
  float v[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // 64 tokens x 16 chunks of 8 states
    const int q = tid + kSplitThreads * i, r = q >> 4, c8 = q & 15;
    load8(Bm + ((ci.tok0 + min(t0 + r, lim - 1)) * G + g) * 128 + 8 * c8, v[i]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = tid + kSplitThreads * i, r = q >> 4, c8 = q & 15;
    if (t0 + r >= lim) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
    }
    store_split8(dst, dst + 16384, (uint32_t)(c8 >> 3) * 8192u + sw128_off((uint32_t)r, (uint32_t)(c8 & 7)), v[i]);
  }
}

// ---------------------------------------------------------------------------- chunk_state
// CTA = (head, chunk), 256 threads. Steps of 64 tokens: A = the step's B tile (MN-major,
// M = 128 dstate in two 64-wide blocks 8 KB apart), landed by a bulk copy (steps 0 and 1 at
// the start, step st + 1 once thread 0 has issued step st's MMAs and step st - 1's are done);
// B operand = the rows u w (N = 64 headdim, MN-major), split by every thread from registers
// loaded two steps ahead; K = 64 tokens. Warp w reads TMEM lanes 32 (w % 4) (dstate n) and
// columns 32 (w / 4) (headdim p) and writes states[p][n] (n contiguous). mode 1 is the
// backward's intra-chunk state gradient HG[p,n] = sum_{l < length} y_grad[l,p] exp(cum_l) C[l,n]
// (backward_kernel.py:23-93): y_grad rows in place of u, C tiles in place of B, weights exp(cum_l).
constexpr int kSsStage = kSplitTile + 2 * 8192;  // B tile hi | lo | (u w) hi | (u w) lo
constexpr size_t kSsSmem = 1024 + 2 * kSsStage;

__global__ void __launch_bounds__(kSplitThreads, 2) split_chunk_state_kernel(
    const float* __restrict__ u, const uint8_t* __restrict__ Bs, const float* __restrict__ dt,
    const float* __restrict__ cum, float* __restrict__ states, ChunkMap cm, int H, int G, int mode) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  __shared__ float sW[256];
  __shared__ uint64_t bars[4];  // MMAs of the stage done [2], B tile of the stage landed [2]
  __shared__ uint32_t tslot[1];
  const int h = blockIdx.x, k = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int g = h / (H / G), tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long kh = (long long)k * H + h;
  const int lim = ci.lim;
  const int nsteps = (lim + 63) >> 6;
  auto bar_mma = [&](int b) { return smem_u32(&bars[b]); };
  auto bar_a = [&](int b) { return smem_u32(&bars[2 + b]); };
  const uint8_t* bsrc = Bs + ((size_t)k * G + g) * 4 * kSplitTile;
  // u rows of step st: 64 tokens x 8 chunks of 8 headdim columns
  float uv0[2][8], uv1[2][8];
  auto load_u = [&](int st, float (&dst)[2][8]) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      load8(u + ((ci.tok0 + min(64 * st + r, lim - 1)) * H + h) * 64 + 8 * c8, dst[i]);
    }
  };
  load_u(0, uv0);  // in flight during the set-up
  if (nsteps > 1) load_u(1, uv1);
  int a_issued = 0;  // B tiles started (thread 0's count)
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&bars[i]), 1);
    fence_mbar_init();
    for (; a_issued < 2 && a_issued < nsteps; ++a_issued) {
      mbar_expect_tx(bar_a(a_issued), (uint32_t)kSplitTile);
      bulk_load(smem_u32(sm + a_issued * kSsStage), bsrc + a_issued * kSplitTile, (uint32_t)kSplitTile,
                bar_a(a_issued));
    }
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 64);
  {
    const float clast = cum[kh * 256 + 255];
    const float cl = cum[kh * 256 + tid], dl = dt[kh * 256 + tid];
    if (mode == 0) sW[tid] = tid < lim ? expf(fminf(clast - cl, 0.f)) * dl : 0.f;
    else sW[tid] = tid < ci.vlim ? expf(cl) : 0.f;  // backward: y_grad rows past the length ignored
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  constexpr uint32_t ID = idesc_f16(128, 64, true, /*a_mn=*/true, /*b_mn=*/true);
  int committed = 0;  // steps whose MMAs were issued and committed
  bool ok = true;
  // step st on stage b = st & 1 (a literal at each call) with its u rows in `cur`
  auto step = [&](const int st, const int b, float (&cur)[2][8]) {
    uint8_t* aH = sm + b * kSsStage;
    uint8_t* aL = aH + 16384;
    uint8_t* xH = aH + kSplitTile;
    uint8_t* xL = xH + 8192;
    // the (u w) half of stage b was last read by the MMAs of step st - 2
    ok = __syncthreads_and(ok && wait_commit(bar_mma(b), st >> 1, kSiteSplitState)) != 0;
    if (!ok) return;
    tc_fence_after();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      const float w = sW[64 * st + r];  // 0 past lim
#pragma unroll
      for (int e = 0; e < 8; ++e) cur[i][e] *= w;
      store_split8(xH, xL, sw128_off((uint32_t)r, (uint32_t)c8), cur[i]);
    }
    if (st + 2 < nsteps) load_u(st + 2, cur);
    const bool landed = mbar_wait(bar_a(b), (uint32_t)(st >> 1) & 1u, kSiteSplitState);
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok && landed) != 0;
    if (!ok) return;
    if (tid == 0) {
      tc_fence_after();
      const uint32_t bh = smem_u32(aH), bl = smem_u32(aL), xh = smem_u32(xH), xl = smem_u32(xL);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma3(tmem, sdesc_sw128(bh + ks * 2048, 8192, 1024), sdesc_sw128(bl + ks * 2048, 8192, 1024),
             sdesc_sw128(xh + ks * 2048, 16, 1024), sdesc_sw128(xl + ks * 2048, 16, 1024), ID,
             (st > 0 || ks > 0) ? 1u : 0u);
      umma_commit(bar_mma(b));
      // the B tile of step st + 1 goes into the stage step st - 1 used, once its MMAs are done
      if (st + 1 < nsteps && st + 1 >= 2) {
        const int nb = (st + 1) & 1;
        if (mbar_wait(bar_mma(nb), (uint32_t)((st - 1) >> 1) & 1u, kSiteSplitState)) {
          mbar_expect_tx(bar_a(nb), (uint32_t)kSplitTile);
          bulk_load(smem_u32(sm + nb * kSsStage), bsrc + (st + 1) * kSplitTile, (uint32_t)kSplitTile,
                    bar_a(nb));
          a_issued = st + 2;
        }
      }
    }
    ++committed;
  };
  for (int st = 0; st < nsteps && ok; st += 2) {
    step(st, 0, uv0);
    if (st + 1 < nsteps && ok) step(st + 1, 1, uv1);
  }
  // the last commit of each stage barrier (all MMAs are done once both have arrived)
  const bool done = wait_commit(bar_mma(0), (committed + 1) >> 1, kSiteSplitState) &&
                    wait_commit(bar_mma(1), committed >> 1, kSiteSplitState);
  tc_fence_after();
  const bool all_ok = __syncthreads_and(ok && done) != 0;
  if (all_ok) {
    const int n = (warp & 3) * 32 + lane, p0 = 32 * (warp >> 2);
    float* out = states + kh * 8192;
    uint32_t v[32];
    tmem_ld32(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)p0, v);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) out[(p0 + j) * 128 + n] = __uint_as_float(v[j]);
  } else if (tid == 0) {
    // after a failed wait no B copy may still be in flight when the CTA exits (bounded)
    for (int st = max(0, a_issued - 2); st < a_issued; ++st)
      mbar_wait(bar_a(st & 1), (uint32_t)(st >> 1) & 1u, kSiteSplitState);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

// ---------------------------------------------------------------------------- bmm_chunk
// CTA = (128 x 128 tile (rows l, columns s) of the lower block triangle, group, chunk),
// 256 threads, two K steps of 64 states: A = C rows, B operand = B rows, both K-major.
// Rows or columns at or past lim are zero. The tile above the diagonal block is not
// written: chunk_scan below reads CB only where s <= l.
constexpr int kBmStage = 4 * 16384;  // C hi | C lo | B hi | B lo
constexpr size_t kBmSmem = 1024 + kBmStage;

__global__ void __launch_bounds__(kSplitThreads, 2) split_bmm_kernel(const float* __restrict__ Bm,
                                                                    const float* __restrict__ Cm,
                                                                    uint8_t* __restrict__ CBs,
                                                                    uint8_t* __restrict__ Cs, ChunkMap cm, int G) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  __shared__ uint64_t bars[1];
  __shared__ uint32_t tslot[1];
  const int t = blockIdx.x, g = blockIdx.y, k = blockIdx.z;
  const int tl = t > 0 ? 1 : 0, ts = t > 1 ? 1 : 0;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int lim = ci.lim;
  if (128 * tl >= lim) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bar = smem_u32(&bars[0]);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  constexpr uint32_t ID = idesc_f16(128, 128, true, false, false);
  uint8_t* cH = sm;
  uint8_t* cL = sm + 16384;
  uint8_t* bH = sm + 32768;
  uint8_t* bL = sm + 49152;
  // the C rows of half tl as chunk_scan's Yoff operand tiles (written by the ts = 0 CTA)
  uint8_t* cdst = Cs + (((size_t)k * G + g) * 2 + tl) * (2 * kSplitTile);
  float cv[4][8], bv[4][8];
  auto load_step = [&](int st) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // 128 rows x 8 chunks of 8 states
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      load8(Cm + ((ci.tok0 + min(128 * tl + r, lim - 1)) * G + g) * 128 + 64 * st + 8 * c8, cv[i]);
      load8(Bm + ((ci.tok0 + min(128 * ts + r, lim - 1)) * G + g) * 128 + 64 * st + 8 * c8, bv[i]);
    }
  };
  load_step(0);
  bool ok = true;
  int commits = 0;
  for (int st = 0; st < 2; ++st) {
    ok = __syncthreads_and(ok && wait_commit(bar, commits, kSiteSplitBmm)) != 0;
    if (!ok) break;
    tc_fence_after();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      if (128 * tl + r >= lim) {
#pragma unroll
        for (int e = 0; e < 8; ++e) cv[i][e] = 0.f;
      }
      if (128 * ts + r >= lim) {
#pragma unroll
        for (int e = 0; e < 8; ++e) bv[i][e] = 0.f;
      }
      const uint32_t off = sw128_off((uint32_t)r, (uint32_t)c8);
      store_split8(cH, cL, off, cv[i]);
      store_split8(bH, bL, off, bv[i]);
      if (ts == 0) store_split8(cdst + st * kSplitTile, cdst + st * kSplitTile + 16384, off, cv[i]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ch = smem_u32(cH), cl = smem_u32(cL), bh = smem_u32(bH), bl = smem_u32(bL);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma3(tmem, sdesc_sw128(ch + ks * 32, 16, 1024), sdesc_sw128(cl + ks * 32, 16, 1024),
             sdesc_sw128(bh + ks * 32, 16, 1024), sdesc_sw128(bl + ks * 32, 16, 1024), ID,
             (st > 0 || ks > 0) ? 1u : 0u);
      umma_commit(bar);
    }
    ++commits;
    if (st == 0) load_step(1);
  }
  const bool done = wait_commit(bar, commits, kSiteSplitBmm);
  tc_fence_after();
  if (__syncthreads_and(ok && done)) {
    // thread = row r (TMEM lane); warps 4..7 take the tile's second 64-column block. The
    // block leaves as chunk_scan's A operand tile: masked to s <= l < lim, split into hi and
    // lo, in the 128-byte-swizzled K-major layout a bulk copy lands as is.
    const int r = (warp & 3) * 32 + lane, cb = warp >> 2, l = 128 * tl + r;
    uint8_t* dst = CBs + (((size_t)k * G + g) * 6 + (tl ? 2 : 0) + 2 * ts + cb) * kSplitTile;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(64 * cb + 32 * hf), v);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int s = 128 * ts + 64 * cb + 32 * hf + 8 * q + e;
          f[e] = (s <= l && l < lim) ? __uint_as_float(v[8 * q + e]) : 0.f;
        }
        store_split8(dst, dst + 16384, sw128_off((uint32_t)r, (uint32_t)(4 * hf + q)), f);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ---------------------------------------------------------------------------- chunk_scan
// CTA = (half m of the chunk: rows l in [128 m, 128 m + 128), head, chunk), 256 threads.
// Steps of K = 64, all with A = 128 rows x 64 (K-major) and B = 64 x 64:
//   steps 0, 1   Yoff += C[l, n-block] prev[p, n-block]^T           (prev K-major)
//   steps 2...   Yin  += M[l, s-block] u[s-block, p]                 (u MN-major)
// with M[l,s] = CB[l,s] exp(min(cum_l - cum_s, 0)) dt_s for s <= l < lim, else 0, over the
// source blocks s < min(128 m + 128, lim). The A tiles (C rows, masked CB) arrive split and
// swizzled from bmm_chunk, one bulk copy each: steps 0 and 1 at the start, step st + 1 as
// soon as thread 0 has issued step st's MMAs and step st - 1's are done; every thread splits
// the B rows, loaded two steps ahead into one of two register sets. When cum is
// non-increasing over the chunk (the min(., 0) clamp is then inert) and falls by at most
// kScFacMax over the half, the decay is factored at the half's first row l0:
//   exp(cum_l - cum_s) = exp(cum_l - cum_l0) * exp(cum_l0 - cum_s),
// the column factor times dt_s scales the u rows (B = w_s u_s, so A is CB itself), and the
// row factor multiplies the row's Yin in the epilogue (a common factor of every term of the
// row's sum, so the fp32 accumulation loses nothing; both factors stay inside fp32's range).
// Other halves rebuild each CB tile in place element by element. The epilogue (thread =
// TMEM lane = row, warps 4..7 the second half of the columns) forms exp(cum_l) Yoff +
// rowf_l Yin in shared memory; then a coalesced pass adds D u and the z gate and writes y.
constexpr int kScThreads = kSplitThreads;
constexpr int kScStage = kSplitTile + 2 * 8192;    // A hi | A lo | B hi | B lo
constexpr size_t kScSmem = 1024 + 2 * kScStage;
constexpr int kScYld = 68;         // row stride (floats) of the epilogue's Y tile (16-byte rows)
constexpr float kScFacMax = 80.f;  // largest decay over a half for the factored form (e^80 < FLT_MAX)

__global__ void __launch_bounds__(kScThreads, 2) split_chunk_scan_kernel(
    const float* __restrict__ u, const float* __restrict__ dt, const float* __restrict__ cum,
    const uint8_t* __restrict__ Cs, const float* __restrict__ prev, const uint8_t* __restrict__ CBs,
    const float* __restrict__ D, const float* __restrict__ z, float* __restrict__ y, ChunkMap cm, int H, int G) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  __shared__ __align__(16) float sCum[256], sDt[256], sW[256];
  __shared__ uint64_t bars[4];  // MMAs of the stage done [2], A tile of the stage landed [2]
  __shared__ uint32_t tslot[1];
  const int m = blockIdx.x, h = blockIdx.y, k = blockIdx.z;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int lim = ci.lim, l0 = 128 * m;
  if (l0 >= lim) return;
  const int g = h / (H / G), tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long kh = (long long)k * H + h;
  const float* pk = prev + kh * 8192;
  const int send = min(l0 + 128, lim);  // source tokens s < send
  const int nsteps = 2 + ((send + 63) >> 6);
  auto bar_mma = [&](int b) { return smem_u32(&bars[b]); };
  auto bar_a = [&](int b) { return smem_u32(&bars[2 + b]); };
  // B rows of step st: prev rows p (steps 0, 1) or u rows 64 (st - 2) + r; 64 rows x 8 chunks of 8
  float bv0[2][8], bv1[2][8];
  auto load_b = [&](int st, float (&dst)[2][8]) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      if (st < 2) load8(pk + r * 128 + 64 * st + 8 * c8, dst[i]);
      else load8(u + ((ci.tok0 + min(64 * (st - 2) + r, lim - 1)) * H + h) * 64 + 8 * c8, dst[i]);
    }
  };
  load_b(0, bv0);  // in flight during the set-up
  load_b(1, bv1);
  const uint8_t* cs = Cs + (((size_t)k * G + g) * 2 + m) * (2 * kSplitTile);
  const uint8_t* cbs = CBs + (((size_t)k * G + g) * 6 + (m ? 2 : 0)) * kSplitTile;
  auto a_src = [&](int st) { return st < 2 ? cs + st * kSplitTile : cbs + (st - 2) * kSplitTile; };
  if (tid == 0) {
    // the barriers, and the A tiles of steps 0 and 1 started at once
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&bars[i]), 1);
    fence_mbar_init();
    for (int st = 0; st < 2; ++st) {
      mbar_expect_tx(bar_a(st), (uint32_t)kSplitTile);
      bulk_load(smem_u32(sm + st * kScStage), a_src(st), (uint32_t)kSplitTile, bar_a(st));
    }
  }
  int a_issued = 2;  // A tiles started (thread 0's count)
  if (warp == 0) tmem_alloc(smem_u32(tslot), 128);
  float c_t;
  {
    // L2 prefetch (128-byte lines) of the epilogue's u and z rows and of the steps' u rows
    const int row = tid >> 1, hb = tid & 1, l = l0 + row;
    if (l < lim) {
      const long long o = ((ci.tok0 + l) * H + h) * 64 + 32 * hb;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(u + o));
      if (z) asm volatile("prefetch.global.L2 [%0];" ::"l"(z + o));
    }
    if (m == 1 && row < lim)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(u + ((ci.tok0 + row) * H + h) * 64 + 32 * hb));
    c_t = cum[kh * 256 + tid];
    sCum[tid] = c_t;
    sDt[tid] = dt[kh * 256 + tid];
  }
  __syncthreads();
  const bool nonincr = tid == 0 || tid >= lim || c_t <= sCum[tid - 1];
  const bool fac = __syncthreads_and(nonincr) && sCum[l0] - sCum[send - 1] <= kScFacMax;
  sW[tid] = (fac && tid < send) ? expf(sCum[l0] - c_t) * sDt[tid] : 0.f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  bool fin = true;
  float4 ue[8], ze[8];
  const int c4 = tid & 15, rb = tid >> 4;
  {
    constexpr uint32_t ID_OFF = idesc_f16(128, 64, true, false, false);
    constexpr uint32_t ID_IN = idesc_f16(128, 64, true, false, /*b_mn=*/true);
    int committed = 0;  // steps whose MMAs were issued and committed (stage st & 1 holds st >> 1 before step st)
    bool ok = true;
    // step st on stage b = st & 1 (a literal at each call) with its B rows in `cur`
    auto step = [&](const int st, const int b, float (&cur)[2][8]) {
      const int s0 = 64 * (st - 2);
      uint8_t* aH = sm + b * kScStage;
      uint8_t* aL = aH + 16384;
      uint8_t* xH = aH + kSplitTile;
      uint8_t* xL = xH + 8192;
      // the B half of stage b was last read by the MMAs of step st - 2
      ok = named_bar_and(1, kSplitThreads, ok && wait_commit(bar_mma(b), st >> 1, kSiteSplitScan));
      if (!ok) return;
      tc_fence_after();
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
        if (st >= 2) {
          // u rows past lim are zero; under the factored decay a row carries w_s
          const float w = s0 + r >= lim ? 0.f : (fac ? sW[s0 + r] : 1.f);
#pragma unroll
          for (int e = 0; e < 8; ++e) cur[i][e] *= w;
        }
        store_split8(xH, xL, sw128_off((uint32_t)r, (uint32_t)c8), cur[i]);
      }
      if (st + 2 < nsteps) load_b(st + 2, cur);
      const bool landed = mbar_wait(bar_a(b), (uint32_t)(st >> 1) & 1u, kSiteSplitScan);
      if (landed && !fac && st >= 2) {
        // element-by-element decay: A = CB exp(min(cum_l - cum_s, 0)) dt_s, rebuilt in place
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
          const uint32_t off = sw128_off((uint32_t)r, (uint32_t)c8);
          const uint4 hv = *reinterpret_cast<const uint4*>(aH + off);
          const uint4 lv = *reinterpret_cast<const uint4*>(aL + off);
          const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, lw[4] = {lv.x, lv.y, lv.z, lv.w};
          const float cl = sCum[l0 + r];
          float f[8];
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const float2 a = unpack2<__nv_bfloat16>(hw[e2]), c = unpack2<__nv_bfloat16>(lw[e2]);
            const int sa = s0 + 8 * c8 + 2 * e2;
            f[2 * e2] = (a.x + c.x) * expf(fminf(cl - sCum[sa], 0.f)) * sDt[sa];
            f[2 * e2 + 1] = (a.y + c.y) * expf(fminf(cl - sCum[sa + 1], 0.f)) * sDt[sa + 1];
          }
          store_split8(aH, aL, off, f);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      ok = named_bar_and(1, kSplitThreads, ok && landed);
      if (!ok) return;
      if (tid == 0) {
        tc_fence_after();
        const uint32_t ah = smem_u32(aH), al = smem_u32(aL), xh = smem_u32(xH), xl = smem_u32(xL);
        if (st < 2) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma3(tmem, sdesc_sw128(ah + ks * 32, 16, 1024), sdesc_sw128(al + ks * 32, 16, 1024),
                 sdesc_sw128(xh + ks * 32, 16, 1024), sdesc_sw128(xl + ks * 32, 16, 1024), ID_OFF,
                 (st > 0 || ks > 0) ? 1u : 0u);
        } else {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma3(tmem + 64, sdesc_sw128(ah + ks * 32, 16, 1024), sdesc_sw128(al + ks * 32, 16, 1024),
                 sdesc_sw128(xh + ks * 2048, 16, 1024), sdesc_sw128(xl + ks * 2048, 16, 1024), ID_IN,
                 (st > 2 || ks > 0) ? 1u : 0u);
        }
        umma_commit(bar_mma(b));
        // the A tile of step st + 1 goes into the stage that step st - 1 used, once its MMAs are done
        if (st + 1 < nsteps && st + 1 >= 2) {
          const int nb = (st + 1) & 1;
          if (mbar_wait(bar_mma(nb), (uint32_t)((st - 1) >> 1) & 1u, kSiteSplitScan)) {
            mbar_expect_tx(bar_a(nb), (uint32_t)kSplitTile);
            bulk_load(smem_u32(sm + nb * kScStage), a_src(st + 1), (uint32_t)kSplitTile, bar_a(nb));
            a_issued = st + 2;
          }
        }
      }
      ++committed;
    };
    for (int st = 0; st < nsteps && ok; st += 2) {
      step(st, 0, bv0);
      if (st + 1 < nsteps && ok) step(st + 1, 1, bv1);
    }
    // The epilogue's u (D term) and z rows, loaded while the last MMAs run: thread (rb, c4)
    // takes 16-byte column piece c4 of rows rb + 16 i (rows clamped; stores skip rows past lim).
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const long long o = ((ci.tok0 + min(l0 + rb + 16 * i, lim - 1)) * H + h) * 64 + 4 * c4;
      ue[i] = D ? __ldg(reinterpret_cast<const float4*>(u + o)) : make_float4(0.f, 0.f, 0.f, 0.f);
      ze[i] = z ? __ldg(reinterpret_cast<const float4*>(z + o)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const bool drained = wait_commit(bar_mma(0), (committed + 1) >> 1, kSiteSplitScan) &&
                         wait_commit(bar_mma(1), committed >> 1, kSiteSplitScan);
    fin = ok && drained;
  }
  tc_fence_after();
  const bool all_ok = __syncthreads_and(fin) != 0;
  if (all_ok) {
    // Y tile [128 rows][64 columns] (row stride kScYld) over the stages, which the MMAs no longer read
    float* sY = reinterpret_cast<float*>(sm);
    const int r = (warp & 3) * 32 + lane, c0 = 32 * (warp >> 2);
    const uint32_t tl = (uint32_t)((warp & 3) * 32) << 16;
    const float el = expf(sCum[l0 + r]);
    const float rowf = fac ? expf(sCum[l0 + r] - sCum[l0]) : 1.f;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      uint32_t vo[16], vi[16];
      tmem_ld16(tmem + tl + (uint32_t)(c0 + 16 * hf), vo);
      tmem_ld16(tmem + tl + 64u + (uint32_t)(c0 + 16 * hf), vi);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 o4;
        o4.x = fmaf(el, __uint_as_float(vo[4 * q]), rowf * __uint_as_float(vi[4 * q]));
        o4.y = fmaf(el, __uint_as_float(vo[4 * q + 1]), rowf * __uint_as_float(vi[4 * q + 1]));
        o4.z = fmaf(el, __uint_as_float(vo[4 * q + 2]), rowf * __uint_as_float(vi[4 * q + 2]));
        o4.w = fmaf(el, __uint_as_float(vo[4 * q + 3]), rowf * __uint_as_float(vi[4 * q + 3]));
        *reinterpret_cast<float4*>(sY + r * kScYld + c0 + 16 * hf + 4 * q) = o4;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
  if (tid == 0 && !all_ok) {
    // after a failed wait no A copy may still be in flight when the CTA exits (bounded)
    for (int st = max(0, a_issued - 2); st < a_issued; ++st)
      mbar_wait(bar_a(st & 1), (uint32_t)(st >> 1) & 1u, kSiteSplitScan);
  }
  if (!all_ok) return;
  const float* sY = reinterpret_cast<const float*>(sm);
  const float4 d4 = D ? __ldg(reinterpret_cast<const float4*>(D + h * 64 + 4 * c4)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = rb + 16 * i, l = l0 + r;
    if (l >= lim) break;
    float4 v = *reinterpret_cast<const float4*>(sY + r * kScYld + 4 * c4);
    if (D) {
      v.x = fmaf(d4.x, ue[i].x, v.x);
      v.y = fmaf(d4.y, ue[i].y, v.y);
      v.z = fmaf(d4.z, ue[i].z, v.z);
      v.w = fmaf(d4.w, ue[i].w, v.w);
    }
    if (z) {
      v.x *= silu(ze[i].x);
      v.y *= silu(ze[i].y);
      v.z *= silu(ze[i].z);
      v.w *= silu(ze[i].w);
    }
    *reinterpret_cast<float4*>(y + ((ci.tok0 + l) * H + h) * 64 + 4 * c4) = v;
  }
}

// ---------------------------------------------------------------------------- backward state-side
// The backward's state-side products for fp32 inputs (backward_kernel.py:255-262, :402-415,
// :522-538), per (half m: rows l in [128 m, 128 m + 128), head, chunk), 256 threads. With
// s_l = exp(min(cum_last - cum_l, 0)), w_l = s_l dt_l and e_l = exp(cum_l) for l < length
// (0 past it):
//   accS[l,p]     = s_l sum_n B[l,n] hg[p,n]           A = B rows (K-major), hg K-major
//   B_grad[l,:]  += w_l sum_p u[l,p] hg[p,:]           A = u rows (K-major), hg MN-major
//   C_grad[l,:]  += e_l sum_p y_grad[l,p] prev[p,:]    A = y_grad rows, prev MN-major
//   gC[l]         = sum_n (that C_grad row) C[l,n]
// hg and prev hold [p][n] rows: one split tile [n block][64 p][64 n] serves as the K-major
// operand of accS and as the MN-major one of B_grad / C_grad. A CTA splits its operands into
// shared memory, runs its product's MMAs (split-bf16, three per K step) into TMEM, and thread =
// TMEM lane = row scales the rows; B_grad / C_grad rows are summed over the group's heads by
// 16-byte atomics in L2, as the CUDA-core kernel does.
// One launch per product (MODE 0: accS, 1: B_grad, 2: C_grad and gC), so that each CTA holds
// only its own operands and several CTAs share an SM.
template <int MODE>
struct SgCfg {
  static constexpr size_t kSmem = 1024 + (MODE == 0 ? 3 : 2) * 32768;  // A rows (64 or 32 KB) | hg or prev 32 KB
  static constexpr uint32_t kCols = MODE == 0 ? 64 : 128;
  static constexpr int kMinBlocks = MODE == 0 ? 2 : 3;
};

template <int MODE>
__global__ void __launch_bounds__(kSplitThreads, SgCfg<MODE>::kMinBlocks) split_state_grad_kernel(
    const float* __restrict__ u, const float* __restrict__ Bm, const float* __restrict__ Cm,
    const float* __restrict__ yg, const float* __restrict__ dt, const float* __restrict__ cum,
    const float* __restrict__ prev, const float* __restrict__ hg, float* __restrict__ accS_out,
    float* __restrict__ Bgrad, float* __restrict__ Cgrad, float* __restrict__ gC_out, ChunkMap cm, int H, int G) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  __shared__ float sF[128], sG[128];  // the row factor (s_l, w_l or e_l) | gC partial sums
  __shared__ uint64_t bars[1];
  __shared__ uint32_t tslot[1];
  const int m = blockIdx.x, h = blockIdx.y, k = blockIdx.z;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int lim = ci.lim, vl = ci.vlim, l0 = 128 * m;
  if (l0 >= lim) return;
  const int g = h / (H / G), tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long kh = (long long)k * H + h;
  constexpr uint32_t AB = MODE == 0 ? 65536u : 32768u;  // bytes of the A rows (hi then lo)
  uint8_t* aH = sm;  // MODE 0: B rows [n block (2)][128 rows][128 B]; else u / y_grad rows [128][64 p]
  uint8_t* aL = sm + AB / 2;
  uint8_t* hH = sm + AB;  // hg (MODE 0, 1) or prev (MODE 2): [n block (2)][64 p][64 n], hi then lo
  uint8_t* hL = sm + AB + 16384;
  const uint32_t bar = smem_u32(&bars[0]);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), SgCfg<MODE>::kCols);
  if (tid < 128) {
    const int l = l0 + tid;
    const float clast = cum[kh * 256 + 255], cl = cum[kh * 256 + l];
    const float s_l = l < vl ? expf(fminf(clast - cl, 0.f)) : 0.f;
    sF[tid] = MODE == 0 ? s_l : (MODE == 1 ? s_l * dt[kh * 256 + l] : (l < vl ? expf(cl) : 0.f));
    sG[tid] = 0.f;
  }
  // operands, split; each batch's four loads issued before its stores
  float v[4][8];
  if (MODE == 0) {
#pragma unroll 1
    for (int bt = 0; bt < 2; ++bt) {  // B rows: 128 x 16 chunks of 8 states
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int q = tid + kSplitThreads * (4 * bt + i), r = q >> 4, c8 = q & 15;
        load8(Bm + ((ci.tok0 + min(l0 + r, lim - 1)) * G + g) * 128 + 8 * c8, v[i]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int q = tid + kSplitThreads * (4 * bt + i), r = q >> 4, c8 = q & 15;
        store_split8(aH, aL, (uint32_t)(c8 >> 3) * 16384u + sw128_off((uint32_t)r, (uint32_t)(c8 & 7)), v[i]);
      }
    }
  } else {
    const float* src = MODE == 1 ? u : yg;  // 128 rows x 8 chunks of 8 headdim columns
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      load8(src + ((ci.tok0 + min(l0 + r, lim - 1)) * H + h) * 64 + 8 * c8, v[i]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      store_split8(aH, aL, sw128_off((uint32_t)r, (uint32_t)c8), v[i]);
    }
  }
  {
    const float* src = (MODE == 2 ? prev : hg) + kh * 8192;  // 64 p x 16 chunks of 8 states
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 4, c8 = q & 15;
      load8(src + r * 128 + 8 * c8, v[i]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 4, c8 = q & 15;
      store_split8(hH, hL, (uint32_t)(c8 >> 3) * 8192u + sw128_off((uint32_t)r, (uint32_t)(c8 & 7)), v[i]);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    const uint32_t ah = smem_u32(aH), al = smem_u32(aL), hh = smem_u32(hH), hl = smem_u32(hL);
    if (MODE == 0) {
      constexpr uint32_t ID_S = idesc_f16(128, 64, true, false, false);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {  // K = 128 states in two blocks
        const uint32_t ka = (uint32_t)(ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u;
        const uint32_t kb = (uint32_t)(ks >> 2) * 8192u + (uint32_t)(ks & 3) * 32u;
        mma3(tmem, sdesc_sw128(ah + ka, 16, 1024), sdesc_sw128(al + ka, 16, 1024), sdesc_sw128(hh + kb, 16, 1024),
             sdesc_sw128(hl + kb, 16, 1024), ID_S, ks > 0 ? 1u : 0u);
      }
    } else {
      constexpr uint32_t ID_G = idesc_f16(128, 128, true, false, /*b_mn=*/true);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)  // K = 64 headdim, N = 128 states
        mma3(tmem, sdesc_sw128(ah + ks * 32, 16, 1024), sdesc_sw128(al + ks * 32, 16, 1024),
             sdesc_sw128(hh + ks * 2048, 8192, 1024), sdesc_sw128(hl + ks * 2048, 8192, 1024), ID_G,
             ks > 0 ? 1u : 0u);
    }
    umma_commit(bar);
  }
  const bool done = mbar_wait(bar, 0u, kSiteSplitState);
  tc_fence_after();
  if (__syncthreads_and(done)) {
    const int r = (warp & 3) * 32 + lane, hc = warp >> 2, l = l0 + r;
    const uint32_t tl = (uint32_t)((warp & 3) * 32) << 16;
    const float f = sF[r];
    if (MODE == 0) {
      uint32_t a[32];
      tmem_ld32(tmem + tl + (uint32_t)(32 * hc), a);
      tmem_wait_ld();
      float4* o = reinterpret_cast<float4*>(accS_out + (kh * 256 + l) * 64 + 32 * hc);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o[j] = make_float4(f * __uint_as_float(a[4 * j]), f * __uint_as_float(a[4 * j + 1]),
                           f * __uint_as_float(a[4 * j + 2]), f * __uint_as_float(a[4 * j + 3]));
    } else {
      const long long row = ((ci.tok0 + l) * G + g) * 128 + 64 * hc;
      float* dst = MODE == 1 ? Bgrad : Cgrad;
      float gsum = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t a[32];
        tmem_ld32(tmem + tl + (uint32_t)(64 * hc + 32 * half), a);
        tmem_wait_ld();
        if (l < vl) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 q = make_float4(f * __uint_as_float(a[4 * j]), f * __uint_as_float(a[4 * j + 1]),
                                         f * __uint_as_float(a[4 * j + 2]), f * __uint_as_float(a[4 * j + 3]));
            atomicAdd(reinterpret_cast<float4*>(dst + row + 32 * half + 4 * j), q);
            if (MODE == 2) {
              const float4 c = __ldg(reinterpret_cast<const float4*>(Cm + row + 32 * half + 4 * j));
              gsum = fmaf(q.x, c.x, fmaf(q.y, c.y, fmaf(q.z, c.z, fmaf(q.w, c.w, gsum))));
            }
          }
        }
      }
      if (MODE == 2) atomicAdd(&sG[r], gsum);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (MODE == 2 && tid < 128) gC_out[kh * 256 + l0 + tid] = l0 + tid < vl ? sG[tid] : 0.f;
  if (warp == 0) tmem_dealloc(tmem, SgCfg<MODE>::kCols);
}

// ---------------------------------------------------------------------------- backward accY
// The backward's intra-chunk product for fp32 inputs (backward_kernel.py:272-293),
//   accY[l,p] = sum_{l <= s < length} CB[s,l] exp(min(cum_s - cum_l, 0)) y_grad[s,p],
// per (half m: rows l in [128 m, 128 m + 128), head, chunk), 256 threads, for the fp32 intra
// kernel (ssd_bwd.cu bwd_intra_split). Steps of 64 source tokens s >= 128 m: A = the
// decay-weighted CB transposed, [l][s], staged MN-major from CB's rows s (l contiguous: two
// 64-wide l blocks 8 KB apart), B operand = the y_grad rows s (MN-major); both split by every
// thread from fp32 loads issued one step ahead; two stages alternate.
constexpr int kAyStage = 2 * 16384 + 2 * 8192;  // A hi | A lo | y hi | y lo
constexpr size_t kAySmem = 1024 + 2 * kAyStage;

__global__ void __launch_bounds__(kSplitThreads, 2) split_bwd_accy_kernel(
    const float* __restrict__ CB, const float* __restrict__ yg, const float* __restrict__ cum,
    float* __restrict__ accY_out, ChunkMap cm, int H, int G) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  __shared__ float sC[256];
  __shared__ uint64_t bars[2];
  __shared__ uint32_t tslot[1];
  const int m = blockIdx.x, h = blockIdx.y, k = blockIdx.z;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int lim = ci.lim, vl = ci.vlim, l0 = 128 * m;
  if (l0 >= lim) return;
  const int g = h / (H / G), tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long kh = (long long)k * H + h;
  const float* cbk = CB + ((long long)k * G + g) * 65536;
  const int s_beg = l0, nsteps = vl > s_beg ? (vl - s_beg + 63) >> 6 : 0;
  float av[4][8], yv[2][8];
  // step st: CB rows s = s_beg + 64 st + r (64 rows x 16 chunks of 8 l), y_grad rows s
  auto load_step = [&](int st) {
    const int s0 = s_beg + 64 * st;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 4, c8 = q & 15;
      load8(cbk + (long long)min(s0 + r, 255) * 256 + l0 + 8 * c8, av[i]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      load8(yg + ((ci.tok0 + min(s0 + r, lim - 1)) * H + h) * 64 + 8 * c8, yv[i]);
    }
  };
  if (nsteps > 0) load_step(0);
  if (tid == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 64);
  sC[tid] = cum[kh * 256 + tid];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  constexpr uint32_t ID = idesc_f16(128, 64, true, /*a_mn=*/true, /*b_mn=*/true);
  bool ok = true;
  int committed = 0;
  for (int st = 0; st < nsteps; ++st) {
    const int b = st & 1, s0 = s_beg + 64 * st;
    uint8_t* aH = sm + b * kAyStage;
    uint8_t* aL = aH + 16384;
    uint8_t* xH = aH + 32768;
    uint8_t* xL = aH + 40960;
    // this stage was last read by the MMAs of step st - 2
    ok = __syncthreads_and(ok && wait_commit(smem_u32(&bars[b]), st >> 1, kSiteSplitState)) != 0;
    if (!ok) break;
    tc_fence_after();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 4, c8 = q & 15, s = s0 + r;
      const float cs_ = sC[min(s, 255)];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int l = l0 + 8 * c8 + e;
        av[i][e] = (s >= l && s < vl && l < vl) ? av[i][e] * expf(fminf(cs_ - sC[l], 0.f)) : 0.f;
      }
      store_split8(aH, aL, (uint32_t)(c8 >> 3) * 8192u + sw128_off((uint32_t)r, (uint32_t)(c8 & 7)), av[i]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      if (s0 + r >= vl) {
#pragma unroll
        for (int e = 0; e < 8; ++e) yv[i][e] = 0.f;
      }
      store_split8(xH, xL, sw128_off((uint32_t)r, (uint32_t)c8), yv[i]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ah = smem_u32(aH), al = smem_u32(aL), xh = smem_u32(xH), xl = smem_u32(xL);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma3(tmem, sdesc_sw128(ah + ks * 2048, 8192, 1024), sdesc_sw128(al + ks * 2048, 8192, 1024),
             sdesc_sw128(xh + ks * 2048, 16, 1024), sdesc_sw128(xl + ks * 2048, 16, 1024), ID,
             (st > 0 || ks > 0) ? 1u : 0u);
      umma_commit(smem_u32(&bars[b]));
    }
    ++committed;
    if (st + 1 < nsteps) load_step(st + 1);
  }
  // step (committed - 1)'s commit completes after every earlier MMA of the CTA
  const bool done = committed == 0 ||
                    wait_commit(smem_u32(&bars[(committed - 1) & 1]), ((committed - 1) >> 1) + 1, kSiteSplitState);
  tc_fence_after();
  if (__syncthreads_and(ok && done)) {
    const int r = (warp & 3) * 32 + lane, c0 = 32 * (warp >> 2);
    float4* o = reinterpret_cast<float4*>(accY_out + (kh * 256 + l0 + r) * 64 + c0);
    if (committed == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)c0, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]), __uint_as_float(v[4 * j + 2]),
                           __uint_as_float(v[4 * j + 3]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

// ---------------------------------------------------------------------------- backward G
// G[l,s] = sum_p y_grad[l,p] u[s,p] for fp32 inputs (the product behind CB_grad,
// backward_kernel.py:632-659), per (128 x 128 block of the lower block triangle, head, chunk):
// y_grad rows (A) and u rows (B operand), both K-major, split; G leaves as fp32 rows for the
// fp32 intra kernel (ssd_bwd.cu bwd_intra_split), which applies the decay, the atomics and
// the decay sums.
constexpr size_t kBgSmem = 1024 + 2 * 32768;  // y rows hi | lo, u rows hi | lo

__global__ void __launch_bounds__(kSplitThreads, 3) split_bwd_g_kernel(const float* __restrict__ u,
                                                                      const float* __restrict__ yg,
                                                                      float* __restrict__ Gout, ChunkMap cm, int H) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024_shared(smem_raw);
  __shared__ uint64_t bars[1];
  __shared__ uint32_t tslot[1];
  const int t = blockIdx.x, h = blockIdx.y, k = blockIdx.z;
  const int lb = t > 0 ? 1 : 0, sb = t > 1 ? 1 : 0;  // (0, 0), (1, 0), (1, 1)
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int lim = ci.lim;
  if (128 * lb >= lim) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long kh = (long long)k * H + h;
  uint8_t* yH = sm;
  uint8_t* yL = sm + 16384;
  uint8_t* uH = sm + 32768;
  uint8_t* uL = sm + 49152;
  const uint32_t bar = smem_u32(&bars[0]);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 128);
  float v[4][8];
#pragma unroll 1
  for (int which = 0; which < 2; ++which) {  // y_grad rows of block lb, u rows of block sb: 128 x 8 chunks
    const float* src = which ? u : yg;
    const int r0 = 128 * (which ? sb : lb);
    uint8_t* dh = which ? uH : yH;
    uint8_t* dl = which ? uL : yL;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      load8(src + ((ci.tok0 + min(r0 + r, lim - 1)) * H + h) * 64 + 8 * c8, v[i]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int q = tid + kSplitThreads * i, r = q >> 3, c8 = q & 7;
      store_split8(dh, dl, sw128_off((uint32_t)r, (uint32_t)c8), v[i]);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    constexpr uint32_t ID = idesc_f16(128, 128, true, false, false);
    const uint32_t yh = smem_u32(yH), yl = smem_u32(yL), uh = smem_u32(uH), ul = smem_u32(uL);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
      mma3(tmem, sdesc_sw128(yh + ks * 32, 16, 1024), sdesc_sw128(yl + ks * 32, 16, 1024),
           sdesc_sw128(uh + ks * 32, 16, 1024), sdesc_sw128(ul + ks * 32, 16, 1024), ID, ks > 0 ? 1u : 0u);
    umma_commit(bar);
  }
  const bool done = mbar_wait(bar, 0u, kSiteSplitState);
  tc_fence_after();
  if (__syncthreads_and(done)) {
    // the tile goes through shared memory (the operands are consumed): [128 rows][32 float4],
    // float4 index ^ (row & 7) so that both the row-per-thread writes and the row-per-warp
    // reads are free of bank conflicts; then each warp stores whole 512-byte rows
    const int r = (warp & 3) * 32 + lane, c0 = 64 * (warp >> 2);
    float4* st = reinterpret_cast<float4*>(sm);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      uint32_t a[32];
      tmem_ld32(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(c0 + 32 * hf), a);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c4 = (c0 >> 2) + 8 * hf + j;
        st[r * 32 + (c4 ^ (r & 7))] = make_float4(__uint_as_float(a[4 * j]), __uint_as_float(a[4 * j + 1]),
                                                  __uint_as_float(a[4 * j + 2]), __uint_as_float(a[4 * j + 3]));
      }
    }
    __syncthreads();
    float* out = Gout + (kh * 256 + 128 * lb) * 256 + 128 * sb;
#pragma unroll 4
    for (int it = 0; it < 16; ++it) {
      const int row = 8 * it + warp;
      reinterpret_cast<float4*>(out + (long long)row * 256)[lane] = st[row * 32 + (lane ^ (row & 7))];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace

// ===========================================================================
// Host side
// ===========================================================================
bool split_supported(int x_dtype, int y_dtype, int P, int N, int cs) {
  return x_dtype == SSD_F32 && y_dtype == SSD_F32 && P == 64 && N == 128 && cs == 256;
}

cudaError_t launch_split_b(const LaunchCtx& c, const float* B, void* Bs) {
  split_b_kernel<<<dim3(4u, (unsigned)c.G, (unsigned)c.nchunks_max), kSplitThreads, 0, c.stream>>>(
      B, static_cast<uint8_t*>(Bs), c.cm, c.G);
  return cudaGetLastError();
}

cudaError_t launch_split_chunk_state(const LaunchCtx& c, const float* u, const void* Bs, const float* dt,
                                     const float* cum, float* states, int mode) {
  cudaError_t e = cudaFuncSetAttribute(split_chunk_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSsSmem);
  if (e != cudaSuccess) return e;
  split_chunk_state_kernel<<<dim3((unsigned)c.H, (unsigned)c.nchunks_max), kSplitThreads, kSsSmem, c.stream>>>(
      u, static_cast<const uint8_t*>(Bs), dt, cum, states, c.cm, c.H, c.G, mode);
  return cudaGetLastError();
}

cudaError_t launch_split_bmm(const LaunchCtx& c, const float* B, const float* C, void* CBs, void* Cs) {
  cudaError_t e =
      cudaFuncSetAttribute(split_bmm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBmSmem);
  if (e != cudaSuccess) return e;
  split_bmm_kernel<<<dim3(3u, (unsigned)c.G, (unsigned)c.nchunks_max), kSplitThreads, kBmSmem, c.stream>>>(
      B, C, static_cast<uint8_t*>(CBs), static_cast<uint8_t*>(Cs), c.cm, c.G);
  return cudaGetLastError();
}

cudaError_t launch_split_chunk_scan(const LaunchCtx& c, const float* u, const float* dt, const float* cum,
                                    const void* Cs, const float* prev, const void* CBs, const float* D,
                                    const float* z, float* y) {
  cudaError_t e = cudaFuncSetAttribute(split_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kScSmem);
  if (e != cudaSuccess) return e;
  split_chunk_scan_kernel<<<dim3(2u, (unsigned)c.H, (unsigned)c.nchunks_max), kScThreads, kScSmem, c.stream>>>(
      u, dt, cum, static_cast<const uint8_t*>(Cs), prev, static_cast<const uint8_t*>(CBs), D, z, y, c.cm, c.H,
      c.G);
  return cudaGetLastError();
}

size_t split_operand_bytes_per_chunk_group() { return (size_t)(6 + 4 + 4) * kSplitTile; }

template <int MODE>
static cudaError_t split_state_grad_mode(const LaunchCtx& c, const float* u, const float* B, const float* C,
                                        const float* y_grad, const float* dt, const float* cum, const float* prev,
                                        const float* hg, float* accS, float* B_grad, float* C_grad, float* gC) {
  auto kern = split_state_grad_kernel<MODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SgCfg<MODE>::kSmem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(2u, (unsigned)c.H, (unsigned)c.nchunks_max), kSplitThreads, SgCfg<MODE>::kSmem, c.stream>>>(
      u, B, C, y_grad, dt, cum, prev, hg, accS, B_grad, C_grad, gC, c.cm, c.H, c.G);
  return cudaGetLastError();
}

cudaError_t launch_split_state_grad(const LaunchCtx& c, const float* u, const float* B, const float* C,
                                    const float* y_grad, const float* dt, const float* cum, const float* prev,
                                    const float* hg, float* accS, float* B_grad, float* C_grad, float* gC) {
  cudaError_t e;
  if ((e = split_state_grad_mode<0>(c, u, B, C, y_grad, dt, cum, prev, hg, accS, B_grad, C_grad, gC)) ||
      (e = split_state_grad_mode<1>(c, u, B, C, y_grad, dt, cum, prev, hg, accS, B_grad, C_grad, gC)))
    return e;
  return split_state_grad_mode<2>(c, u, B, C, y_grad, dt, cum, prev, hg, accS, B_grad, C_grad, gC);
}

cudaError_t launch_split_bwd_accy(const LaunchCtx& c, const float* CB, const float* y_grad, const float* cum,
                                  float* accY) {
  cudaError_t e = cudaFuncSetAttribute(split_bwd_accy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kAySmem);
  if (e != cudaSuccess) return e;
  split_bwd_accy_kernel<<<dim3(2u, (unsigned)c.H, (unsigned)c.nchunks_max), kSplitThreads, kAySmem, c.stream>>>(
      CB, y_grad, cum, accY, c.cm, c.H, c.G);
  return cudaGetLastError();
}

cudaError_t launch_split_bwd_g(const LaunchCtx& c, const float* u, const float* y_grad, float* G) {
  cudaError_t e =
      cudaFuncSetAttribute(split_bwd_g_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBgSmem);
  if (e != cudaSuccess) return e;
  split_bwd_g_kernel<<<dim3(3u, (unsigned)c.H, (unsigned)c.nchunks_max), kSplitThreads, kBgSmem, c.stream>>>(
      u, y_grad, G, c.cm, c.H);
  return cudaGetLastError();
}

SSDB200_DEFINE_ERROR_FETCH(fetch_error_split)

}  // namespace ssdb200
