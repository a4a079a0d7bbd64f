// ssd_tc.cu - tensor-core (tcgen05 + TMA) chunk_state and chunk_scan for 16-bit
// inputs with headdim 64, dstate 128, chunk 256.
//
// chunk_state (ssd_scan/forward_kernel.py:107-185), one CTA per (head, chunk):
//   S^T[n, p] = sum_l B[l, n] * (x[l, p] * w_l),  w_l = exp(min(cum_last - cum_l, 0)) * dt_l
//   M = 128 (dstate), N = 64 (headdim), K = 256 tokens, both operands MN-major
//   (token rows of 128 B as TMA lands them); x is scaled by w_l in shared memory.
//
// chunk_scan (ssd_scan/forward_kernel.py:350-455 with bmm_chunk :270-328 fused),
// one CTA per (128-row half of a chunk, head, chunk):
//   MMA1  CB[l, s]   = C[l, :] . B[s, :]            M 128, N 128|256, K 128 (K-major)
//   CB -> registers: M[l, s] = CB * exp(min(cum_l - cum_s, 0)) * dt_s  (s <= l, s < lim)
//         -> bf16/fp16, written back over the B tile in the K-major layout
//   MMA3  Yoff[l, p] = C[l, :] . prev[p, :]         M 128, N 64, K 128 (K-major)
//   MMA2  Yin[l, p]  = sum_s M[l, s] x[s, p]         M 128, N 64, K 128|256 (x MN-major)
//   y = exp(cum_l) * Yoff + Yin (+ D x) (* silu z)
//
// All shared-memory tiles use the 128-byte swizzle; TMEM accumulators are fp32.
// Every mbarrier wait is bounded (sm100::mbar_wait) and a kernel that gives up
// records a site code in the error flag and returns after releasing TMEM.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace ssdb200 {

using namespace sm100;

enum : unsigned int {
  kSiteStateTma = 0x101,
  kSiteStateMma = 0x102,
  kSiteScanTma = 0x201,
  kSiteScanMma1 = 0x202,
  kSiteScanMma2 = 0x203,
};

template <bool BF16> struct T16Of;
template <> struct T16Of<true> { using type = __nv_bfloat16; };
template <> struct T16Of<false> { using type = __half; };

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ---------------------------------------------------------------------------
// chunk_state
// ---------------------------------------------------------------------------
constexpr int kStateSmem = 65536 + 32768 + 1024 + 64 + 1024;

template <bool BF16>
__global__ void __launch_bounds__(128, 1) tc_chunk_state_kernel(const __grid_constant__ CUtensorMap tm_x,
                                                                const __grid_constant__ CUtensorMap tm_b,
                                                                const float* __restrict__ dt,
                                                                const float* __restrict__ cum,
                                                                float* __restrict__ states, ChunkMap cm, int H,
                                                                int hpg) {
  using T16 = typename T16Of<BF16>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB = smem;            // 2 x (256 rows x 128 B): dstate halves
  uint8_t* sX = smem + 65536;    // 256 rows x 128 B
  float* sW = reinterpret_cast<float*>(smem + 98304);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 98304 + 1024);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);

  const int h = blockIdx.x, k = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int g = h / hpg;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bar_tma = smem_u32(&bars[0]), bar_mma = smem_u32(&bars[1]);

  if (tid == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_b);
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (tid == 0) {
    mbar_expect_tx(bar_tma, 3u * 32768u);
    const int t0 = (int)ci.tok0;
    tma_load_3d(smem_u32(sX), &tm_x, 0, h, t0, bar_tma);
    tma_load_3d(smem_u32(sB), &tm_b, 0, g, t0, bar_tma);
    tma_load_3d(smem_u32(sB + 32768), &tm_b, 64, g, t0, bar_tma);
  }
  const float* dtk = dt + ((long long)k * H + h) * 256;
  const float* cmk = cum + ((long long)k * H + h) * 256;
  const float clast = cmk[255];
  for (int l = tid; l < 256; l += 128) {
    float w = 0.f;
    if (l < ci.lim) w = __expf(fminf(clast - cmk[l], 0.f)) * dtk[l];
    sW[l] = w;
  }
  __syncthreads();
  bool tma_ok = mbar_wait(bar_tma, 0, kSiteStateTma);
  if (tma_ok) {
    // x rows scaled by w_l in place; rows past `lim` become exact zeros.
    for (int q = tid; q < 2048; q += 128) {
      uint4* pch = reinterpret_cast<uint4*>(sX + q * 16);
      const int l = q >> 3;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (l < ci.lim) {
        const float w = sW[l];
        uint4 a = *pch;
        float2 f;
        f = unpack2<T16>(a.x); v.x = pack2<T16>(f.x * w, f.y * w);
        f = unpack2<T16>(a.y); v.y = pack2<T16>(f.x * w, f.y * w);
        f = unpack2<T16>(a.z); v.z = pack2<T16>(f.x * w, f.y * w);
        f = unpack2<T16>(a.w); v.w = pack2<T16>(f.x * w, f.y * w);
      }
      *pch = v;
    }
  }
  fence_proxy_async_smem();
  const bool ok = __syncthreads_and(tma_ok) != 0;
  if (ok && tid == 0) {
    tc_fence_after();
    const uint32_t idesc = idesc_f16(128, 64, BF16, /*a_mn=*/true, /*b_mn=*/true);
    const uint32_t a0 = smem_u32(sB), b0 = smem_u32(sX);
#pragma unroll
    for (int ks = 0; ks < 16; ++ks) {
      const uint64_t ad = sdesc_sw128(a0 + ks * 2048, 32768, 1024);
      const uint64_t bd = sdesc_sw128(b0 + ks * 2048, 16, 1024);
      umma_f16(tmem, ad, bd, idesc, ks > 0 ? 1u : 0u);
    }
    umma_commit(bar_mma);
  }
  __syncwarp();
  bool mma_ok = false;
  if (ok) mma_ok = mbar_wait(bar_mma, 0, kSiteStateMma);
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
    // Give in-flight copies / MMAs a last bounded chance to land before exit.
    if (!tma_ok) mbar_wait(bar_tma, 0, kSiteStateTma);
    if (ok && !mma_ok) mbar_wait(bar_mma, 0, kSiteStateMma);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

// ---------------------------------------------------------------------------
// chunk_scan (+ bmm_chunk)
// ---------------------------------------------------------------------------
constexpr int kScanSmem = 32768 + 65536 + 32768 + 16384 + 2048 + 64 + 1024;

template <bool BF16, typename YT>
__global__ void __launch_bounds__(128, 1) tc_chunk_scan_kernel(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_c,
    const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_h,
    const float* __restrict__ dt, const float* __restrict__ cum, const float* __restrict__ D,
    const typename T16Of<BF16>::type* __restrict__ z, YT* __restrict__ y, ChunkMap cm, int H, int hpg) {
  using T16 = typename T16Of<BF16>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sC = smem;              // 2 x (128 rows x 128 B): dstate halves of C rows [128m, 128m+128)
  uint8_t* sB = smem + 32768;      // 2 x (S rows x 128 B): dstate halves of B rows [0, S); later M tiles
  uint8_t* sX = smem + 98304;      // S rows x 128 B: x rows [0, S)
  uint8_t* sH = smem + 131072;     // 2 x (64 rows x 128 B): dstate halves of prev[p, :]
  float* sDt = reinterpret_cast<float*>(smem + 147456);
  float* sCum = sDt + 256;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 147456 + 2048);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 3);

  const int m = blockIdx.x & 1, h = blockIdx.x >> 1, k = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int lbase = 128 * m;
  if (lbase >= ci.lim) return;  // no token of this half belongs to the row
  const int S = 128 * (m + 1);
  const int g = h / hpg;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bar_tma = smem_u32(&bars[0]), bar_m1 = smem_u32(&bars[1]), bar_m2 = smem_u32(&bars[2]);

  if (tid == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_c);
    prefetch_tmap(&tm_b);
    prefetch_tmap(&tm_h);
    mbar_init(bar_tma, 1);
    mbar_init(bar_m1, 1);
    mbar_init(bar_m2, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (tid == 0) {
    const uint32_t bytes = 32768u + (uint32_t)S * 256u + (uint32_t)S * 128u + 16384u;
    mbar_expect_tx(bar_tma, bytes);
    const int t0 = (int)ci.tok0;
    tma_load_3d(smem_u32(sC), &tm_c, 0, g, t0 + lbase, bar_tma);
    tma_load_3d(smem_u32(sC + 16384), &tm_c, 64, g, t0 + lbase, bar_tma);
    for (int rb = 0; rb <= m; ++rb) {
      tma_load_3d(smem_u32(sB + rb * 16384), &tm_b, 0, g, t0 + 128 * rb, bar_tma);
      tma_load_3d(smem_u32(sB + S * 128 + rb * 16384), &tm_b, 64, g, t0 + 128 * rb, bar_tma);
      tma_load_3d(smem_u32(sX + rb * 16384), &tm_x, 0, h, t0 + 128 * rb, bar_tma);
    }
    tma_load_3d(smem_u32(sH), &tm_h, 0, 0, k * H + h, bar_tma);
    tma_load_3d(smem_u32(sH + 8192), &tm_h, 64, 0, k * H + h, bar_tma);
  }
  {
    const float* dtk = dt + ((long long)k * H + h) * 256;
    const float* cmk = cum + ((long long)k * H + h) * 256;
    for (int i = tid; i < 256; i += 128) {
      sDt[i] = dtk[i];
      sCum[i] = cmk[i];
    }
  }
  __syncthreads();
  const bool tma_ok = mbar_wait(bar_tma, 0, kSiteScanTma);
  const bool ok0 = __syncthreads_and(tma_ok) != 0;

  if (ok0 && tid == 0) {
    tc_fence_after();
    const uint32_t id1 = idesc_f16(128, S, BF16, false, false);
    const uint32_t c0 = smem_u32(sC), b0 = smem_u32(sB);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t j = ks >> 2, kk = (ks & 3) * 32;
      const uint64_t ad = sdesc_sw128(c0 + j * 16384 + kk, 16, 1024);
      const uint64_t bd = sdesc_sw128(b0 + j * (uint32_t)S * 128 + kk, 16, 1024);
      umma_f16(tmem, ad, bd, id1, ks > 0 ? 1u : 0u);
    }
    umma_commit(bar_m1);
  }
  __syncwarp();
  bool m1_ok = false;
  if (ok0) m1_ok = mbar_wait(bar_m1, 0, kSiteScanMma1);
  tc_fence_after();
  const bool ok1 = ok0 && (__syncthreads_and(m1_ok) != 0);

  const int r = warp * 32 + lane;  // row inside this half
  const int l = lbase + r;         // row inside the chunk
  const float cl = sCum[l];
  if (ok1) {
    // x rows past `lim` -> exact zeros, so they cannot leak into Yin.
    for (int q = tid; q < S * 8; q += 128) {
      const int s = q >> 3;
      if (s >= ci.lim) *reinterpret_cast<uint4*>(sX + q * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
    const int warp_lmax = lbase + warp * 32 + 31;
    for (int cb = 0; cb < S / 32; ++cb) {
      const int s0 = cb * 32;
      uint32_t v[32];
      const bool any = s0 <= warp_lmax;  // warp-uniform
      if (any) {
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + s0, v);
        tmem_wait_ld();
      }
      uint32_t pk[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int sa = s0 + 2 * jj, sb2 = sa + 1;
        float a = 0.f, b = 0.f;
        if (any && sa <= l && sa < ci.lim) a = __uint_as_float(v[2 * jj]) * __expf(fminf(cl - sCum[sa], 0.f)) * sDt[sa];
        if (any && sb2 <= l && sb2 < ci.lim) b = __uint_as_float(v[2 * jj + 1]) * __expf(fminf(cl - sCum[sb2], 0.f)) * sDt[sb2];
        pk[jj] = pack2<T16>(a, b);
      }
      uint8_t* base = sB + (s0 >> 6) * 16384;
      const uint32_t c16 = (s0 & 63) >> 3;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(base + sw128_off(r, c16 + q)) =
            make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  const bool ok2 = ok1 && (__syncthreads_and(ok1) != 0);
  if (ok2 && tid == 0) {
    tc_fence_after();
    const uint32_t c0 = smem_u32(sC), h0 = smem_u32(sH), m0 = smem_u32(sB), x0 = smem_u32(sX);
    const uint32_t id3 = idesc_f16(128, 64, BF16, false, false);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t j = ks >> 2, kk = (ks & 3) * 32;
      const uint64_t ad = sdesc_sw128(c0 + j * 16384 + kk, 16, 1024);
      const uint64_t bd = sdesc_sw128(h0 + j * 8192 + kk, 16, 1024);
      umma_f16(tmem, ad, bd, id3, ks > 0 ? 1u : 0u);
    }
    const uint32_t id2 = idesc_f16(128, 64, BF16, false, true);
    for (int ks = 0; ks < S / 16; ++ks) {
      const uint32_t sb = ks >> 2, kk = (ks & 3) * 32;
      const uint64_t ad = sdesc_sw128(m0 + sb * 16384 + kk, 16, 1024);
      const uint64_t bd = sdesc_sw128(x0 + ks * 2048, 16, 1024);
      umma_f16(tmem + 64, ad, bd, id2, ks > 0 ? 1u : 0u);
    }
    umma_commit(bar_m2);
  }
  __syncwarp();
  bool m2_ok = false;
  if (ok2) m2_ok = mbar_wait(bar_m2, 0, kSiteScanMma2);
  tc_fence_after();
  const bool ok3 = ok2 && (__syncthreads_and(m2_ok) != 0);
  if (ok3) {
    const float el = __expf(cl);
    const long long tok = ci.tok0 + l;
    const bool valid = l < ci.lim;
    const long long yrow = (tok * H + h) * 64;
#pragma unroll
    for (int pc = 0; pc < 2; ++pc) {
      uint32_t ro[32], ri[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + pc * 32, ro);
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 64 + pc * 32, ri);
      tmem_wait_ld();
      if (valid) {
        float o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = fmaf(el, __uint_as_float(ro[j]), __uint_as_float(ri[j]));
        if (D) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 xv = *reinterpret_cast<const uint4*>(sX + sw128_off(l, pc * 4 + q));
            const uint32_t w4[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = unpack2<T16>(w4[e]);
              const int p = pc * 32 + q * 8 + 2 * e;
              o[q * 8 + 2 * e] = fmaf(D[h * 64 + p], f.x, o[q * 8 + 2 * e]);
              o[q * 8 + 2 * e + 1] = fmaf(D[h * 64 + p + 1], f.y, o[q * 8 + 2 * e + 1]);
            }
          }
        }
        if (z) {
          const uint4* zp = reinterpret_cast<const uint4*>(z + yrow + pc * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 zv = zp[q];
            const uint32_t w4[4] = {zv.x, zv.y, zv.z, zv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = unpack2<T16>(w4[e]);
              o[q * 8 + 2 * e] *= silu(f.x);
              o[q * 8 + 2 * e + 1] *= silu(f.y);
            }
          }
        }
        if constexpr (sizeof(YT) == 4) {
          float4* yp = reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + yrow + pc * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) yp[q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        } else {
          uint4* yp = reinterpret_cast<uint4*>(y + yrow + pc * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            yp[q] = make_uint4(pack2<YT>(o[8 * q], o[8 * q + 1]), pack2<YT>(o[8 * q + 2], o[8 * q + 3]),
                               pack2<YT>(o[8 * q + 4], o[8 * q + 5]), pack2<YT>(o[8 * q + 6], o[8 * q + 7]));
        }
      }
    }
  }
  if (!ok3 && tid == 0) {
    if (!tma_ok) mbar_wait(bar_tma, 0, kSiteScanTma);
    if (ok0 && !m1_ok) mbar_wait(bar_m1, 0, kSiteScanMma1);
    if (ok2 && !m2_ok) mbar_wait(bar_m2, 0, kSiteScanMma2);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------------------
// Host side: tensor maps and launches
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 3-D map over a row-major tensor of 16-bit elements (d0 innermost), 128-byte swizzle.
static bool make_map_3d(CUtensorMap* map, const void* base, bool bf16, uint64_t d0, uint64_t d1, uint64_t d2,
                        uint32_t b0, uint32_t b1, uint32_t b2) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool tc_supported(int x_dtype, int P, int N, int cs) {
  return (x_dtype == SSD_BF16 || x_dtype == SSD_F16) && P == 64 && N == 128 && cs == 256;
}

cudaError_t launch_tc_chunk_state(const LaunchCtx& c, int x_dtype, const void* u, const void* B, const float* dt,
                                  const float* cum, float* states, int* tmap_status) {
  const bool bf16 = x_dtype == SSD_BF16;
  CUtensorMap mx, mb;
  if (!make_map_3d(&mx, u, bf16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 256) ||
      !make_map_3d(&mb, B, bf16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 256)) {
    *tmap_status = 1;
    return cudaErrorInvalidValue;
  }
  *tmap_status = 0;
  dim3 grid((unsigned)c.H, (unsigned)c.nchunks_max);
  const int hpg = c.H / c.G;
  if (bf16) {
    cudaFuncSetAttribute(tc_chunk_state_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStateSmem);
    tc_chunk_state_kernel<true><<<grid, 128, kStateSmem, c.stream>>>(mx, mb, dt, cum, states, c.cm, c.H, hpg);
  } else {
    cudaFuncSetAttribute(tc_chunk_state_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStateSmem);
    tc_chunk_state_kernel<false><<<grid, 128, kStateSmem, c.stream>>>(mx, mb, dt, cum, states, c.cm, c.H, hpg);
  }
  return cudaGetLastError();
}

template <bool BF16, typename YT>
static cudaError_t tc_scan_launch(const LaunchCtx& c, const CUtensorMap& mx, const CUtensorMap& mc,
                                  const CUtensorMap& mb, const CUtensorMap& mh, const float* dt, const float* cum,
                                  const float* D, const void* z, void* y) {
  auto kern = tc_chunk_scan_kernel<BF16, YT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kScanSmem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)(2 * c.H), (unsigned)c.nchunks_max);
  kern<<<grid, 128, kScanSmem, c.stream>>>(mx, mc, mb, mh, dt, cum, D,
                                           reinterpret_cast<const typename T16Of<BF16>::type*>(z),
                                           reinterpret_cast<YT*>(y), c.cm, c.H, c.H / c.G);
  return cudaGetLastError();
}

cudaError_t launch_tc_chunk_scan(const LaunchCtx& c, int x_dtype, int y_dtype, const void* u, const float* dt,
                                 const float* cum, const void* B, const void* C, const void* prev16,
                                 const float* D, const void* z, void* y, int* tmap_status) {
  const bool bf16 = x_dtype == SSD_BF16;
  CUtensorMap mx, mc, mb, mh;
  // prev16 holds the previous-chunk states in the input's 16-bit type, so every
  // MMA of the kernel has operands of one type.
  const uint64_t nch = (uint64_t)c.nchunks_max;
  if (!make_map_3d(&mx, u, bf16, 64, (uint64_t)c.H, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mc, C, bf16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mb, B, bf16, 128, (uint64_t)c.G, (uint64_t)c.T, 64, 1, 128) ||
      !make_map_3d(&mh, prev16, bf16, 128, 64, nch * (uint64_t)c.H, 64, 64, 1)) {
    *tmap_status = 1;
    return cudaErrorInvalidValue;
  }
  *tmap_status = 0;
  if (y_dtype == SSD_F32) {
    if (bf16) return tc_scan_launch<true, float>(c, mx, mc, mb, mh, dt, cum, D, z, y);
    return tc_scan_launch<false, float>(c, mx, mc, mb, mh, dt, cum, D, z, y);
  }
  if (y_dtype == x_dtype) {
    if (bf16) return tc_scan_launch<true, __nv_bfloat16>(c, mx, mc, mb, mh, dt, cum, D, z, y);
    return tc_scan_launch<false, __half>(c, mx, mc, mb, mh, dt, cum, D, z, y);
  }
  return cudaErrorInvalidValue;
}

SSDB200_DEFINE_ERROR_FETCH(fetch_error_tc)

}  // namespace ssdb200
