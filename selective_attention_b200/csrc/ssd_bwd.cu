// ssd_bwd.cu - SSD chunked-scan backward (triton_kernels/ssd_scan/backward.py:467-555).
//
// The reference recomputes the forward intermediates and runs nine kernels with
// fp32 intermediates in HBM. Here the same maths runs as six CUDA-core kernels
// (fp32 FFMA, operands staged in shared memory, register-tiled), with the work of
// several reference kernels merged where they share operands:
//   bwd_chunk_states   chunk states S (forward recompute) and the intra-chunk state
//                      gradient sum_l y_grad exp(cum) C, one pass over the chunk
//   bwd_state_pass     forward recurrence (S -> prev states, in place) and the
//                      reverse recurrence (state gradients, decay_last gradient,
//                      h_init gradient) in one kernel per (row, head, 1024 elements)
//   bwd_cb             CB = C B^T for the lower tiles of each chunk
//   bwd_state_grad     the state-side products: B h_grad^T (for u_grad), u h_grad
//                      (B_grad), y_grad prev (C_grad) and the C-side decay gradient
//   bwd_intra          the intra-chunk products: CB^T y_grad (u_grad), y_grad u^T
//                      (CB_grad), the intra-chunk and B-side decay gradients, and
//                      the dt transform's backward (delta_raw_grad, A / bias partials)
//   bwd_bmm            CB_grad^T C into B_grad and CB_grad B into C_grad
// Group sums over heads (B_grad, C_grad, CB_grad) are fp32 atomic adds in L2.
#include "common.cuh"
#include "kernels.h"

namespace ssdb200 {
namespace {

__device__ __forceinline__ float ld_any(const void* p, long long i, int dt) {
  if (dt == SSD_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == SSD_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ void st_any(void* p, long long i, int dt, float v) {
  if (dt == SSD_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dt == SSD_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__device__ __forceinline__ float comp(const float4& v, int q) {
  return q == 0 ? v.x : (q == 1 ? v.y : (q == 2 ? v.z : v.w));
}

__device__ __forceinline__ float dot4(const float4& a, const float4& b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

// Sum over the 16 lanes of a half warp (lanes sharing tid >> 4).
__device__ __forceinline__ float half_warp_sum(float v) {
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Exclusive prefix sum over a block of NW warps (one value per thread); `tmp` holds NW
// floats of shared memory. Also returns the block total.
template <int NW = 8>
__device__ __forceinline__ float block_excl_scan(float v, float* tmp, float& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  float before = 0.f, all = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const float t = tmp[w];
    if (w < warp) before += t;
    all += t;
  }
  __syncthreads();
  total = all;
  return before + x - v;
}

template <int NW = 8>
__device__ __forceinline__ float block_sum(float v, float* tmp) {
  float total;
  block_excl_scan<NW>(v, tmp, total);
  return total;
}

// 8 consecutive elements from element i (i % 8 == 0, 16-byte aligned) as fp32.
__device__ __forceinline__ void ld8(const void* p, long long i, int dt, float (&o)[8]) {
  if (dt == SSD_F32) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    const float4 a = __ldg(q), b = __ldg(q + 1);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  } else {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i));
    float2 f[4];
    if (dt == SSD_BF16) {
      f[0] = unpack2<__nv_bfloat16>(w.x); f[1] = unpack2<__nv_bfloat16>(w.y);
      f[2] = unpack2<__nv_bfloat16>(w.z); f[3] = unpack2<__nv_bfloat16>(w.w);
    } else {
      f[0] = unpack2<__half>(w.x); f[1] = unpack2<__half>(w.y);
      f[2] = unpack2<__half>(w.z); f[3] = unpack2<__half>(w.w);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      o[2 * e] = f[e].x;
      o[2 * e + 1] = f[e].y;
    }
  }
}

// 4 consecutive elements from element i (i % 4 == 0, aligned) as fp32.
__device__ __forceinline__ float4 ld4(const void* p, long long i, int dt) {
  if (dt == SSD_F32) return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i));
  const uint2 w = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p) + i));
  float2 a, b;
  if (dt == SSD_BF16) {
    a = unpack2<__nv_bfloat16>(w.x);
    b = unpack2<__nv_bfloat16>(w.y);
  } else {
    a = unpack2<__half>(w.x);
    b = unpack2<__half>(w.y);
  }
  return make_float4(a.x, a.y, b.x, b.y);
}

// Column of token r in row `row` of a transposed ([feature][token]) tile: 4-token groups
// XOR-swizzled by the row's 8-row block, so the staging stores (lanes 8 rows apart) spread
// over the banks; a 4-token group stays one aligned float4 (tiles of <= 64 tokens).
__device__ __forceinline__ int tok_col(int row, int r) { return r ^ (((row >> 3) & 7) << 2); }

// Stage R token rows of a token-major tensor into shared memory as fp32: row r is
// token tok0 + t0 + r, its columns [0, W) start at element (tok0 + t0 + r) * rs + co
// (W, rs, co multiples of 8). Rows with t0 + r >= lim are zero; each value is scaled by
// scale[t0 + r] when `scale` is given. COLS=false writes dst[r * ldd + c], COLS=true
// dst[c * ldd + tok_col(c, r)] (R <= 64). All of a thread's loads (V 16-byte vectors,
// R * W / 8 <= NT V) are
// issued before its stores, so the tile costs one memory latency.
template <int V, bool COLS, int NT = 256>
__device__ __forceinline__ void stage(float* dst, int ldd, const void* src, int dt, long long tok0, int t0, int R,
                                      long long rs, long long co, int W, int lim, const float* scale) {
  const int vpr = W >> 3, nv = R * vpr;
  float v[V][8];
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int vi = threadIdx.x + NT * j;
    const int r = vi / vpr, c = (vi - r * vpr) << 3;
    if (vi < nv && t0 + r < lim) {
      ld8(src, (tok0 + t0 + r) * rs + co + c, dt, v[j]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = 0.f;
    }
  }
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int vi = threadIdx.x + NT * j;
    if (vi >= nv) continue;
    const int r = vi / vpr, c = (vi - r * vpr) << 3;
    const float sc = scale ? scale[t0 + r] : 1.f;
    if (COLS) {
#pragma unroll
      for (int e = 0; e < 8; ++e) dst[(c + e) * ldd + tok_col(c + e, r)] = v[j][e] * sc;
    } else {
      *reinterpret_cast<float4*>(dst + r * ldd + c) =
          make_float4(v[j][0] * sc, v[j][1] * sc, v[j][2] * sc, v[j][3] * sc);
      *reinterpret_cast<float4*>(dst + r * ldd + c + 4) =
          make_float4(v[j][4] * sc, v[j][5] * sc, v[j][6] * sc, v[j][7] * sc);
    }
  }
}

constexpr int kLT = 32;        // token rows per tile
constexpr int kPmax = 64, kNmax = 128, kCSmax = 256;
constexpr int kLDT = kLT + 4;  // [feature][token] tiles
constexpr int kLDN = kNmax + 4;
constexpr int kLDP = kPmax + 4;

// ===========================================================================
// bwd_chunk_states: per (chunk, head), one product per CTA (blockIdx.z):
//   z = 0: S[p,n]  = sum_{l<len} u[l,p] exp(min(cum_last - cum_l, 0)) dt_l B[l,n]
//          (the chunk_state forward recomputed, backward.py:487; dt = 0 past len)
//   z = 1: HG[p,n] = sum_{l<len} y_grad[l,p] exp(cum_l) C[l,n]   (backward_kernel.py:23-93)
// 64-token tiles staged transposed ([feature][token]); thread (tp, tn) owns
// p = tp + 16 i (i < 4), n = tn + 16 j (j < 8).
// ===========================================================================
__global__ void __launch_bounds__(256, 2) bwd_chunk_states_kernel(
    const void* __restrict__ u, const void* __restrict__ Bm, const void* __restrict__ Cm,
    const void* __restrict__ yg, const float* __restrict__ dt, const float* __restrict__ cum,
    float* __restrict__ states, float* __restrict__ hg, ChunkMap cm, int H, int G, int P, int N, int xdt,
    int ydt) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int h = blockIdx.x, k = blockIdx.y, which = blockIdx.z, tid = threadIdx.x;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int cs = cm.cs, g = h / (H / G), vl = ci.vlim;
  constexpr int TT = 64, LD = TT + 4;  // 64-token tiles, [feature][token]
  float* aT = sm;                   // [kPmax][LD]
  float* bT = aT + kPmax * LD;      // [kNmax][LD]
  float* scl = bT + kNmax * LD;     // [kCSmax]
  const long long kh = (long long)k * H + h;
  const float clast = cum[kh * cs + cs - 1];
  for (int i = tid; i < kCSmax; i += 256) {
    const float c = i < vl ? cum[kh * cs + i] : 0.f;
    scl[i] = i < vl ? (which == 0 ? expf(fminf(clast - c, 0.f)) * dt[kh * cs + i] : expf(c)) : 0.f;
  }
  const void* asrc = which == 0 ? u : yg;
  const void* bsrc = which == 0 ? Bm : Cm;
  const int adt = which == 0 ? xdt : ydt;
  const int tp = tid >> 4, tn = tid & 15;
  int pr[4], nr[8], ps[4], ns[8];  // row offsets and their token swizzles (tok_col)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = min(tp + 16 * i, P - 1);
    pr[i] = r * LD;
    ps[i] = tok_col(r, 0);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int r = min(tn + 16 * j, N - 1);
    nr[j] = r * LD;
    ns[j] = tok_col(r, 0);
  }
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  for (int l0 = 0; l0 < vl; l0 += TT) {
    __syncthreads();
    stage<2, true>(aT, LD, asrc, adt, ci.tok0, l0, TT, (long long)H * P, (long long)h * P, P, vl, scl);
    stage<4, true>(bT, LD, bsrc, xdt, ci.tok0, l0, TT, (long long)G * N, (long long)g * N, N, vl, nullptr);
    __syncthreads();
#pragma unroll 2
    for (int l = 0; l < TT; l += 4) {
      float4 a[4], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = lds4(aT + pr[i] + (l ^ ps[i]));
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = lds4(bT + nr[j] + (l ^ ns[j]));
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = dot4(a[i], b[j], acc[i][j]);
    }
  }
  float* out = (which == 0 ? states : hg) + kh * P * N;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = tp + 16 * i;
    if (p >= P) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = tn + 16 * j;
      if (n < N) out[p * N + n] = acc[i][j];
    }
  }
}

// ===========================================================================
// bwd_state_pass: per (row, head, 1024 state elements), 4 elements per thread.
// Forward (forward_kernel.py:244-249): states[c] <- prev; prev = exp(cl_c) prev + S_c.
// Reverse (backward_kernel.py:144-157), g = gradient of the state leaving chunk c:
//   dlast_c = sum(prev_c * g) * exp(cl_c)   (per-warp partials, summed by bwd_intra)
//   hg[c] <- g;  g = exp(cl_c) g + hg_intra[c];   h_init_grad = g after chunk 0.
// ===========================================================================
// With prev16 / hg16 set (the tensor-core path), the chunk-initial states and the state
// gradients are also written rounded to the inputs' 16-bit type (x16: SSD_BF16 or SSD_F16),
// as the operands the state-side products load by TMA.
__device__ __forceinline__ void store4_16(uint16_t* dst, float4 v, int x16) {
  const uint2 w = x16 == SSD_BF16 ? make_uint2(pack2<__nv_bfloat16>(v.x, v.y), pack2<__nv_bfloat16>(v.z, v.w))
                                  : make_uint2(pack2<__half>(v.x, v.y), pack2<__half>(v.z, v.w));
  *reinterpret_cast<uint2*>(dst) = w;
}

__global__ void __launch_bounds__(256) bwd_state_pass_kernel(
    float* __restrict__ states, float* __restrict__ hg, const float* __restrict__ cum,
    const float* __restrict__ h_init, const float* __restrict__ h_last_grad, float* __restrict__ h_init_grad,
    float* __restrict__ dl_part, ChunkMap cm, int H, int PN, uint16_t* __restrict__ prev16,
    uint16_t* __restrict__ hg16, int x16) {
  const int row = blockIdx.z, h = blockIdx.y;
  const int nparts = gridDim.x * 8, part = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int e0 = (blockIdx.x * 256 + threadIdx.x) * 4;
  const bool act = e0 < PN;
  int first, count;
  if (cm.packed) {
    const int2 r = cm.rows[row];
    first = r.x;
    count = r.y;
  } else {
    first = row * cm.nc;
    count = cm.nc;
  }
  const int cs = cm.cs;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  auto at = [&](float* base, int c) { return base + ((long long)(first + c) * H + h) * PN + e0; };
  auto scale = [&](int c) { return expf(cum[((long long)(first + c) * H + h) * cs + cs - 1]); };
  const long long hoff = ((long long)row * H + h) * PN + e0;
  float4 prev = (h_init && act) ? *reinterpret_cast<const float4*>(h_init + hoff) : zero;
  float4 nxt = (act && count > 0) ? *reinterpret_cast<const float4*>(at(states, 0)) : zero;
  for (int c = 0; c < count; ++c) {
    const float4 sv = nxt;
    if (act && c + 1 < count) nxt = *reinterpret_cast<const float4*>(at(states, c + 1));
    const float sc = scale(c);
    if (act) {
      *reinterpret_cast<float4*>(at(states, c)) = prev;
      if (prev16) store4_16(prev16 + (at(states, c) - states), prev, x16);
    }
    prev.x = fmaf(sc, prev.x, sv.x);
    prev.y = fmaf(sc, prev.y, sv.y);
    prev.z = fmaf(sc, prev.z, sv.z);
    prev.w = fmaf(sc, prev.w, sv.w);
  }
  float4 gr = (h_last_grad && act) ? *reinterpret_cast<const float4*>(h_last_grad + hoff) : zero;
  float4 pv_n = zero, hg_n = zero;
  if (act && count > 0) {
    pv_n = *reinterpret_cast<const float4*>(at(states, count - 1));
    hg_n = *reinterpret_cast<const float4*>(at(hg, count - 1));
  }
  for (int c = count - 1; c >= 0; --c) {
    const float4 pv = pv_n, hgi = hg_n;
    if (act && c > 0) {
      pv_n = *reinterpret_cast<const float4*>(at(states, c - 1));
      hg_n = *reinterpret_cast<const float4*>(at(hg, c - 1));
    }
    const float sc = scale(c);
    float d = act ? dot4(pv, gr, 0.f) : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
    if ((threadIdx.x & 31) == 0) dl_part[((long long)(first + c) * H + h) * nparts + part] = d * sc;
    if (act) {
      *reinterpret_cast<float4*>(at(hg, c)) = gr;
      if (hg16) store4_16(hg16 + (at(hg, c) - hg), gr, x16);
    }
    gr.x = fmaf(sc, gr.x, hgi.x);
    gr.y = fmaf(sc, gr.y, hgi.y);
    gr.z = fmaf(sc, gr.z, hgi.z);
    gr.w = fmaf(sc, gr.w, hgi.w);
  }
  if (h_init_grad && act) *reinterpret_cast<float4*>(h_init_grad + hoff) = gr;
}

// ===========================================================================
// bwd_cb: CB[l,s] = sum_n C[l,n] B[s,n] (forward_kernel.py:270-328) for the lower
// 64x64 tiles of each chunk; rows / columns past seq_len are zero.
// ===========================================================================
__global__ void __launch_bounds__(256) bwd_cb_kernel(const void* __restrict__ Bm, const void* __restrict__ Cm,
                                                     float* __restrict__ CB, ChunkMap cm, int G, int N, int xdt) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int k = blockIdx.z, g = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  int t = blockIdx.x, ti = 0;
  while (t > ti) {
    t -= ti + 1;
    ++ti;
  }
  const int tj = t, cs = cm.cs, l0 = ti * 64, s0 = tj * 64, tid = threadIdx.x;
  float* cS = sm;               // [64][kLDN]
  float* bS = sm + 64 * kLDN;   // [64][kLDN]
  stage<4, false>(cS, kLDN, Cm, xdt, ci.tok0, l0, 64, (long long)G * N, (long long)g * N, N, ci.lim, nullptr);
  stage<4, false>(bS, kLDN, Bm, xdt, ci.tok0, s0, 64, (long long)G * N, (long long)g * N, N, ci.lim, nullptr);
  __syncthreads();
  const int ty = tid >> 4, tx = tid & 15;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int n = 0; n < N; n += 4) {
    float4 a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = lds4(cS + (ty + 16 * i) * kLDN + n);
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = lds4(bS + (tx + 16 * j) * kLDN + n);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = dot4(a[i], b[j], acc[i][j]);
  }
  float* out = CB + ((long long)k * G + g) * cs * cs;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = l0 + ty + 16 * i;
    if (l >= cs) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = s0 + tx + 16 * j;
      if (s < cs) out[l * cs + s] = acc[i][j];
    }
  }
}

// ===========================================================================
// bwd_state_grad: per (chunk, head), 32-token row tiles. With scale_l =
// exp(min(cum_last - cum_l, 0)):
//   accS[l,p] = scale_l sum_n B[l,n] hg[p,n]             (backward_kernel.py:255-262)
//   B_grad[l,:] += scale_l dt_l sum_p u[l,p] hg[p,:]       (:402-415)
//   C_grad[l,:] += exp(cum_l) sum_p y_grad[l,p] prev[p,:]  (:522-533)
//   gC[l] = sum_n (that C_grad row) C[l,n]                 (:537-538)
// accS goes to a scratch buffer for bwd_intra; rows at or past `length` are zero.
// ===========================================================================
__global__ void __launch_bounds__(256, 2) bwd_state_grad_kernel(
    const void* __restrict__ u, const void* __restrict__ Bm, const void* __restrict__ Cm,
    const void* __restrict__ yg, const float* __restrict__ dt, const float* __restrict__ cum,
    const float* __restrict__ prev, const float* __restrict__ hg, float* __restrict__ accS_out,
    float* __restrict__ Bgrad, float* __restrict__ Cgrad, float* __restrict__ gC_out, ChunkMap cm, int H, int G,
    int P, int N, int xdt, int ydt) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int h = blockIdx.x, k = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int cs = cm.cs, g = h / (H / G), tid = threadIdx.x;
  float* hgS = sm;                  // [kPmax][kLDN]
  float* pvS = hgS + kPmax * kLDN;  // [kPmax][kLDN]
  float* bt = pvS + kPmax * kLDN;   // [kLT][kLDN]
  float* uw = bt + kLT * kLDN;      // [kLT][kLDP]
  float* ye = uw + kLT * kLDP;      // [kLT][kLDP]
  float* sS = ye + kLT * kLDP;      // [kCSmax] exp(min(cum_last - cum_l, 0))
  float* wS = sS + kCSmax;          // [kCSmax] sS * dt
  float* eS = wS + kCSmax;          // [kCSmax] exp(cum_l)
  const long long kh = (long long)k * H + h;
  const float* hgk = hg + kh * P * N;
  const float* pvk = prev + kh * P * N;
  const int vl = ci.vlim;
  {
    float4 ha[8], pa[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int idx = (tid + 256 * j) * 4;
      if (idx < P * N) {
        ha[j] = __ldg(reinterpret_cast<const float4*>(hgk + idx));
        pa[j] = __ldg(reinterpret_cast<const float4*>(pvk + idx));
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int idx = (tid + 256 * j) * 4;
      if (idx < P * N) {
        const int p = idx / N, n = idx - p * N;
        *reinterpret_cast<float4*>(hgS + p * kLDN + n) = ha[j];
        *reinterpret_cast<float4*>(pvS + p * kLDN + n) = pa[j];
      }
    }
  }
  const float clast = cum[kh * cs + cs - 1];
  for (int i = tid; i < cs; i += 256) {
    const float c = cum[kh * cs + i];
    const float sc = i < vl ? expf(fminf(clast - c, 0.f)) : 0.f;
    sS[i] = sc;
    wS[i] = sc * dt[kh * cs + i];
    eS[i] = i < vl ? expf(c) : 0.f;
  }
  const int tl = tid >> 4, tq = tid & 15;
  int prow[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) prow[j] = min(tq + 16 * j, P - 1) * kLDN;

  for (int l0 = 0; l0 < ci.lim; l0 += kLT) {
    __syncthreads();
    const long long rsB = (long long)G * N, coB = (long long)g * N, rsU = (long long)H * P, coU = (long long)h * P;
    stage<2, false>(bt, kLDN, Bm, xdt, ci.tok0, l0, kLT, rsB, coB, N, vl, nullptr);
    stage<1, false>(uw, kLDP, u, xdt, ci.tok0, l0, kLT, rsU, coU, P, vl, wS);
    stage<1, false>(ye, kLDP, yg, ydt, ci.tok0, l0, kLT, rsU, coU, P, vl, eS);
    __syncthreads();

    // accS: rows l = tl + 16 i, columns p = tq + 16 j
    float aS[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) aS[i][j] = 0.f;
    for (int n = 0; n < N; n += 4) {
      float4 a[2], b[4];
#pragma unroll
      for (int i = 0; i < 2; ++i) a[i] = lds4(bt + (tl + 16 * i) * kLDN + n);
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = lds4(hgS + prow[j] + n);
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) aS[i][j] = dot4(a[i], b[j], aS[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int l = l0 + tl + 16 * i;
      if (l >= cs) continue;
      const float sc = sS[l];
      float* o = accS_out + (kh * cs + l) * P;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int p = tq + 16 * j;
        if (p < P) o[p] = aS[i][j] * sc;
      }
    }

    // B_grad / C_grad rows: l = tl + 16 i, columns n = 4 tq + 64 jj + (0..3)
    float bA[2][8], cA[2][8];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) bA[i][j] = cA[i][j] = 0.f;
    for (int p = 0; p < P; p += 4) {
      float4 au[2], ay[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        au[i] = lds4(uw + (tl + 16 * i) * kLDP + p);
        ay[i] = lds4(ye + (tl + 16 * i) * kLDP + p);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float* hr = hgS + (p + q) * kLDN + 4 * tq;
        const float* vr = pvS + (p + q) * kLDN + 4 * tq;
        const float4 h0 = lds4(hr), h1 = lds4(hr + 64), v0 = lds4(vr), v1 = lds4(vr + 64);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float a = comp(au[i], q), y = comp(ay[i], q);
          bA[i][0] = fmaf(a, h0.x, bA[i][0]);
          bA[i][1] = fmaf(a, h0.y, bA[i][1]);
          bA[i][2] = fmaf(a, h0.z, bA[i][2]);
          bA[i][3] = fmaf(a, h0.w, bA[i][3]);
          bA[i][4] = fmaf(a, h1.x, bA[i][4]);
          bA[i][5] = fmaf(a, h1.y, bA[i][5]);
          bA[i][6] = fmaf(a, h1.z, bA[i][6]);
          bA[i][7] = fmaf(a, h1.w, bA[i][7]);
          cA[i][0] = fmaf(y, v0.x, cA[i][0]);
          cA[i][1] = fmaf(y, v0.y, cA[i][1]);
          cA[i][2] = fmaf(y, v0.z, cA[i][2]);
          cA[i][3] = fmaf(y, v0.w, cA[i][3]);
          cA[i][4] = fmaf(y, v1.x, cA[i][4]);
          cA[i][5] = fmaf(y, v1.y, cA[i][5]);
          cA[i][6] = fmaf(y, v1.z, cA[i][6]);
          cA[i][7] = fmaf(y, v1.w, cA[i][7]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int lr = tl + 16 * i, l = l0 + lr;
      float gsum = 0.f;
      if (l < vl) {
        const long long row = ((ci.tok0 + l) * G + g) * (long long)N;
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int n0 = 4 * tq + 64 * jj;
          if (n0 < N) {
            atomicAdd(reinterpret_cast<float4*>(Bgrad + row + n0),
                      make_float4(bA[i][4 * jj], bA[i][4 * jj + 1], bA[i][4 * jj + 2], bA[i][4 * jj + 3]));
            atomicAdd(reinterpret_cast<float4*>(Cgrad + row + n0),
                      make_float4(cA[i][4 * jj], cA[i][4 * jj + 1], cA[i][4 * jj + 2], cA[i][4 * jj + 3]));
            const float4 cr = ld4(Cm, row + n0, xdt);
            gsum = fmaf(cA[i][4 * jj], cr.x, gsum);
            gsum = fmaf(cA[i][4 * jj + 1], cr.y, gsum);
            gsum = fmaf(cA[i][4 * jj + 2], cr.z, gsum);
            gsum = fmaf(cA[i][4 * jj + 3], cr.w, gsum);
          }
        }
      }
      gsum = half_warp_sum(gsum);
      if (tq == 0 && l < cs) gC_out[kh * cs + l] = l < vl ? gsum : 0.f;
    }
  }
}

// dt backward per (chunk, head), one token t per thread, NT threads >= cs
// (backward_kernel.py:984-1039):
//   total = decay_intra + excl_cumsum(gB shifted) + rev_cumsum(gC) + dlast
//   delta_raw_grad = (total A + ddt), 0 where dt was clamped, * sigmoid(pre) (softplus)
// and the A / bias partials of the chunk. cols, rows, gBs, ddts: [cs] in shared or global
// memory; revc [kCSmax] and tmp [16] in shared memory.
template <int NT>
__device__ __forceinline__ void dt_backward(const float* cols, const float* rows, const float* gBs, const float* ddts,
                                            float* revc, float* tmp, const float* __restrict__ gC,
                                            const float* __restrict__ dl_part, int nsl, const void* __restrict__ delta_raw,
                                            const float* __restrict__ A, const float* __restrict__ delta_bias,
                                            void* __restrict__ draw_grad, float* __restrict__ A_part,
                                            float* __restrict__ bias_part, const ChunkInfo& ci, long long kh, int h,
                                            int H, int cs, int vl, int ddt_dtype, int use_sp, float dmin, float dmax) {
  const int tid = threadIdx.x;
  const int t = tid;
  float dlast = 0.f;
  for (int i = 0; i < nsl; ++i) dlast += dl_part[kh * nsl + i];
  float unused;
  const float xi = t < cs ? cols[t] - rows[t] : 0.f;
  const float intra = block_excl_scan<NT / 32>(xi, tmp, unused);
  const float xb = t < vl - 1 ? gBs[t] : 0.f;
  const float dB = block_excl_scan<NT / 32>(xb, tmp, unused);
  // sum_{m >= tr} gC_m: thread t scans element tr = cs-1-t, so threads before it hold m > tr
  const int tr = cs - 1 - t;
  const float xc = (tr >= 0 && tr < vl) ? gC[kh * cs + tr] : 0.f;
  const float exc = block_excl_scan<NT / 32>(xc, tmp, unused);
  if (tr >= 0) revc[tr] = exc + xc;
  __syncthreads();
  float aP = 0.f, bP = 0.f;
  if (t < ci.lim) {
    const long long tok = ci.tok0 + t;
    float gg = 0.f;
    if (t < vl) {
      const float total = intra + dB + revc[t] + dlast;
      const float pre = ld_any(delta_raw, tok * H + h, ddt_dtype) + (delta_bias ? delta_bias[h] : 0.f);
      const bool sp = use_sp && pre <= 20.0f;
      float d = sp ? logf(expf(pre) + 1.0f) : pre;
      const bool clamped = (d < dmin) || (d > dmax);
      d = fminf(fmaxf(d, dmin), dmax);
      gg = clamped ? 0.f : total * A[h] + ddts[t];
      if (sp) gg *= 1.0f / (1.0f + expf(-pre));
      aP = total * d;
      bP = gg;
    }
    st_any(draw_grad, tok * H + h, ddt_dtype, gg);
  }
  const float as = block_sum<NT / 32>(aP, tmp);
  const float bs = block_sum<NT / 32>(bP, tmp);
  if (tid == 0) {
    A_part[kh] = as;
    bias_part[kh] = bs;
  }
}

// ===========================================================================
// bwd_intra: per (chunk, head); u and y_grad of the whole chunk in shared memory.
//   accY[l,p] = sum_{l<=s<len} CB[s,l] exp(min(cum_s - cum_l, 0)) y_grad[s,p]   (:272-293)
//   acc = accS + accY;  u_grad = acc dt_l;  ddt[l] = sum_p acc u  (:296-314)
//   gB[l] = dt_l sum_p accS u  (= sum_n B_grad contribution * B, :417-421)
//   CB_grad[l,s] += (y_grad[l] . u[s]) dt_s exp(min(cum_l - cum_s, 0)), s <= l  (:632-659)
//   w[l,s] = CB_grad_h[l,s] CB[l,s] (s < l):  row sums and column sums give the
//   intra-chunk decay gradient decay[j] = sum_{m<j} (col_m - row_m)  (:847-895)
// then the dt backward (:984-1039):
//   total = decay_intra + excl_cumsum(gB shifted) + rev_cumsum(gC) + dlast
//   delta_raw_grad = (total A + ddt), 0 where dt was clamped, * sigmoid(pre) (softplus)
//   A / bias partials per (chunk, head).
// ===========================================================================
// Column of element (row, c) of the intra kernel's M tile: 4-column groups XOR-swizzled by
// the row's 4-row block, so the tile's transposed writes (lanes 4 rows apart) spread over
// the banks while each 4-column group stays one aligned float4 for the reads.
__device__ __forceinline__ int mt_col(int row, int c) { return c ^ (((row >> 2) & 7) << 2); }

constexpr int kIT = 512;         // bwd_intra threads
constexpr int kIR = 64;          // bwd_intra row tile
constexpr int kIB = 128;         // bwd_intra column block
constexpr int kLDB = kIB + 4;

__global__ void __launch_bounds__(kIT, 1) bwd_intra_kernel(
    const void* __restrict__ u, const void* __restrict__ yg, const void* __restrict__ delta_raw,
    const float* __restrict__ A, const float* __restrict__ delta_bias, const float* __restrict__ dt,
    const float* __restrict__ cum, const float* __restrict__ CB, const float* __restrict__ accS,
    const float* __restrict__ gC, const float* __restrict__ dl_part, int nsl,
    float* __restrict__ CBg,
    void* __restrict__ u_grad, void* __restrict__ draw_grad, float* __restrict__ A_part,
    float* __restrict__ bias_part, ChunkMap cm, int H, int G, int P, int xdt, int ydt, int ddt_dtype, int use_sp,
    float dmin, float dmax) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int h = blockIdx.x, k = blockIdx.y, tid = threadIdx.x;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) {
    if (tid == 0) {
      A_part[(long long)k * H + h] = 0.f;
      bias_part[(long long)k * H + h] = 0.f;
    }
    return;
  }
  const int cs = cm.cs, g = h / (H / G), vl = ci.vlim;
  float* uS = sm;                     // [kCSmax][kLDP]
  float* yS = uS + kCSmax * kLDP;     // [kCSmax][kLDP]
  float* Mt = yS + kCSmax * kLDP;     // [kIR][kLDB]: rows l of the tile, kIB columns s
  float* cbS = Mt + kIR * kLDB;       // [kIR][kLDB]: CB rows of the tile, kIB columns
  float* dts = cbS + kIR * kLDB;      // [kCSmax] each below
  float* cms = dts + kCSmax;
  float* rows = cms + kCSmax;
  float* cols = rows + kCSmax;
  float* ddts = cols + kCSmax;
  float* gBs = ddts + kCSmax;
  float* revc = gBs + kCSmax;
  float* tmp = revc + kCSmax;         // [16]
  const long long kh = (long long)k * H + h;
  const long long kg = ((long long)k * G + g) * cs * cs;
  stage<4, false, kIT>(uS, kLDP, u, xdt, ci.tok0, 0, cs, (long long)H * P, (long long)h * P, P, vl, nullptr);
  stage<4, false, kIT>(yS, kLDP, yg, ydt, ci.tok0, 0, cs, (long long)H * P, (long long)h * P, P, vl, nullptr);
  for (int i = tid; i < kCSmax; i += kIT) {
    dts[i] = i < cs ? dt[kh * cs + i] : 0.f;
    cms[i] = i < cs ? cum[kh * cs + i] : 0.f;
    rows[i] = cols[i] = ddts[i] = gBs[i] = 0.f;
  }
  __syncthreads();
  const int tl = tid >> 4, tq = tid & 15;  // rows l0 + tl + 32 i (i < 2)
  const int p0 = 4 * tq;
  const bool pvalid = p0 < P;

  for (int l0 = 0; l0 < ci.lim; l0 += kIR) {
    // accY: rows l = l0 + tl + 32 i, columns p0 .. p0 + 3
    float aY[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) aY[i][j] = 0.f;
    for (int s0 = l0; s0 < vl; s0 += kIB) {
      __syncthreads();
      {
        // CB rows s = s0 + c (c < kIB), columns l0 + r4 .. + 3: four 16-byte loads per thread
        float4 cb[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int vi = tid + kIT * j, c = vi >> 4, r4 = (vi & 15) * 4, s = s0 + c;
          cb[j] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (s < vl && l0 + r4 < cs)
            cb[j] = __ldg(reinterpret_cast<const float4*>(CB + kg + (long long)s * cs + l0 + r4));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int vi = tid + kIT * j, c = vi >> 4, r4 = (vi & 15) * 4, s = s0 + c;
          const float cs_ = s < cs ? cms[s] : 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int l = l0 + r4 + e;
            float v = 0.f;
            if (s >= l && s < vl && l < vl) v = comp(cb[j], e) * expf(fminf(cs_ - cms[l], 0.f));
            Mt[(r4 + e) * kLDB + mt_col(r4 + e, c)] = v;
          }
        }
      }
      __syncthreads();
      if (pvalid) {
        const int cend = min(kIB, cs - s0);  // yS rows stay inside the chunk
#pragma unroll 2
        for (int c = 0; c < cend; c += 4) {
          float4 a[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) a[i] = lds4(Mt + (tl + 32 * i) * kLDB + mt_col(tl + 32 * i, c));
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 y4 = lds4(yS + (s0 + c + q) * kLDP + p0);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const float m = comp(a[i], q);
              aY[i][0] = fmaf(m, y4.x, aY[i][0]);
              aY[i][1] = fmaf(m, y4.y, aY[i][1]);
              aY[i][2] = fmaf(m, y4.z, aY[i][2]);
              aY[i][3] = fmaf(m, y4.w, aY[i][3]);
            }
          }
        }
      }
    }
    // u_grad, ddt, gB for the tile rows
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int l = l0 + tl + 32 * i;
      float dpart = 0.f, bpart = 0.f;
      if (l < cs && pvalid) {
        float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (l < vl) s4 = *reinterpret_cast<const float4*>(accS + (kh * cs + l) * P + p0);
        const float4 acc = make_float4(s4.x + aY[i][0], s4.y + aY[i][1], s4.z + aY[i][2], s4.w + aY[i][3]);
        const float4 u4 = lds4(uS + l * kLDP + p0);
        dpart = dot4(acc, u4, 0.f);
        bpart = dot4(s4, u4, 0.f);
        if (l < ci.lim) {
          const float d = l < vl ? dts[l] : 0.f;
          const long long off = ((ci.tok0 + l) * H + h) * (long long)P + p0;
          st_any(u_grad, off, xdt, acc.x * d);
          st_any(u_grad, off + 1, xdt, acc.y * d);
          st_any(u_grad, off + 2, xdt, acc.z * d);
          st_any(u_grad, off + 3, xdt, acc.w * d);
        }
      }
      dpart = half_warp_sum(dpart);
      bpart = half_warp_sum(bpart);
      if (tq == 0 && l < cs) {
        ddts[l] = dpart;
        gBs[l] = bpart * dts[l];
      }
    }
    // CB_grad and the intra-chunk decay terms: rows l = l0 + tl + 32 i, columns
    // s = sb + tq + 16 j of kIB-wide column blocks left of the tile's end.
    float rs[2] = {0.f, 0.f};
    const int send = min(l0 + kIR, vl);
    for (int sb = 0; sb < send; sb += kIB) {
      __syncthreads();  // cbS of the previous block consumed
      {
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int vi = tid + kIT * j, r = vi >> 5, c4 = (vi & 31) * 4;
          v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (sb + c4 < cs && l0 + r < vl)
            v[j] = __ldg(reinterpret_cast<const float4*>(CB + kg + (long long)(l0 + r) * cs + sb + c4));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int vi = tid + kIT * j, r = vi >> 5, c4 = (vi & 31) * 4;
          *reinterpret_cast<float4*>(cbS + r * kLDB + c4) = v[j];
        }
      }
      __syncthreads();
      float gm[2][8];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) gm[i][j] = 0.f;
      int srow[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) srow[j] = min(sb + tq + 16 * j, cs - 1) * kLDP;
      int lrow[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) lrow[i] = min(l0 + tl + 32 * i, cs - 1) * kLDP;
      for (int p = 0; p < P; p += 4) {
        float4 a[2], b[8];
#pragma unroll
        for (int i = 0; i < 2; ++i) a[i] = lds4(yS + lrow[i] + p);
#pragma unroll
        for (int j = 0; j < 8; ++j) b[j] = lds4(uS + srow[j] + p);
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) gm[i][j] = dot4(a[i], b[j], gm[i][j]);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int l = l0 + tl + 32 * i;
        if (l >= vl) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int s = sb + tq + 16 * j;
          if (s > l) continue;
          const float cbg = gm[i][j] * dts[s] * expf(fminf(cms[l] - cms[s], 0.f));
          atomicAdd(CBg + kg + (long long)l * cs + s, cbg);
          if (s < l) {
            const float w = cbg * cbS[(tl + 32 * i) * kLDB + tq + 16 * j];
            rs[i] += w;
            atomicAdd(&cols[s], w);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float r = half_warp_sum(rs[i]);
      const int l = l0 + tl + 32 * i;
      if (tq == 0 && l < cs) rows[l] = r;
    }
  }
  __syncthreads();

  // dt backward, one token per thread
  dt_backward<kIT>(cols, rows, gBs, ddts, revc, tmp, gC, dl_part, nsl, delta_raw, A, delta_bias, draw_grad, A_part,
                   bias_part, ci, kh, h, H, cs, vl, ddt_dtype, use_sp, dmin, dmax);
}

// bwd_intra_split: the intra-chunk step for fp32 inputs at headdim 64, chunk 256, after the
// tensor-core products (ssd_split.cu): accY (split_bwd_accy) and G = y_grad u^T
// (split_bwd_g, lower 128 x 128 blocks) arrive in global memory, so this kernel keeps no
// operand rows in shared memory and runs several CTAs per SM. Per (head, chunk), 256 threads,
// 16 per row (4 headdim columns / 4 source tokens each):
//   acc = accS + accY: u_grad = acc dt_l, ddt[l] = sum_p acc u, gB[l] = dt_l sum_p accS u
//   CB_grad[l,s] += G[l,s] dt_s exp(min(cum_l - cum_s, 0))  (s <= l < length), 16-byte L2 atomics
//   w = that term * CB[l,s] (s < l): rows[l] = sum_s w, cols[s] = sum_l w
// then the dt backward (backward_kernel.py:296-314, :417-421, :632-659, :847-895).
__global__ void __launch_bounds__(256) bwd_intra_split_kernel(
    const float* __restrict__ u, const void* __restrict__ delta_raw, const float* __restrict__ A,
    const float* __restrict__ delta_bias, const float* __restrict__ dt, const float* __restrict__ cum,
    const float* __restrict__ CB, const float* __restrict__ accS, const float* __restrict__ gC,
    const float* __restrict__ accY, const float* __restrict__ Gyu, const float* __restrict__ dl_part, int nsl,
    float* __restrict__ CBg, float* __restrict__ u_grad, void* __restrict__ draw_grad, float* __restrict__ A_part,
    float* __restrict__ bias_part, ChunkMap cm, int H, int G, int ddt_dtype, int use_sp, float dmin, float dmax) {
  constexpr int cs = 256, P = 64;
  __shared__ float dts[cs], cms[cs], rows[cs], cols[cs], ddts[cs], gBs[cs], revc[cs], tmp[16];
  const int h = blockIdx.x, k = blockIdx.y, tid = threadIdx.x;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) {
    if (tid == 0) {
      A_part[(long long)k * H + h] = 0.f;
      bias_part[(long long)k * H + h] = 0.f;
    }
    return;
  }
  const int g = h / (H / G), vl = ci.vlim, lim = ci.lim;
  const long long kh = (long long)k * H + h;
  const long long kg = ((long long)k * G + g) * cs * cs;
  dts[tid] = dt[kh * cs + tid];
  cms[tid] = cum[kh * cs + tid];
  cols[tid] = 0.f;
  __syncthreads();
  const int grp = tid >> 4, tq = tid & 15;
  // per-row products: rows l = grp + 16 m, columns 4 tq .. 4 tq + 3
#pragma unroll 4
  for (int m = 0; m < 16; ++m) {
    const int l = grp + 16 * m;
    float dpart = 0.f, bpart = 0.f;
    if (l < vl) {
      const float4 s4 = __ldg(reinterpret_cast<const float4*>(accS + (kh * cs + l) * P) + tq);
      const float4 y4 = __ldg(reinterpret_cast<const float4*>(accY + (kh * cs + l) * P) + tq);
      const float4 u4 = __ldg(reinterpret_cast<const float4*>(u + ((ci.tok0 + l) * H + h) * P) + tq);
      const float4 acc = make_float4(s4.x + y4.x, s4.y + y4.y, s4.z + y4.z, s4.w + y4.w);
      dpart = dot4(acc, u4, 0.f);
      bpart = dot4(s4, u4, 0.f);
      const float d = dts[l];
      reinterpret_cast<float4*>(u_grad + ((ci.tok0 + l) * H + h) * P)[tq] =
          make_float4(acc.x * d, acc.y * d, acc.z * d, acc.w * d);
    } else if (l < lim) {
      reinterpret_cast<float4*>(u_grad + ((ci.tok0 + l) * H + h) * P)[tq] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    dpart = half_warp_sum(dpart);
    bpart = half_warp_sum(bpart);
    if (tq == 0) {
      ddts[l] = dpart;
      gBs[l] = bpart * dts[l];
    }
  }
  // CB_grad and the decay sums: rows l = grp + 16 m, source tokens s0 + 4 tq .. + 3 in
  // 64-token steps; a warp's two rows step to the larger row so that the sums stay uniform.
#pragma unroll 1
  for (int m = 0; m < 16; ++m) {
    const int l = grp + 16 * m, lw = ((tid >> 5) << 1) + 1 + 16 * m;
    const float cl = cms[l];
    const float* gr = Gyu + (kh * cs + l) * cs;
    const float* cbr = CB + kg + (long long)l * cs;
    float* cgr = CBg + kg + (long long)l * cs;
    float rsum = 0.f;
    for (int s0 = 0; s0 <= min(lw, vl - 1); s0 += 64) {
      const int s = s0 + 4 * tq;
      if (l < vl && s <= l) {
        const float4 gv = __ldg(reinterpret_cast<const float4*>(gr + s));
        const float4 cb = __ldg(reinterpret_cast<const float4*>(cbr + s));
        float c[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int se = s + e;
          c[e] = se <= l ? comp(gv, e) * dts[se] * expf(fminf(cl - cms[se], 0.f)) : 0.f;
          if (se < l) {
            const float w = c[e] * comp(cb, e);
            rsum += w;
            atomicAdd(&cols[se], w);
          }
        }
        atomicAdd(reinterpret_cast<float4*>(cgr + s), make_float4(c[0], c[1], c[2], c[3]));
      }
    }
    rsum = half_warp_sum(rsum);
    if (tq == 0) rows[l] = rsum;
  }
  __syncthreads();
  dt_backward<256>(cols, rows, gBs, ddts, revc, tmp, gC, dl_part, nsl, delta_raw, A, delta_bias, draw_grad, A_part,
                   bias_part, ci, kh, h, H, cs, vl, ddt_dtype, use_sp, dmin, dmax);
}

// bwd_dt: the dt backward alone, for the tensor-core intra kernel (ssd_bwd_tc.cu), which
// leaves ddt, gB, the row and the column decay sums per (chunk, head) in rows4 planes 0..3.
__global__ void __launch_bounds__(256) bwd_dt_kernel(
    const float* __restrict__ rows4, long long plane, const void* __restrict__ delta_raw, const float* __restrict__ A,
    const float* __restrict__ delta_bias, const float* __restrict__ gC, const float* __restrict__ dl_part, int nsl,
    void* __restrict__ draw_grad, float* __restrict__ A_part, float* __restrict__ bias_part, ChunkMap cm, int H,
    int ddt_dtype, int use_sp, float dmin, float dmax) {
  __shared__ float revc[kCSmax];
  __shared__ float tmp[16];
  const int h = blockIdx.x, k = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) {
    if (threadIdx.x == 0) {
      A_part[(long long)k * H + h] = 0.f;
      bias_part[(long long)k * H + h] = 0.f;
    }
    return;
  }
  const long long kh = (long long)k * H + h;
  const int cs = cm.cs;
  const float* base = rows4 + kh * cs;
  dt_backward<256>(base + 3 * plane, base + 2 * plane, base + plane, base, revc, tmp, gC, dl_part, nsl, delta_raw,
                   A, delta_bias, draw_grad, A_part, bias_part, ci, kh, h, H, cs, ci.vlim, ddt_dtype, use_sp, dmin,
                   dmax);
}

// ===========================================================================
// bwd_bmm: bmm_chunk_backward (backward_kernel.py:686-780, called twice at
// backward.py:534-535), per (64-row tile, group, chunk):
//   C_grad[l,:] += sum_{s<=l} CB_grad[l,s] B[s,:]     (blockIdx.x <  nt)
//   B_grad[s,:] += sum_{l>=s} CB_grad[l,s] C[l,:]     (blockIdx.x >= nt)
// Each output row belongs to one CTA: read-modify-write, no atomics.
// ===========================================================================
__global__ void __launch_bounds__(256) bwd_bmm_kernel(const void* __restrict__ Bm, const void* __restrict__ Cm,
                                                      const float* __restrict__ CBg, float* __restrict__ Bgrad,
                                                      float* __restrict__ Cgrad, ChunkMap cm, int G, int N,
                                                      int xdt) {
  constexpr int LDA = kLT + 4;
  __shared__ __align__(16) float At[64 * LDA];
  __shared__ __align__(16) float Bt[kLT * kLDN];
  const int k = blockIdx.z, g = blockIdx.y, tid = threadIdx.x;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int cs = cm.cs, vl = ci.vlim, nt = (cs + 63) / 64;
  const int which = blockIdx.x / nt, r0 = (blockIdx.x - which * nt) * 64;
  if (r0 >= vl) return;
  const float* cbg = CBg + ((long long)k * G + g) * cs * cs;
  const void* X = which == 0 ? Bm : Cm;
  float* out = which == 0 ? Cgrad : Bgrad;
  const int kbeg = which == 0 ? 0 : r0;
  const int kend = which == 0 ? min(r0 + 64, vl) : vl;
  const int tl = tid >> 4, tq = tid & 15;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int kb = kbeg; kb < kend; kb += kLT) {
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int vi = tid + 256 * j;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (which == 0) {  // A[r][c] = CB_grad[r0 + r][kb + c]: row r, 4 columns from c4
        const int r = vi >> 3, c4 = (vi & 7) * 4;
        if (r0 + r < cs && kb + c4 < cs)
          v = __ldg(reinterpret_cast<const float4*>(cbg + (long long)(r0 + r) * cs + kb + c4));
        if (kb + c4 >= kend) v.x = 0.f;
        if (kb + c4 + 1 >= kend) v.y = 0.f;
        if (kb + c4 + 2 >= kend) v.z = 0.f;
        if (kb + c4 + 3 >= kend) v.w = 0.f;
        *reinterpret_cast<float4*>(At + r * LDA + c4) = v;
      } else {           // A[r][c] = CB_grad[kb + c][r0 + r]: CB_grad row kb + c, 4 columns from r4
        const int c = vi >> 4, r4 = (vi & 15) * 4;
        if (kb + c < kend && r0 + r4 < cs)
          v = __ldg(reinterpret_cast<const float4*>(cbg + (long long)(kb + c) * cs + r0 + r4));
#pragma unroll
        for (int e = 0; e < 4; ++e) At[(r4 + e) * LDA + c] = comp(v, e);
      }
    }
    stage<2, false>(Bt, kLDN, X, xdt, ci.tok0, kb, kLT, (long long)G * N, (long long)g * N, N, kend, nullptr);
    __syncthreads();
#pragma unroll 2
    for (int c = 0; c < kLT; c += 4) {
      float4 a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = lds4(At + (tl + 16 * i) * LDA + c);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 b0 = lds4(Bt + (c + q) * kLDN + 4 * tq), b1 = lds4(Bt + (c + q) * kLDN + 64 + 4 * tq);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float m = comp(a[i], q);
          acc[i][0] = fmaf(m, b0.x, acc[i][0]);
          acc[i][1] = fmaf(m, b0.y, acc[i][1]);
          acc[i][2] = fmaf(m, b0.z, acc[i][2]);
          acc[i][3] = fmaf(m, b0.w, acc[i][3]);
          acc[i][4] = fmaf(m, b1.x, acc[i][4]);
          acc[i][5] = fmaf(m, b1.y, acc[i][5]);
          acc[i][6] = fmaf(m, b1.z, acc[i][6]);
          acc[i][7] = fmaf(m, b1.w, acc[i][7]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + tl + 16 * i;
    if (r >= vl) continue;
    const long long row = ((ci.tok0 + r) * G + g) * (long long)N;
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int n0 = 4 * tq + 64 * jj;
      if (n0 >= N) continue;
      float4* o = reinterpret_cast<float4*>(out + row + n0);
      float4 v = *o;
      v.x += acc[i][4 * jj];
      v.y += acc[i][4 * jj + 1];
      v.z += acc[i][4 * jj + 2];
      v.w += acc[i][4 * jj + 3];
      *o = v;
    }
  }
}

// A_grad[h] = sum_k A_part[k,h]; delta_bias_grad likewise (fixed order: deterministic).
__global__ void __launch_bounds__(256) bwd_param_reduce_kernel(const float* __restrict__ A_part,
                                                               const float* __restrict__ bias_part,
                                                               float* __restrict__ A_grad,
                                                               float* __restrict__ bias_grad, int nchunks, int H) {
  __shared__ float tmp[8];
  const int h = blockIdx.x;
  float a = 0.f, b = 0.f;
  for (int k = threadIdx.x; k < nchunks; k += 256) {
    a += A_part[(long long)k * H + h];
    b += bias_part[(long long)k * H + h];
  }
  a = block_sum(a, tmp);
  b = block_sum(b, tmp);
  if (threadIdx.x == 0) {
    A_grad[h] = a;
    if (bias_grad) bias_grad[h] = b;
  }
}

constexpr size_t kSmemStates = (size_t)((kPmax + kNmax) * 68 + kCSmax) * sizeof(float);
constexpr size_t kSmemCB = (size_t)(2 * 64 * kLDN) * sizeof(float);
constexpr size_t kSmemStateGrad =
    (size_t)(2 * kPmax * kLDN + kLT * kLDN + 2 * kLT * kLDP + 3 * kCSmax) * sizeof(float);
constexpr size_t kSmemIntra = (size_t)(2 * kCSmax * kLDP + 2 * kIR * kLDB + 7 * kCSmax + 16) * sizeof(float);

cudaError_t opt_in(const void* fn, size_t bytes) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

bool bwd_supported(int P, int N, int cs) {
  return P >= 8 && P <= kPmax && P % 8 == 0 && N >= 8 && N <= kNmax && N % 8 == 0 && cs >= kLT &&
         cs <= kCSmax && cs % kLT == 0;
}

size_t bwd_dl_slices(int P, int N) { return (size_t)((P * N / 4 + 255) / 256) * 8; }

cudaError_t launch_ssd_bwd(const LaunchCtx& c, const BwdArgs& a) {
  const int H = c.H, G = c.G, P = c.P, N = c.N, cs = c.cs, PN = P * N;
  const int nk = c.nchunks_max;
  if (nk > 65535 || H > 65535 || c.nrows > 65535) return cudaErrorInvalidValue;
  cudaError_t e;
  if ((e = opt_in((const void*)bwd_chunk_states_kernel, kSmemStates))) return e;
  if ((e = opt_in((const void*)bwd_cb_kernel, kSmemCB))) return e;
  if ((e = opt_in((const void*)bwd_state_grad_kernel, kSmemStateGrad))) return e;
  if ((e = opt_in((const void*)bwd_intra_kernel, kSmemIntra))) return e;
  const size_t bc_bytes = (size_t)c.T * G * N * sizeof(float);
  if ((e = cudaMemsetAsync(a.B_grad, 0, bc_bytes, c.stream))) return e;
  if ((e = cudaMemsetAsync(a.C_grad, 0, bc_bytes, c.stream))) return e;
  if ((e = cudaMemsetAsync(a.CBg, 0, (size_t)nk * G * cs * cs * sizeof(float), c.stream))) return e;
  if ((e = launch_chunk_cumsum(c, a.dt_dtype, a.A, a.delta_raw, a.delta_bias, a.dt, a.cum))) return e;
  const dim3 gkh((unsigned)H, (unsigned)nk);
  // grid x = head: the heads of one chunk run side by side and share its B, C, CB in L2
  const bool tc = bwd_state_grad_tc_supported(a.x_dtype, a.y_dtype, P, N, cs);
  // fp32 inputs at P 64, N 128, cs 256: the recompute and the state-side products on tcgen05
  // with split-bf16 products (ssd_split.cu); 16-byte loads of u, B, C and y_grad
  const bool split32 = !tc && a.Bs_split && a.Cs_split && split_supported(a.x_dtype, a.y_dtype, P, N, cs) &&
                       ((reinterpret_cast<uintptr_t>(a.u) | reinterpret_cast<uintptr_t>(a.B) |
                         reinterpret_cast<uintptr_t>(a.C) | reinterpret_cast<uintptr_t>(a.y_grad)) & 15u) == 0;
  if (tc) {
    if ((e = launch_bwd_chunk_states_tc(c, a))) return e;
  } else if (split32) {
    // fp32 inputs: the chunk states and HG on tcgen05 with split-bf16 products (the forward's
    // chunk_state kernel; B and C split once per (chunk, group))
    const float *u32 = static_cast<const float*>(a.u), *B32 = static_cast<const float*>(a.B),
                *C32 = static_cast<const float*>(a.C), *y32 = static_cast<const float*>(a.y_grad);
    if ((e = launch_split_b(c, B32, a.Bs_split)) || (e = launch_split_b(c, C32, a.Cs_split)) ||
        (e = launch_split_chunk_state(c, u32, a.Bs_split, a.dt, a.cum, a.states, 0)) ||
        (e = launch_split_chunk_state(c, y32, a.Cs_split, a.dt, a.cum, a.hg, 1)))
      return e;
  } else {
    bwd_chunk_states_kernel<<<dim3((unsigned)H, (unsigned)nk, 2u), 256, kSmemStates, c.stream>>>(
        a.u, a.B, a.C, a.y_grad, a.dt, a.cum, a.states, a.hg, c.cm, H, G, P, N, a.x_dtype, a.y_dtype);
    if ((e = cudaGetLastError())) return e;
  }
  if (a.ev[1]) cudaEventRecord(a.ev[1], c.stream);
  const int nsl = (int)bwd_dl_slices(P, N);  // per-warp partials of the decay_last gradient
  bwd_state_pass_kernel<<<dim3((unsigned)(nsl / 8), (unsigned)H, (unsigned)c.nrows), 256, 0, c.stream>>>(
      a.states, a.hg, a.cum, a.h_init, a.h_last_grad, a.h_init_grad, a.dl_part, c.cm, H, PN, tc ? a.prev16 : nullptr,
      tc ? a.hg16 : nullptr, a.x_dtype);
  if ((e = cudaGetLastError())) return e;
  const int nt = (cs + 63) / 64;
  if (tc) {
    if ((e = launch_bwd_cb_tc(c, a))) return e;
  } else {
    bwd_cb_kernel<<<dim3((unsigned)(nt * (nt + 1) / 2), (unsigned)G, (unsigned)nk), 256, kSmemCB, c.stream>>>(
        a.B, a.C, a.CB, c.cm, G, N, a.x_dtype);
    if ((e = cudaGetLastError())) return e;
  }
  if (a.ev[2]) cudaEventRecord(a.ev[2], c.stream);
  if (tc) {
    if ((e = launch_bwd_state_grad_grp_tc(c, a))) return e;
  } else if (split32) {
    if ((e = launch_split_state_grad(c, static_cast<const float*>(a.u), static_cast<const float*>(a.B),
                                     static_cast<const float*>(a.C), static_cast<const float*>(a.y_grad), a.dt,
                                     a.cum, a.states, a.hg, a.accS, a.B_grad, a.C_grad, a.gC)))
      return e;
  } else {
    bwd_state_grad_kernel<<<gkh, 256, kSmemStateGrad, c.stream>>>(
        a.u, a.B, a.C, a.y_grad, a.dt, a.cum, a.states, a.hg, a.accS, a.B_grad, a.C_grad, a.gC, c.cm, H, G, P, N,
        a.x_dtype, a.y_dtype);
    if ((e = cudaGetLastError())) return e;
  }
  if (a.ev[3]) cudaEventRecord(a.ev[3], c.stream);
  if (tc) {
    if ((e = launch_bwd_intra_tc(c, a))) return e;
    bwd_dt_kernel<<<gkh, 256, 0, c.stream>>>(a.rows4, (long long)nk * H * cs, a.delta_raw, a.A, a.delta_bias, a.gC,
                                              a.dl_part, nsl, a.delta_raw_grad, a.A_part, a.bias_part, c.cm, H,
                                              a.dt_dtype, c.use_sp, c.dmin, c.dmax);
  } else if (split32) {
    if ((e = launch_split_bwd_accy(c, a.CB, static_cast<const float*>(a.y_grad), a.cum, a.accY)) ||
        (e = launch_split_bwd_g(c, static_cast<const float*>(a.u), static_cast<const float*>(a.y_grad), a.Gyu)))
      return e;
    bwd_intra_split_kernel<<<gkh, 256, 0, c.stream>>>(
        static_cast<const float*>(a.u), a.delta_raw, a.A, a.delta_bias, a.dt, a.cum, a.CB, a.accS, a.gC, a.accY,
        a.Gyu, a.dl_part, nsl, a.CBg, static_cast<float*>(a.u_grad), a.delta_raw_grad, a.A_part, a.bias_part, c.cm,
        H, G, a.dt_dtype, c.use_sp, c.dmin, c.dmax);
  } else {
    bwd_intra_kernel<<<gkh, kIT, kSmemIntra, c.stream>>>(
        a.u, a.y_grad, a.delta_raw, a.A, a.delta_bias, a.dt, a.cum, a.CB, a.accS, a.gC, a.dl_part, nsl,
        a.CBg,
        a.u_grad, a.delta_raw_grad, a.A_part, a.bias_part, c.cm, H, G, P, a.x_dtype, a.y_dtype, a.dt_dtype,
        c.use_sp, c.dmin, c.dmax);
  }
  if ((e = cudaGetLastError())) return e;
  if (a.ev[4]) cudaEventRecord(a.ev[4], c.stream);
  if (tc) {
    if ((e = launch_bwd_bmm_tc(c, a))) return e;
  } else {
    bwd_bmm_kernel<<<dim3((unsigned)(2 * nt), (unsigned)G, (unsigned)nk), 256, 0, c.stream>>>(
        a.B, a.C, a.CBg, a.B_grad, a.C_grad, c.cm, G, N, a.x_dtype);
    if ((e = cudaGetLastError())) return e;
  }
  bwd_param_reduce_kernel<<<(unsigned)H, 256, 0, c.stream>>>(a.A_part, a.bias_part, a.A_grad, a.delta_bias_grad,
                                                             nk, H);
  return cudaGetLastError();
}

}  // namespace ssdb200
