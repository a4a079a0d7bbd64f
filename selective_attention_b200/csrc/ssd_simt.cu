// ssd_simt.cu - bandwidth kernels shared by both SSD paths (chunk_cumsum,
// state_passing, packed chunk table) and the CUDA-core (FFMA) versions of
// chunk_state, bmm_chunk and chunk_scan used for fp32 inputs and for shapes the
// tensor-core kernels do not cover.
#include "common.cuh"
#include "kernels.h"

namespace ssdb200 {

// ===========================================================================
// chunk_cumsum: ssd_scan/forward_kernel.py:19-87.
// One warp per (chunk, head): lane i owns tokens [i*E, i*E + E), E = ceil(cs/32),
// loads and transforms them (bias, softplus, clamp, length mask), scans them
// sequentially and adds the exclusive shuffle scan of the lane totals. Writes dt
// and cum, both (nchunks, H, cs).
// ===========================================================================
template <typename DT>
__global__ void __launch_bounds__(256) chunk_cumsum_kernel(
    const float* __restrict__ A, const DT* __restrict__ delta_raw, const float* __restrict__ delta_bias,
    float* __restrict__ dt_out, float* __restrict__ cum_out, ChunkMap cm, int H, int use_sp,
    float dmin, float dmax) {
  const int k = blockIdx.x;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 8 + warp;
  if (h >= H) return;
  const int cs = cm.cs;
  const int E = (cs + 31) >> 5;  // tokens per lane (<= 8)
  const float a = A[h];
  const float bias = delta_bias ? delta_bias[h] : 0.f;
  float dv[8], vals[8], raw[8];
  float run = 0.f;
  // all eight loads issued before any is used (indices clamped into the chunk, values masked)
#pragma unroll
  for (int e = 0; e < 8; ++e)
    raw[e] = Ld<DT>::f(delta_raw + (ci.tok0 + min(lane * E + e, max(ci.vlim - 1, 0))) * (long long)H + h);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int t = lane * E + e;
    const float v = (e < E && t < ci.vlim) ? dt_transform(raw[e] + bias, use_sp, dmin, dmax) : 0.f;
    dv[e] = v;
    run += v * a;
    vals[e] = run;
  }
  float incl = run;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  const float excl = incl - run;
  const long long base = ((long long)k * H + h) * cs;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int t = lane * E + e;
    if (e < E && t < cs) {
      dt_out[base + t] = dv[e];
      cum_out[base + t] = excl + vals[e];
    }
  }
}

// ===========================================================================
// state_passing: ssd_scan/forward_kernel.py:202-250.
// One thread per 4 consecutive state elements of one (row, head); walks the row's
// chunks in order: out[c] = prev; prev = exp(cum_last[c]) * prev + S[c].
// Prev states overwrite S in place (fp32), as the reference does.
// ===========================================================================
__global__ void __launch_bounds__(256) state_passing_kernel(float* __restrict__ states, const float* __restrict__ cum,
                                                           const float* __restrict__ h_init,
                                                           float* __restrict__ h_last, ChunkMap cm, int H, int PN) {
  const int row = blockIdx.z, h = blockIdx.y;
  const int e0 = (blockIdx.x * 256 + threadIdx.x) * 4;
  if (e0 >= PN) return;
  int first, count;
  if (cm.packed) {
    int2 r = cm.rows[row];
    first = r.x;
    count = r.y;
  } else {
    first = row * cm.nc;
    count = cm.nc;
  }
  const int cs = cm.cs;
  float4 prev = make_float4(0.f, 0.f, 0.f, 0.f);
  if (h_init) prev = *reinterpret_cast<const float4*>(h_init + ((long long)row * H + h) * PN + e0);
  float4 nxt = make_float4(0.f, 0.f, 0.f, 0.f);
  if (count > 0) nxt = *reinterpret_cast<const float4*>(states + ((long long)first * H + h) * PN + e0);
  for (int c = 0; c < count; ++c) {
    const long long kk = first + c;
    const float4 s = nxt;
    if (c + 1 < count) nxt = *reinterpret_cast<const float4*>(states + ((kk + 1) * H + h) * PN + e0);
    const long long off = (kk * H + h) * PN + e0;
    *reinterpret_cast<float4*>(states + off) = prev;
    const float sc = expf(cum[(kk * H + h) * cs + cs - 1]);
    prev.x = sc * prev.x + s.x;
    prev.y = sc * prev.y + s.y;
    prev.z = sc * prev.z + s.z;
    prev.w = sc * prev.w + s.w;
  }
  *reinterpret_cast<float4*>(h_last + ((long long)row * H + h) * PN + e0) = prev;
}

// ===========================================================================
// state_passing for the tensor-core chunk_scan (P = 64, N = 128): the same
// recurrence, but the prev states go to a separate buffer in the input's 16-bit
// type laid out [chunk][head][n][p] (p contiguous), and S is left untouched.
// One CTA per (32 dstate rows, head, row); thread (n, p pairs) reads S coalesced
// along n and the tile is transposed through shared memory for 16-byte stores.
// ===========================================================================
template <typename P16>
__global__ void __launch_bounds__(256) state_passing16_kernel(
    const float* __restrict__ states, P16* __restrict__ prev16, const float* __restrict__ cum,
    const float* __restrict__ h_init, float* __restrict__ h_last, ChunkMap cm, int H) {
  constexpr int P = 64, N = 128, PN = P * N;
  __shared__ uint32_t sT[32 * 33];  // [n][p pair], padded rows
  const int row = blockIdx.z, h = blockIdx.y, n0 = blockIdx.x * 32;
  const int tid = threadIdx.x, nl = tid & 31, pr = tid >> 5;
  int first, count;
  if (cm.packed) {
    const int2 r = cm.rows[row];
    first = r.x;
    count = r.y;
  } else {
    first = row * cm.nc;
    count = cm.nc;
  }
  // thread's elements: n = n0 + nl, p = 2 (pr + 8 i) + e, i < 4, e < 2
  float prev[8];
  const long long hoff = ((long long)row * H + h) * PN + n0 + nl;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 2; ++e) prev[2 * i + e] = h_init ? h_init[hoff + (2 * (pr + 8 * i) + e) * N] : 0.f;
  const int orow = tid >> 3, oq = tid & 7;  // read-out: row n0 + orow, p [8 oq, 8 oq + 8)
  for (int c = 0; c < count; ++c) {
    const long long kk = first + c;
    const long long soff = (kk * H + h) * PN + n0 + nl;
    float s[8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int e = 0; e < 2; ++e) s[2 * i + e] = states[soff + (2 * (pr + 8 * i) + e) * N];
#pragma unroll
    for (int i = 0; i < 4; ++i) sT[nl * 33 + pr + 8 * i] = pack2<P16>(prev[2 * i], prev[2 * i + 1]);
    __syncthreads();
    uint4 v;
    v.x = sT[orow * 33 + 4 * oq];
    v.y = sT[orow * 33 + 4 * oq + 1];
    v.z = sT[orow * 33 + 4 * oq + 2];
    v.w = sT[orow * 33 + 4 * oq + 3];
    *reinterpret_cast<uint4*>(prev16 + (kk * H + h) * PN + (long long)(n0 + orow) * P + 8 * oq) = v;
    __syncthreads();
    const float sc = expf(cum[(kk * H + h) * cm.cs + cm.cs - 1]);
#pragma unroll
    for (int j = 0; j < 8; ++j) prev[j] = sc * prev[j] + s[j];
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 2; ++e) h_last[hoff + (2 * (pr + 8 * i) + e) * N] = prev[2 * i + e];
}

// ===========================================================================
// Packed mode: chunk table from cu_seqlens (one CTA). Sequence i of length len
// gets ceil(len/cs) chunks starting at token cu[i]; rows[i] = {first, count}.
// ===========================================================================
template <typename IT>
__global__ void __launch_bounds__(1024) build_chunk_table_kernel(const IT* __restrict__ cu, int nseq, int cs,
                                                                 ChunkEntry* __restrict__ table,
                                                                 int2* __restrict__ rows, int* __restrict__ count) {
  __shared__ int warp_sums[32];
  __shared__ int running_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) running_s = 0;
  __syncthreads();
  for (int base = 0; base < nseq; base += 1024) {
    const int i = base + tid;
    long long start = 0, len = 0;
    int n = 0;
    if (i < nseq) {
      start = (long long)cu[i];
      len = (long long)cu[i + 1] - start;
      if (len < 0) len = 0;
      n = (int)((len + cs - 1) / cs);
    }
    int incl = n;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
      int wi = w;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        int o = __shfl_up_sync(0xffffffffu, wi, off);
        if (lane >= off) wi += o;
      }
      warp_sums[lane] = wi - w;  // exclusive prefix of warp totals
    }
    __syncthreads();
    const int running = running_s;
    const int first = running + warp_sums[warp] + incl - n;
    if (i < nseq) {
      rows[i] = make_int2(first, n);
      for (int c = 0; c < n; ++c) {
        ChunkEntry e;
        e.row = i;
        e.c = c;
        e.tok0 = start + (long long)c * cs;
        long long rem = len - (long long)c * cs;
        e.lim = (int)(rem < cs ? rem : cs);
        e.pad = 0;
        table[first + c] = e;
      }
    }
    __syncthreads();
    if (tid == 1023) running_s = first + n;
    __syncthreads();
  }
  if (tid == 0) *count = running_s;
}

// ===========================================================================
// CUDA-core chunk_state: ssd_scan/forward_kernel.py:107-185.
// CTA = (4096-output slice of P*N, head, chunk); 16 outputs per thread.
// Token tiles of 32 are staged in shared memory as x*w and B.
// ===========================================================================
template <typename T>
__global__ void __launch_bounds__(256) simt_chunk_state_kernel(
    const T* __restrict__ u, const T* __restrict__ Bm, const float* __restrict__ dt,
    const float* __restrict__ cum, float* __restrict__ states, ChunkMap cm, int H, int G, int P, int N) {
  extern __shared__ float sm[];
  const int k = blockIdx.z, h = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int cs = cm.cs, hpg = H / G, g = h / hpg;
  float* xs = sm;            // [32][P]
  float* bs = sm + 32 * P;   // [32][N]
  const int tid = threadIdx.x;
  const int PN = P * N;
  int pp[16], nn[16];
  const int o0 = blockIdx.x * 4096 + tid * 16;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    int o = o0 + i;
    if (o >= PN) o = PN - 1;
    pp[i] = o / N;
    nn[i] = o - pp[i] * N;
  }
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  const float* dtk = dt + ((long long)k * H + h) * cs;
  const float* cmk = cum + ((long long)k * H + h) * cs;
  const float clast = cmk[cs - 1];
  for (int l0 = 0; l0 < ci.lim; l0 += 32) {
    for (int idx = tid; idx < 32 * P; idx += 256) {
      const int l = idx / P, p = idx - l * P;
      float v = 0.f;
      if (l0 + l < ci.lim) {
        const float w = expf(fminf(clast - cmk[l0 + l], 0.f)) * dtk[l0 + l];
        v = Ld<T>::f(u + ((ci.tok0 + l0 + l) * H + h) * (long long)P + p) * w;
      }
      xs[idx] = v;
    }
    for (int idx = tid; idx < 32 * N; idx += 256) {
      const int l = idx / N, n = idx - l * N;
      float v = 0.f;
      if (l0 + l < ci.lim) v = Ld<T>::f(Bm + ((ci.tok0 + l0 + l) * G + g) * (long long)N + n);
      bs[idx] = v;
    }
    __syncthreads();
    const int lmax = min(32, ci.lim - l0);
    for (int l = 0; l < lmax; ++l) {
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = fmaf(xs[l * P + pp[i]], bs[l * N + nn[i]], acc[i]);
    }
    __syncthreads();
  }
  float* out = states + ((long long)k * H + h) * PN;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (o0 + i < PN) out[o0 + i] = acc[i];
}

// ===========================================================================
// CUDA-core bmm_chunk: ssd_scan/forward_kernel.py:270-328.
// CB[k,g,l,s] = sum_n C[l,n] B[s,n] for l,s < lim (zero outside), written for the
// whole cs x cs block (the reference writes only the lower tiles when causal).
// ===========================================================================
template <typename T>
__global__ void __launch_bounds__(256) simt_bmm_chunk_kernel(const T* __restrict__ Bm, const T* __restrict__ Cm,
                                                             float* __restrict__ CB, ChunkMap cm, int G, int N) {
  const int k = blockIdx.z, g = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int cs = cm.cs;
  const int o0 = blockIdx.x * 4096 + threadIdx.x * 16;
  float* out = CB + ((long long)k * G + g) * cs * cs;
  for (int i = 0; i < 16; ++i) {
    const int o = o0 + i;
    if (o >= cs * cs) break;
    const int l = o / cs, s = o - l * cs;
    float acc = 0.f;
    if (l < ci.lim && s < ci.lim) {
      const T* cr = Cm + ((ci.tok0 + l) * G + g) * (long long)N;
      const T* br = Bm + ((ci.tok0 + s) * G + g) * (long long)N;
      for (int n = 0; n < N; ++n) acc = fmaf(Ld<T>::f(cr + n), Ld<T>::f(br + n), acc);
    }
    out[o] = acc;
  }
}

// ===========================================================================
// CUDA-core chunk_scan: ssd_scan/forward_kernel.py:350-455, plus the D/z epilogue
// of modules/ssm.py:145-150. 16 outputs (l, p) per thread.
//   y = exp(cum_l) * sum_n C[l,n] prev[p,n]
//     + sum_{s<=l, s<lim} CB[l,s] exp(min(cum_l - cum_s, 0)) dt_s u[s,p]
// ===========================================================================
template <typename T, typename YT>
__global__ void __launch_bounds__(256) simt_chunk_scan_kernel(
    const T* __restrict__ u, const float* __restrict__ dt, const float* __restrict__ cum,
    const T* __restrict__ Cm, const float* __restrict__ prev, const float* __restrict__ CB,
    const float* __restrict__ D, const T* __restrict__ z, YT* __restrict__ y, ChunkMap cm, int H, int G,
    int P, int N) {
  const int k = blockIdx.z, h = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int cs = cm.cs, hpg = H / G, g = h / hpg;
  const float* dtk = dt + ((long long)k * H + h) * cs;
  const float* cmk = cum + ((long long)k * H + h) * cs;
  const float* hp = prev + ((long long)k * H + h) * (long long)P * N;
  const float* cbk = CB + ((long long)k * G + g) * cs * cs;
  const int o0 = blockIdx.x * 4096 + threadIdx.x * 16;
  for (int i = 0; i < 16; ++i) {
    const int o = o0 + i;
    if (o >= cs * P) break;
    const int l = o / P, p = o - l * P;
    if (l >= ci.lim) continue;
    const long long tok = ci.tok0 + l;
    const float cl = cmk[l];
    float acc = 0.f;
    const T* cr = Cm + (tok * G + g) * (long long)N;
    for (int n = 0; n < N; ++n) acc = fmaf(Ld<T>::f(cr + n), hp[p * N + n], acc);
    acc *= expf(cl);
    const int smax = min(l, ci.lim - 1);
    for (int s = 0; s <= smax; ++s) {
      const float m = cbk[l * cs + s] * expf(fminf(cl - cmk[s], 0.f)) * dtk[s];
      acc = fmaf(m, Ld<T>::f(u + ((ci.tok0 + s) * H + h) * (long long)P + p), acc);
    }
    const long long yo = (tok * H + h) * (long long)P + p;
    if (D) acc = fmaf(D[h * P + p], Ld<T>::f(u + yo), acc);
    if (z) acc *= silu(Ld<T>::f(z + yo));
    y[yo] = from_f32<YT>(acc);
  }
}


// ===========================================================================
// Tiled CUDA-core versions (P <= 64 and N <= 256, both multiples of 4): 64 x 64 output
// tiles per CTA, operand tiles staged in shared memory as fp32, 4 x 4 outputs per thread
// (rows tr + 16 i, columns 4 tc + j) from 16-byte shared-memory loads.
// ===========================================================================
constexpr int kTT = 64;       // output tile
constexpr int kTK = 32;       // reduction slice
constexpr int kTLD = kTK + 4; // [row][k] tiles
constexpr int kTLP = kTT + 4; // [k][col] tiles

__device__ __forceinline__ float c4(const float4& v, int e) { return e == 0 ? v.x : (e == 1 ? v.y : (e == 2 ? v.z : v.w)); }

// acc[i][j] += sum_k A[ar + 16 i][k] * Bt[k][4 bc + j]; A is [row][k] (kTLD), Bt is [k][col] (kTLP).
__device__ __forceinline__ void mma_rk_kc(float (&acc)[4][4], const float* A, const float* Bt, int ar, int bc,
                                          int kn) {
  for (int k = 0; k < kn; k += 4) {
    float4 a[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(A + (ar + 16 * i) * kTLD + k);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float4 b = *reinterpret_cast<const float4*>(Bt + (k + kk) * kTLP + 4 * bc);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x = c4(a[i], kk);
        acc[i][0] = fmaf(x, b.x, acc[i][0]);
        acc[i][1] = fmaf(x, b.y, acc[i][1]);
        acc[i][2] = fmaf(x, b.z, acc[i][2]);
        acc[i][3] = fmaf(x, b.w, acc[i][3]);
      }
    }
  }
}

// chunk_scan (forward_kernel.py:350-455 + the D / z epilogue of modules/ssm.py:145-150):
// CTA = (64-row tile of the chunk, head, chunk), all P columns.
//   y = exp(cum_l) C_l . prev + sum_{s <= l, s < lim} CB[l,s] exp(min(cum_l - cum_s, 0)) dt_s u_s
template <typename T, typename YT>
__global__ void __launch_bounds__(256) simt_chunk_scan_tiled_kernel(
    const T* __restrict__ u, const float* __restrict__ dt, const float* __restrict__ cum,
    const T* __restrict__ Cm, const float* __restrict__ prev, const float* __restrict__ CB,
    const float* __restrict__ D, const T* __restrict__ z, YT* __restrict__ y, ChunkMap cm, int H, int G,
    int P, int N) {
  __shared__ __align__(16) float As[kTT * kTLD];  // C rows [l][n] | M [l][s]
  __shared__ __align__(16) float Bs[kTK * kTLP];  // prev^T [n][p] | u [s][p]
  __shared__ float cml[kTT];
  const int k = blockIdx.z, h = blockIdx.y, l0 = blockIdx.x * kTT;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  if (l0 >= ci.lim) return;
  const int cs = cm.cs, g = h / (H / G), lim = ci.lim;
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  const float* dtk = dt + ((long long)k * H + h) * cs;
  const float* cmk = cum + ((long long)k * H + h) * cs;
  const float* hp = prev + ((long long)k * H + h) * (long long)P * N;
  const float* cbk = CB + ((long long)k * G + g) * cs * cs;
  if (tid < kTT) cml[tid] = l0 + tid < cs ? cmk[l0 + tid] : 0.f;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  // C . prev^T over slices of 32 states
  for (int n0 = 0; n0 < N; n0 += kTK) {
    __syncthreads();
    // all loads of the slice issued before any store (indices clamped into range, values masked)
    float cv[8], pv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + 256 * i, r = idx >> 5, c = idx & 31;
      const int l = min(l0 + r, lim - 1), n = min(n0 + c, N - 1), p = min(r, P - 1);
      cv[i] = Ld<T>::f(Cm + ((ci.tok0 + l) * G + g) * (long long)N + n);
      pv[i] = hp[(long long)p * N + n];  // prev^T: Bs[n][p], prev rows read along n
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + 256 * i, r = idx >> 5, c = idx & 31;
      const bool nok = n0 + c < N;
      As[r * kTLD + c] = (l0 + r < lim && nok) ? cv[i] : 0.f;
      Bs[c * kTLP + r] = (r < P && nok) ? pv[i] : 0.f;
    }
    __syncthreads();
    mma_rk_kc(acc, As, Bs, tr, tc, kTK);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float e = expf(cml[tr + 16 * i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] *= e;
  }
  // intra-chunk term over source slices of 32 tokens up to the tile's last row
  const int send = min(l0 + kTT, lim);
  for (int s0 = 0; s0 < send; s0 += kTK) {
    __syncthreads();
    float mv[8], cs8[8], dt8[8], uv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + 256 * i, r = idx >> 5, c = idx & 31;
      const int l = min(l0 + r, lim - 1), sidx = min(s0 + c, lim - 1);
      mv[i] = cbk[(long long)l * cs + sidx];
      cs8[i] = cmk[sidx];
      dt8[i] = dtk[sidx];
      const int ur = min(s0 + (idx >> 6), lim - 1), up = min(idx & 63, P - 1);
      uv[i] = Ld<T>::f(u + ((ci.tok0 + ur) * H + h) * (long long)P + up);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + 256 * i, r = idx >> 5, c = idx & 31, l = l0 + r, sidx = s0 + c;
      As[r * kTLD + c] = (l < lim && sidx <= l) ? mv[i] * expf(fminf(cml[r] - cs8[i], 0.f)) * dt8[i] : 0.f;
      const int ur = idx >> 6, up = idx & 63;
      Bs[ur * kTLP + up] = (s0 + ur < lim && up < P) ? uv[i] : 0.f;
    }
    __syncthreads();
    mma_rk_kc(acc, As, Bs, tr, tc, kTK);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = l0 + tr + 16 * i;
    if (l >= lim) continue;
    const long long tok = ci.tok0 + l;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int p = 4 * tc + j;
      if (p >= P) continue;
      const long long yo = (tok * H + h) * (long long)P + p;
      float v = acc[i][j];
      if (D) v = fmaf(D[h * P + p], Ld<T>::f(u + yo), v);
      if (z) v *= silu(Ld<T>::f(z + yo));
      y[yo] = from_f32<YT>(v);
    }
  }
}

// bmm_chunk (forward_kernel.py:270-328): CTA = (64 x 64 tile of CB, group, chunk);
// CB[l,s] = sum_n C[l,n] B[s,n] for l, s < lim, zero outside.
template <typename T>
__global__ void __launch_bounds__(256) simt_bmm_chunk_tiled_kernel(const T* __restrict__ Bm, const T* __restrict__ Cm,
                                                                   float* __restrict__ CB, ChunkMap cm, int G, int N) {
  __shared__ __align__(16) float As[kTT * kTLD];  // C rows [l][n]
  __shared__ __align__(16) float Bs[kTK * kTLP];  // B^T [n][s]
  const int k = blockIdx.z, g = blockIdx.y;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int cs = cm.cs, nt = (cs + kTT - 1) / kTT;
  const int l0 = (blockIdx.x / nt) * kTT, s0 = (blockIdx.x % nt) * kTT, lim = ci.lim;
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  if (l0 < lim && s0 < lim) {
    for (int n0 = 0; n0 < N; n0 += kTK) {
      __syncthreads();
      float cv[8], bv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = tid + 256 * i, r = idx >> 5, c = idx & 31, n = min(n0 + c, N - 1);
        cv[i] = Ld<T>::f(Cm + ((ci.tok0 + min(l0 + r, lim - 1)) * G + g) * (long long)N + n);
        bv[i] = Ld<T>::f(Bm + ((ci.tok0 + min(s0 + r, lim - 1)) * G + g) * (long long)N + n);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = tid + 256 * i, r = idx >> 5, c = idx & 31;
        const bool nok = n0 + c < N;
        As[r * kTLD + c] = (l0 + r < lim && nok) ? cv[i] : 0.f;
        Bs[c * kTLP + r] = (s0 + r < lim && nok) ? bv[i] : 0.f;
      }
      __syncthreads();
      mma_rk_kc(acc, As, Bs, tr, tc, kTK);
    }
  }
  float* out = CB + ((long long)k * G + g) * cs * cs;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = l0 + tr + 16 * i;
    if (l >= cs) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int sidx = s0 + 4 * tc + j;
      if (sidx < cs) out[(long long)l * cs + sidx] = (l < lim && sidx < lim) ? acc[i][j] : 0.f;
    }
  }
}

// chunk_state (forward_kernel.py:107-185): CTA = (64-state-column tile, head, chunk);
// states[p,n] = sum_l u[l,p] exp(min(cum_last - cum_l, 0)) dt_l B[l,n] over l < lim.
template <typename T>
__global__ void __launch_bounds__(256) simt_chunk_state_tiled_kernel(
    const T* __restrict__ u, const T* __restrict__ Bm, const float* __restrict__ dt,
    const float* __restrict__ cum, float* __restrict__ states, ChunkMap cm, int H, int G, int P, int N) {
  __shared__ __align__(16) float As[kTT * kTLD];  // (u w)^T [p][l]
  __shared__ __align__(16) float Bs[kTK * kTLP];  // B [l][n]
  const int k = blockIdx.z, h = blockIdx.y, n0 = blockIdx.x * kTT;
  ChunkInfo ci;
  if (!chunk_info(cm, k, ci)) return;
  const int cs = cm.cs, g = h / (H / G), lim = ci.lim;
  const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  const float* dtk = dt + ((long long)k * H + h) * cs;
  const float* cmk = cum + ((long long)k * H + h) * cs;
  const float clast = cmk[cs - 1];
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int t0 = 0; t0 < lim; t0 += kTK) {
    __syncthreads();
    float xv[8], bv[8], c8[8], d8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + 256 * i, r = idx >> 6, c = idx & 63;  // token r, column c
      const int l = min(t0 + r, lim - 1);
      xv[i] = Ld<T>::f(u + ((ci.tok0 + l) * H + h) * (long long)P + min(c, P - 1));
      bv[i] = Ld<T>::f(Bm + ((ci.tok0 + l) * G + g) * (long long)N + min(n0 + c, N - 1));
      c8[i] = cmk[l];
      d8[i] = dtk[l];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + 256 * i, r = idx >> 6, c = idx & 63;
      const bool lok = t0 + r < lim;
      As[c * kTLD + r] = (lok && c < P) ? xv[i] * (expf(fminf(clast - c8[i], 0.f)) * d8[i]) : 0.f;
      Bs[r * kTLP + c] = (lok && n0 + c < N) ? bv[i] : 0.f;
    }
    __syncthreads();
    mma_rk_kc(acc, As, Bs, tr, tc, kTK);
  }
  float* out = states + ((long long)k * H + h) * (long long)P * N;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = tr + 16 * i;
    if (p >= P) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + 4 * tc + j;
      if (n < N) out[(long long)p * N + n] = acc[i][j];
    }
  }
}

inline bool simt_tiled_ok(int P, int N) { return P <= 64 && N <= 256; }

// ===========================================================================
// Host launchers
// ===========================================================================
template <typename DT>
static cudaError_t launch_cumsum_t(const LaunchCtx& c, const float* A, const void* dr, const float* bias,
                                   float* dt, float* cum) {
  dim3 grid(c.nchunks_max, (unsigned)((c.H + 7) / 8));
  chunk_cumsum_kernel<DT><<<grid, 256, 0, c.stream>>>(A, (const DT*)dr, bias, dt, cum, c.cm, c.H, c.use_sp,
                                                      c.dmin, c.dmax);
  return cudaGetLastError();
}

cudaError_t launch_chunk_cumsum(const LaunchCtx& c, int dt_dtype, const float* A, const void* delta_raw,
                                const float* delta_bias, float* dt, float* cum) {
  switch (dt_dtype) {
    case SSD_F32: return launch_cumsum_t<float>(c, A, delta_raw, delta_bias, dt, cum);
    case SSD_BF16: return launch_cumsum_t<__nv_bfloat16>(c, A, delta_raw, delta_bias, dt, cum);
    case SSD_F16: return launch_cumsum_t<__half>(c, A, delta_raw, delta_bias, dt, cum);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_state_passing(const LaunchCtx& c, float* states, void* prev16, int prev_dtype,
                                 const float* cum, const float* h_init, float* h_last) {
  const int PN = c.P * c.N;
  if (prev16) {
    if (c.P != 64 || c.N != 128) return cudaErrorInvalidValue;
    dim3 g16(4u, (unsigned)c.H, (unsigned)c.nrows);
    if (prev_dtype == SSD_BF16)
      state_passing16_kernel<__nv_bfloat16><<<g16, 256, 0, c.stream>>>(states, (__nv_bfloat16*)prev16, cum, h_init,
                                                                       h_last, c.cm, c.H);
    else if (prev_dtype == SSD_F16)
      state_passing16_kernel<__half><<<g16, 256, 0, c.stream>>>(states, (__half*)prev16, cum, h_init, h_last, c.cm,
                                                                c.H);
    else
      return cudaErrorInvalidValue;
    return cudaGetLastError();
  }
  dim3 grid((unsigned)((PN / 4 + 255) / 256), (unsigned)c.H, (unsigned)c.nrows);
  state_passing_kernel<<<grid, 256, 0, c.stream>>>(states, cum, h_init, h_last, c.cm, c.H, PN);
  return cudaGetLastError();
}

cudaError_t launch_build_chunk_table(cudaStream_t s, const void* cu, int cu64, int nseq, int cs, ChunkEntry* table,
                                     int2* rows, int* count) {
  if (cu64)
    build_chunk_table_kernel<long long><<<1, 1024, 0, s>>>((const long long*)cu, nseq, cs, table, rows, count);
  else
    build_chunk_table_kernel<int><<<1, 1024, 0, s>>>((const int*)cu, nseq, cs, table, rows, count);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t simt_state_t(const LaunchCtx& c, const void* u, const void* B, const float* dt,
                                const float* cum, float* states) {
  const int PN = c.P * c.N;
  if (simt_tiled_ok(c.P, c.N)) {
    simt_chunk_state_tiled_kernel<T><<<dim3((unsigned)((c.N + kTT - 1) / kTT), (unsigned)c.H, (unsigned)c.nchunks_max),
                                       256, 0, c.stream>>>((const T*)u, (const T*)B, dt, cum, states, c.cm, c.H, c.G,
                                                           c.P, c.N);
    return cudaGetLastError();
  }
  dim3 grid((unsigned)((PN + 4095) / 4096), (unsigned)c.H, (unsigned)c.nchunks_max);
  size_t sm = (size_t)32 * (c.P + c.N) * sizeof(float);
  if (sm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(simt_chunk_state_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sm);
    if (e != cudaSuccess) return e;
  }
  simt_chunk_state_kernel<T><<<grid, 256, sm, c.stream>>>((const T*)u, (const T*)B, dt, cum, states, c.cm, c.H,
                                                          c.G, c.P, c.N);
  return cudaGetLastError();
}

cudaError_t launch_simt_chunk_state(const LaunchCtx& c, int x_dtype, const void* u, const void* B,
                                    const float* dt, const float* cum, float* states) {
  switch (x_dtype) {
    case SSD_F32: return simt_state_t<float>(c, u, B, dt, cum, states);
    case SSD_BF16: return simt_state_t<__nv_bfloat16>(c, u, B, dt, cum, states);
    case SSD_F16: return simt_state_t<__half>(c, u, B, dt, cum, states);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
static cudaError_t simt_bmm_t(const LaunchCtx& c, const void* B, const void* C, float* CB) {
  if (simt_tiled_ok(c.P, c.N)) {
    const int nt = (c.cs + kTT - 1) / kTT;
    simt_bmm_chunk_tiled_kernel<T><<<dim3((unsigned)(nt * nt), (unsigned)c.G, (unsigned)c.nchunks_max), 256, 0,
                                     c.stream>>>((const T*)B, (const T*)C, CB, c.cm, c.G, c.N);
    return cudaGetLastError();
  }
  dim3 grid((unsigned)((c.cs * c.cs + 4095) / 4096), (unsigned)c.G, (unsigned)c.nchunks_max);
  simt_bmm_chunk_kernel<T><<<grid, 256, 0, c.stream>>>((const T*)B, (const T*)C, CB, c.cm, c.G, c.N);
  return cudaGetLastError();
}

cudaError_t launch_simt_bmm_chunk(const LaunchCtx& c, int x_dtype, const void* B, const void* C, float* CB) {
  switch (x_dtype) {
    case SSD_F32: return simt_bmm_t<float>(c, B, C, CB);
    case SSD_BF16: return simt_bmm_t<__nv_bfloat16>(c, B, C, CB);
    case SSD_F16: return simt_bmm_t<__half>(c, B, C, CB);
  }
  return cudaErrorInvalidValue;
}

template <typename T, typename YT>
static cudaError_t simt_scan_t(const LaunchCtx& c, const void* u, const float* dt, const float* cum, const void* C,
                               const float* prev, const float* CB, const float* D, const void* z, void* y) {
  if (simt_tiled_ok(c.P, c.N)) {
    simt_chunk_scan_tiled_kernel<T, YT><<<dim3((unsigned)((c.cs + kTT - 1) / kTT), (unsigned)c.H,
                                               (unsigned)c.nchunks_max),
                                          256, 0, c.stream>>>((const T*)u, dt, cum, (const T*)C, prev, CB, D,
                                                              (const T*)z, (YT*)y, c.cm, c.H, c.G, c.P, c.N);
    return cudaGetLastError();
  }
  dim3 grid((unsigned)((c.cs * c.P + 4095) / 4096), (unsigned)c.H, (unsigned)c.nchunks_max);
  simt_chunk_scan_kernel<T, YT><<<grid, 256, 0, c.stream>>>((const T*)u, dt, cum, (const T*)C, prev, CB, D,
                                                            (const T*)z, (YT*)y, c.cm, c.H, c.G, c.P, c.N);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t simt_scan_y(const LaunchCtx& c, int y_dtype, const void* u, const float* dt, const float* cum,
                               const void* C, const float* prev, const float* CB, const float* D, const void* z,
                               void* y) {
  switch (y_dtype) {
    case SSD_F32: return simt_scan_t<T, float>(c, u, dt, cum, C, prev, CB, D, z, y);
    case SSD_BF16: return simt_scan_t<T, __nv_bfloat16>(c, u, dt, cum, C, prev, CB, D, z, y);
    case SSD_F16: return simt_scan_t<T, __half>(c, u, dt, cum, C, prev, CB, D, z, y);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_simt_chunk_scan(const LaunchCtx& c, int x_dtype, int y_dtype, const void* u, const float* dt,
                                   const float* cum, const void* C, const float* prev, const float* CB,
                                   const float* D, const void* z, void* y) {
  switch (x_dtype) {
    case SSD_F32: return simt_scan_y<float>(c, y_dtype, u, dt, cum, C, prev, CB, D, z, y);
    case SSD_BF16: return simt_scan_y<__nv_bfloat16>(c, y_dtype, u, dt, cum, C, prev, CB, D, z, y);
    case SSD_F16: return simt_scan_y<__half>(c, y_dtype, u, dt, cum, C, prev, CB, D, z, y);
  }
  return cudaErrorInvalidValue;
}

SSDB200_DEFINE_ERROR_FETCH(fetch_error_simt)

}  // namespace ssdb200
