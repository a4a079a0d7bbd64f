// sattn_train.cu - training-mode selective attention and its backward.
//
// SelectiveMHA.forward with self.training (modules/selective_attention.py:232-280):
//   S[i,j]   = scale q_i . k_j, causal (j <= i) or not                       (_build_attn_matrix :89-99)
//   stats    = mean and std over the valid scores of each head: i, j below the row's length
//              (and j <= i when causal), over batch and both positions       (:234-251)
//   lg[j]    = log(select_gate[j]) std penalty, -inf for keys past the length (:259-268)
//   P[i,:]   = softmax_j(S[i,j] + lg[j] for j != i, S[i,i] on the diagonal)   (_gated_softmax :125-144)
//   out[i]   = sum_j P[i,j] v_j                                               (:278)
// The std feeds the gate, so the backward has a path through the statistics:
//   dlg[j]   = sum_{i != j} dS[i,j],  dS = P (dP - D_i),  dP = dO v^T,  D_i = dO_i . out_i
//   dstd     = sum_{b, j < len} dlg[j] log(g[j]) penalty;  d select_gate[j] = dlg[j] std penalty / g[j]
//   dS_total = dS + c (S - mean) on valid scores,  c = dstd / (count std)  (d std / d S = (S - mean) / (count std))
//   dq_i = scale sum_j dS_total[i,j] k_j,  dk_j = scale sum_i dS_total[i,j] q_i,  dv_j = sum_i P[i,j] dO_i
//
// CUDA-core kernels (64 x 64 tiles, 256 threads, fp32 arithmetic on any input type); 16-bit
// inputs with head_dim 64 take the tensor-core versions further below:
//   stats      per (query tile, head, row): sums of the valid scores and of their squares
//   stats_fin  per head: mean, std, count (fp64 sums)
//   gate       lg = log(g) std penalty, -inf past the length
//   fwd        online-softmax attention with the row log-sum-exp saved (flash style)
//   rowdot     D_i = dO_i . out_i
//   dv         per key tile over the query tiles: dv and dlg
//   fin        per head: dstd, c, d select_gate
//   dk         per key tile: dk with dS_total
//   dq         per query tile: dq with dS_total
#include <math.h>

#include <cudaTypedefs.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "sattn_tiles.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace ssdb200 {
namespace {

using namespace sm100;

constexpr int kLDT = kPT + 4;  // fp32 64 x 64 score tiles

// sc[a][c] = sum_d A[ra + 16 a][d] * Bm[rb + 16 c][d] over the staged rows (ld floats apart).
__device__ __forceinline__ void tile_dot(float (&sc)[4][4], const float* A, const float* Bm, int ld, int ra, int rb,
                                         int D) {
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c) sc[a][c] = 0.f;
  for (int d = 0; d < D; d += 4) {
    float4 x[4], y[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) x[a] = *reinterpret_cast<const float4*>(A + (ra + 16 * a) * ld + d);
#pragma unroll
    for (int c = 0; c < 4; ++c) y[c] = *reinterpret_cast<const float4*>(Bm + (rb + 16 * c) * ld + d);
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t = sc[a][c];
        t = fmaf(x[a].x, y[c].x, t);
        t = fmaf(x[a].y, y[c].y, t);
        t = fmaf(x[a].z, y[c].z, t);
        sc[a][c] = fmaf(x[a].w, y[c].w, t);
      }
  }
}

// acc[a][4 g + e] += sum_r W[wr + 16 a][r] * R[r][dcol[g] + e] over the 64 tile rows r.
__device__ __forceinline__ void tile_acc(float (&acc)[4][8], const float* W, const float* R, int ld, int wr,
                                         const int (&dcol)[2]) {
#pragma unroll 2
  for (int r = 0; r < kPT; r += 4) {
    float4 w[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) w[a] = *reinterpret_cast<const float4*>(W + (wr + 16 * a) * kLDT + r);
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      float4 x[2];
#pragma unroll
      for (int g = 0; g < 2; ++g) x[g] = *reinterpret_cast<const float4*>(R + (r + rr) * ld + dcol[g]);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float p = rr == 0 ? w[a].x : (rr == 1 ? w[a].y : (rr == 2 ? w[a].z : w[a].w));
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          acc[a][4 * g] = fmaf(p, x[g].x, acc[a][4 * g]);
          acc[a][4 * g + 1] = fmaf(p, x[g].y, acc[a][4 * g + 1]);
          acc[a][4 * g + 2] = fmaf(p, x[g].z, acc[a][4 * g + 2]);
          acc[a][4 * g + 3] = fmaf(p, x[g].w, acc[a][4 * g + 3]);
        }
      }
    }
  }
}

__device__ __forceinline__ int row_len(const int64_t* lengths, int b, int L) {
  if (!lengths) return L;
  const long long n = lengths[b];
  return n < 0 ? 0 : (n > L ? L : (int)n);
}

// Key j takes part in query i's softmax: causal order, inside the tensor, and a finite logit
// (a key past the length has lg = -inf, except on the diagonal, which is not gated).
__device__ __forceinline__ float logit(float s, int qi, int kj, float g, int L, int causal) {
  if ((causal && kj > qi) || kj >= L || qi >= L) return -INFINITY;
  return kj == qi ? s : s + g;
}

__device__ __forceinline__ bool stat_valid(int qi, int kj, int len, int causal) {
  return qi < len && kj < len && (!causal || kj <= qi);
}

// Sum over a CTA of NW warps (red: NW slots of shared memory); every thread gets the total.
template <typename V, int NW = 8>
__device__ __forceinline__ V block_sum256(V v, V* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  V t = 0;
#pragma unroll
  for (int i = 0; i < NW; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ void dcols(int (&dcol)[2], int tc, int D) {
#pragma unroll
  for (int g = 0; g < 2; ++g) dcol[g] = min(4 * tc + 64 * g, D - 4);
}

template <typename T>
__device__ __forceinline__ void store_rows(T* dst, const float (&acc)[4][8], int r0, int tr, int tc, int L, int D,
                                           float mul) {
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int r = r0 + tr + 16 * a;
    if (r >= L) continue;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int d = 4 * tc + 64 * g;
      if (d >= D) continue;
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[(long long)r * D + d + e] = from_f32<T>(acc[a][4 * g + e] * mul);
    }
  }
}

// ---------------------------------------------------------------------------- statistics
template <typename T>
__global__ void __launch_bounds__(256) sattn_train_stats_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                                const int64_t* __restrict__ lengths, int H, int L,
                                                                int D, float scale, int causal, double* part) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  __shared__ double red[8];
  const int LD = D + 4;
  float* Qs = sm;
  float* Ks = Qs + kPT * LD;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const long long bh = (long long)b * H + h;
  const int len = row_len(lengths, b, L);
  const int q0 = qt * kPT, tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  float s1 = 0.f, s2 = 0.f;
  if (q0 < len) {
    stage_rows64<T>(Qs, LD, q + bh * L * D, q0, L, D);
    const int kend = causal ? min(q0 + kPT, len) : len;
    for (int k0 = 0; k0 < kend; k0 += kPT) {
      __syncthreads();
      stage_rows64<T>(Ks, LD, k + bh * L * D, k0, L, D);
      __syncthreads();
      float sc[4][4];
      tile_dot(sc, Qs, Ks, LD, tr, tc, D);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (stat_valid(q0 + tr + 16 * a, k0 + tc + 16 * c, len, causal)) {
            const float s = sc[a][c] * scale;
            s1 += s;
            s2 = fmaf(s, s, s2);
          }
    }
  }
  const double t1 = block_sum256<double>((double)s1, red);
  const double t2 = block_sum256<double>((double)s2, red);
  if (tid == 0) {
    part[(bh * gridDim.x + qt) * 2] = t1;
    part[(bh * gridDim.x + qt) * 2 + 1] = t2;
  }
}

// stats[h] = (mean, std, count, c): c is filled by the backward.
__global__ void __launch_bounds__(256) sattn_train_stats_fin_kernel(const double* __restrict__ part,
                                                                    const int64_t* __restrict__ lengths, int B, int H,
                                                                    int L, int nqt, int causal, float* stats) {
  __shared__ double red[8];
  const int h = blockIdx.x;
  double s1 = 0.0, s2 = 0.0, n = 0.0;
  for (int idx = threadIdx.x; idx < B * nqt; idx += 256) {
    const int b = idx / nqt, qt = idx - b * nqt;
    const double* p = part + (((long long)b * H + h) * nqt + qt) * 2;
    s1 += p[0];
    s2 += p[1];
  }
  for (int b = threadIdx.x; b < B; b += 256) {
    const double len = row_len(lengths, b, L);
    n += causal ? len * (len + 1.0) * 0.5 : len * len;
  }
  s1 = block_sum256<double>(s1, red);
  s2 = block_sum256<double>(s2, red);
  n = block_sum256<double>(n, red);
  if (threadIdx.x == 0) {
    const double N = n < 1.0 ? 1.0 : n;  // count.clamp(min=1) (:245-250)
    const double mean = s1 / N;
    const double var = s2 / N - mean * mean;
    stats[h * 4] = (float)mean;
    stats[h * 4 + 1] = (float)sqrt(var > 0.0 ? var : 0.0);
    stats[h * 4 + 2] = (float)n;
    stats[h * 4 + 3] = 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) sattn_train_gate_kernel(const T* __restrict__ gate,
                                                               const int64_t* __restrict__ lengths,
                                                               const float* __restrict__ stats, int H, int L,
                                                               long long n, float penalty, float* __restrict__ lg) {
  const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  const int j = (int)(i % L);
  const long long bh = i / L;
  const int h = (int)(bh % H), b = (int)(bh / H);
  lg[i] = j < row_len(lengths, b, L) ? logf(to_f32<T>(gate[i])) * stats[h * 4 + 1] * penalty : -INFINITY;
}

// ---------------------------------------------------------------------------- forward
template <typename T>
__global__ void __launch_bounds__(256) sattn_train_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                              const T* __restrict__ v, const float* __restrict__ lg,
                                                              T* __restrict__ out, float* __restrict__ lse, int H,
                                                              int L, int D, float scale, int causal) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int LD = D + 4;
  float* Qs = sm;
  float* Ks = Qs + kPT * LD;
  float* Vs = Ks + kPT * LD;
  float* Ps = Vs + kPT * LD;  // [64][kLDT]
  float* gs = Ps + kPT * kLDT;
  const int nt = (int)gridDim.x;
  const int qt = causal ? nt - 1 - (int)blockIdx.x : (int)blockIdx.x;  // causal: longest rows first
  const long long bh = (long long)blockIdx.z * H + blockIdx.y;
  const int q0 = qt * kPT, tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  stage_rows64<T>(Qs, LD, q + bh * L * D, q0, L, D);
  float o[4][8], m[4], l[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    m[a] = -INFINITY;
    l[a] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[a][e] = 0.f;
  }
  int dcol[2];
  dcols(dcol, tc, D);
  const int kend = causal ? qt + 1 : nt;
  for (int kt = 0; kt < kend; ++kt) {
    const int k0 = kt * kPT;
    __syncthreads();
    stage_rows64<T>(Ks, LD, k + bh * L * D, k0, L, D);
    stage_rows64<T>(Vs, LD, v + bh * L * D, k0, L, D);
    if (tid < kPT) gs[tid] = k0 + tid < L ? lg[bh * L + k0 + tid] : -INFINITY;
    __syncthreads();
    float sc[4][4];
    tile_dot(sc, Qs, Ks, LD, tr, tc, D);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int qi = q0 + tr + 16 * a;
      float rmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        sc[a][c] = logit(sc[a][c] * scale, qi, k0 + tc + 16 * c, gs[tc + 16 * c], L, causal);
        rmax = fmaxf(rmax, sc[a][c]);
      }
      rmax = hw_max(rmax);
      const float mn = fmaxf(m[a], rmax);
      const float corr = m[a] == -INFINITY ? 0.f : expf(m[a] - mn);
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float p = sc[a][c] == -INFINITY ? 0.f : expf(sc[a][c] - mn);
        rs += p;
        Ps[(tr + 16 * a) * kLDT + tc + 16 * c] = p;
      }
      l[a] = l[a] * corr + hw_sum(rs);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[a][e] *= corr;
      m[a] = mn;
    }
    __syncthreads();
    tile_acc(o, Ps, Vs, LD, tr, dcol);
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int qi = q0 + tr + 16 * a;
    if (qi < L && tc == 0) lse[bh * L + qi] = m[a] + logf(l[a]);
    const float inv = 1.0f / l[a];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[a][e] *= inv;
  }
  store_rows<T>(out + bh * L * D, o, q0, tr, tc, L, D, 1.f);
}

// ---------------------------------------------------------------------------- backward
// D_i = dO_i . out_i, one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) sattn_train_rowdot_kernel(const T* __restrict__ dout, const T* __restrict__ out,
                                                                 long long rows, int D, float* __restrict__ Di) {
  const long long r = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s = fmaf(to_f32<T>(dout[r * D + d]), to_f32<T>(out[r * D + d]), s);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) Di[r] = s;
}

// Key-major sweep: thread (tk, tq) owns keys k0 + tk + 16 a and, per query tile, queries
// q0 + tq + 16 c. MODE 0: dv and dlg (softmax part of dS). MODE 1: dk with dS_total.
template <typename T, int MODE>
__global__ void __launch_bounds__(256) sattn_train_bwd_kv_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ dout,
    const float* __restrict__ lg, const float* __restrict__ lse, const float* __restrict__ Di,
    const float* __restrict__ stats, const int64_t* __restrict__ lengths, int H, int L, int D, float scale,
    int causal, T* __restrict__ dkv, float* __restrict__ dlg) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int LD = D + 4;
  float* Ks = sm;
  float* Vs = Ks + kPT * LD;
  float* Qs = Vs + kPT * LD;
  float* Os = Qs + kPT * LD;    // dO tile
  float* Wt = Os + kPT * LD;    // [key][query]: P^T (MODE 0) or dS_total^T (MODE 1)
  float* ls = Wt + kPT * kLDT;  // lse of the query tile
  float* ds = ls + kPT;         // D_i of the query tile
  const int nt = (int)gridDim.x, kt = (int)blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const long long bh = (long long)b * H + h;
  const int len = row_len(lengths, b, L);
  const int k0 = kt * kPT, tid = threadIdx.x, tk = tid >> 4, tq = tid & 15;
  const float mean = stats[h * 4], c_st = stats[h * 4 + 3];
  stage_rows64<T>(Ks, LD, k + bh * L * D, k0, L, D);
  stage_rows64<T>(Vs, LD, v + bh * L * D, k0, L, D);
  float g[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int kj = k0 + tk + 16 * a;
    g[a] = kj < L ? lg[bh * L + kj] : -INFINITY;
  }
  float acc[4][8], dl[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    dl[a] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[a][e] = 0.f;
  }
  int dcol[2];
  dcols(dcol, tq, D);
  for (int qt = causal ? kt : 0; qt < nt; ++qt) {
    const int q0 = qt * kPT;
    __syncthreads();
    stage_rows64<T>(Qs, LD, q + bh * L * D, q0, L, D);
    stage_rows64<T>(Os, LD, dout + bh * L * D, q0, L, D);
    if (tid < kPT) {
      ls[tid] = q0 + tid < L ? lse[bh * L + q0 + tid] : 0.f;
      ds[tid] = q0 + tid < L ? Di[bh * L + q0 + tid] : 0.f;
    }
    __syncthreads();
    float st[4][4], dp[4][4];
    tile_dot(st, Ks, Qs, LD, tk, tq, D);
    tile_dot(dp, Vs, Os, LD, tk, tq, D);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int kj = k0 + tk + 16 * a;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int qi = q0 + tq + 16 * c;
        const float s = st[a][c] * scale;
        const float x = logit(s, qi, kj, g[a], L, causal);
        const float p = x == -INFINITY ? 0.f : expf(x - ls[tq + 16 * c]);
        const float dsm = p * (dp[a][c] - ds[tq + 16 * c]);
        float w;
        if (MODE == 0) {
          if (kj != qi) dl[a] += dsm;
          w = p;
        } else {
          w = dsm + (stat_valid(qi, kj, len, causal) ? c_st * (s - mean) : 0.f);
        }
        Wt[(tk + 16 * a) * kLDT + tq + 16 * c] = w;
      }
    }
    __syncthreads();
    tile_acc(acc, Wt, MODE == 0 ? Os : Qs, LD, tk, dcol);
  }
  if (MODE == 0) {
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float t = hw_sum(dl[a]);
      const int kj = k0 + tk + 16 * a;
      if (tq == 0 && kj < L) dlg[bh * L + kj] = t;
    }
  }
  store_rows<T>(dkv + bh * L * D, acc, k0, tk, tq, L, D, MODE == 0 ? 1.f : scale);
}

// Per head: dstd, the statistics coefficient c, and d select_gate.
template <typename T>
__global__ void __launch_bounds__(256) sattn_train_bwd_fin_kernel(const T* __restrict__ gate,
                                                                  const int64_t* __restrict__ lengths,
                                                                  const float* __restrict__ dlg, int B, int H, int L,
                                                                  float penalty, float* stats, T* __restrict__ dgate) {
  __shared__ double red[8];
  const int h = blockIdx.x;
  const float sd = stats[h * 4 + 1];
  double acc = 0.0;
  for (long long idx = threadIdx.x; idx < (long long)B * L; idx += 256) {
    const int b = (int)(idx / L), j = (int)(idx - (long long)b * L);
    const long long i = ((long long)b * H + h) * L + j;
    float dg = 0.f;
    if (j < row_len(lengths, b, L)) {
      const float gv = to_f32<T>(gate[i]);
      acc += (double)dlg[i] * (double)logf(gv) * (double)penalty;
      dg = dlg[i] * sd * penalty / gv;
    }
    dgate[i] = from_f32<T>(dg);
  }
  acc = block_sum256<double>(acc, red);
  if (threadIdx.x == 0) {
    const double n = stats[h * 4 + 2] < 1.f ? 1.0 : (double)stats[h * 4 + 2];
    stats[h * 4 + 3] = sd > 0.f ? (float)(acc / (n * (double)sd)) : 0.f;
  }
}

// Query-major sweep for dq: thread (tr, tc) owns queries q0 + tr + 16 a, keys k0 + tc + 16 c.
template <typename T>
__global__ void __launch_bounds__(256) sattn_train_bwd_q_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const T* __restrict__ dout,
    const float* __restrict__ lg, const float* __restrict__ lse, const float* __restrict__ Di,
    const float* __restrict__ stats, const int64_t* __restrict__ lengths, int H, int L, int D, float scale,
    int causal, T* __restrict__ dq) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int LD = D + 4;
  float* Qs = sm;
  float* Os = Qs + kPT * LD;
  float* Ks = Os + kPT * LD;
  float* Vs = Ks + kPT * LD;
  float* Ws = Vs + kPT * LD;  // dS_total [query][key]
  float* gs = Ws + kPT * kLDT;
  const int nt = (int)gridDim.x;
  const int qt = causal ? nt - 1 - (int)blockIdx.x : (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const long long bh = (long long)b * H + h;
  const int len = row_len(lengths, b, L);
  const int q0 = qt * kPT, tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
  const float mean = stats[h * 4], c_st = stats[h * 4 + 3];
  stage_rows64<T>(Qs, LD, q + bh * L * D, q0, L, D);
  stage_rows64<T>(Os, LD, dout + bh * L * D, q0, L, D);
  float lr[4], dr[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int qi = q0 + tr + 16 * a;
    lr[a] = qi < L ? lse[bh * L + qi] : 0.f;
    dr[a] = qi < L ? Di[bh * L + qi] : 0.f;
  }
  float acc[4][8];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[a][e] = 0.f;
  int dcol[2];
  dcols(dcol, tc, D);
  const int kend = causal ? qt + 1 : nt;
  for (int kt = 0; kt < kend; ++kt) {
    const int k0 = kt * kPT;
    __syncthreads();
    stage_rows64<T>(Ks, LD, k + bh * L * D, k0, L, D);
    stage_rows64<T>(Vs, LD, v + bh * L * D, k0, L, D);
    if (tid < kPT) gs[tid] = k0 + tid < L ? lg[bh * L + k0 + tid] : -INFINITY;
    __syncthreads();
    float sc[4][4], dp[4][4];
    tile_dot(sc, Qs, Ks, LD, tr, tc, D);
    tile_dot(dp, Os, Vs, LD, tr, tc, D);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int qi = q0 + tr + 16 * a;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int kj = k0 + tc + 16 * c;
        const float s = sc[a][c] * scale;
        const float x = logit(s, qi, kj, gs[tc + 16 * c], L, causal);
        const float p = x == -INFINITY ? 0.f : expf(x - lr[a]);
        Ws[(tr + 16 * a) * kLDT + tc + 16 * c] =
            p * (dp[a][c] - dr[a]) + (stat_valid(qi, kj, len, causal) ? c_st * (s - mean) : 0.f);
      }
    }
    __syncthreads();
    tile_acc(acc, Ws, Ks, LD, tr, dcol);
  }
  store_rows<T>(dq + bh * L * D, acc, q0, tr, tc, L, D, scale);
}

template <typename T>
cudaError_t train_fwd_t(const SattnTrainArgs& a, cudaStream_t s) {
  const int H = a.H, L = a.L, D = a.D, nt = (L + kPT - 1) / kPT;
  const size_t LDf = (size_t)(D + 4);
  const size_t sm_stats = 2 * kPT * LDf * sizeof(float);
  const size_t sm_fwd = (3 * kPT * LDf + kPT * kLDT + kPT) * sizeof(float);
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(sattn_train_stats_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sm_stats)))
    return e;
  if ((e = cudaFuncSetAttribute(sattn_train_fwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_fwd)))
    return e;
  const dim3 grid((unsigned)nt, (unsigned)H, (unsigned)a.B);
  sattn_train_stats_kernel<T><<<grid, 256, sm_stats, s>>>((const T*)a.q, (const T*)a.k, a.lengths, H, L, D, a.scale,
                                                          a.causal, a.part);
  if ((e = cudaGetLastError())) return e;
  sattn_train_stats_fin_kernel<<<(unsigned)H, 256, 0, s>>>(a.part, a.lengths, a.B, H, L, nt, a.causal, a.stats);
  if ((e = cudaGetLastError())) return e;
  const long long n = (long long)a.B * H * L;
  sattn_train_gate_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const T*)a.gate, a.lengths, a.stats, H, L, n,
                                                                         a.penalty, a.lg);
  if ((e = cudaGetLastError())) return e;
  sattn_train_fwd_kernel<T><<<grid, 256, sm_fwd, s>>>((const T*)a.q, (const T*)a.k, (const T*)a.v, a.lg, (T*)a.out,
                                                      a.lse, H, L, D, a.scale, a.causal);
  return cudaGetLastError();
}

template <typename T>
cudaError_t train_bwd_t(const SattnTrainArgs& a, const void* dout, void* dq, void* dk, void* dv, void* dgate,
                        cudaStream_t s) {
  const int H = a.H, L = a.L, D = a.D, nt = (L + kPT - 1) / kPT;
  const size_t LDf = (size_t)(D + 4);
  const size_t sm_kv = (4 * kPT * LDf + kPT * kLDT + 2 * kPT) * sizeof(float);
  const size_t sm_q = (4 * kPT * LDf + kPT * kLDT + kPT) * sizeof(float);
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(sattn_train_bwd_kv_kernel<T, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sm_kv)))
    return e;
  if ((e = cudaFuncSetAttribute(sattn_train_bwd_kv_kernel<T, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sm_kv)))
    return e;
  if ((e = cudaFuncSetAttribute(sattn_train_bwd_q_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_q)))
    return e;
  const long long rows = (long long)a.B * H * L;
  sattn_train_rowdot_kernel<T><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>((const T*)dout, (const T*)a.out, rows, D,
                                                                          a.Di);
  if ((e = cudaGetLastError())) return e;
  const dim3 grid((unsigned)nt, (unsigned)H, (unsigned)a.B);
  sattn_train_bwd_kv_kernel<T, 0><<<grid, 256, sm_kv, s>>>((const T*)a.q, (const T*)a.k, (const T*)a.v,
                                                           (const T*)dout, a.lg, a.lse, a.Di, a.stats, a.lengths, H,
                                                           L, D, a.scale, a.causal, (T*)dv, a.dlg);
  if ((e = cudaGetLastError())) return e;
  sattn_train_bwd_fin_kernel<T><<<(unsigned)H, 256, 0, s>>>((const T*)a.gate, a.lengths, a.dlg, a.B, H, L, a.penalty,
                                                            a.stats, (T*)dgate);
  if ((e = cudaGetLastError())) return e;
  sattn_train_bwd_kv_kernel<T, 1><<<grid, 256, sm_kv, s>>>((const T*)a.q, (const T*)a.k, (const T*)a.v,
                                                           (const T*)dout, a.lg, a.lse, a.Di, a.stats, a.lengths, H,
                                                           L, D, a.scale, a.causal, (T*)dk, nullptr);
  if ((e = cudaGetLastError())) return e;
  sattn_train_bwd_q_kernel<T><<<grid, 256, sm_q, s>>>((const T*)a.q, (const T*)a.k, (const T*)a.v, (const T*)dout,
                                                      a.lg, a.lse, a.Di, a.stats, a.lengths, H, L, D, a.scale,
                                                      a.causal, (T*)dq);
  return cudaGetLastError();
}


// ============================================================================ tensor cores
// 16-bit inputs with head_dim 64: the same passes on tcgen05, 128 x 128 tiles moved by TMA
// (128-byte swizzle), products in TMEM, thread = TMEM lane = row of the CTA's own tile.
//   stats_tc  S = Q K^T per key tile, the valid scores' sums from the TMEM rows
//   (forward attention: the pipelined prefill kernel with lse, sattn.cu)
//   bwd_tc    MODE 0 (per key tile): S^T = K Q^T, dP^T = V dO^T -> P^T, dS^T (softmax part)
//             and the centred valid scores (S - mean)^T; dv += P^T dO, dk_s += dS^T Q,
//             g += (S - mean)^T Q (TS form, the 16-bit operands from TMEM), dlg from the rows;
//             dk = scale (dk_s + c g) once c is known (combine kernel);
//             MODE 2 (per query tile): S = Q K^T, dP = dO V^T -> dS_total; dq += dS_total K
// Every wait is bounded; a CTA that gives up records a site code and skips its remaining
// work (its MMAs and copies in flight are waited for, bounded, before TMEM is released).
constexpr unsigned int kSiteTrTma = 0x331, kSiteTrMma = 0x332;
constexpr int kTrTile = 128 * 128;  // bytes of a 128-row x 64-column 16-bit tile

constexpr size_t kStSmem = 1024 + 3 * kTrTile + 64;

template <typename T>
__global__ void __launch_bounds__(128) sattn_train_stats_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                                   const __grid_constant__ CUtensorMap tm_k,
                                                                   const int64_t* __restrict__ lengths, int H, int L,
                                                                   float scale, int causal, double* part) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smraw[];
  uint8_t* base = align1024_shared(smraw);
  uint8_t* sQ = base;
  auto sK = [&](int st) { return base + kTrTile * (1 + st); };
  __shared__ uint64_t bars[5];  // Q, K[2], S[2]
  __shared__ uint32_t tslot[1];
  __shared__ double red[8];
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int qt = blockIdx.y, bh = blockIdx.x;
  const int b = bh / H;
  const int len = row_len(lengths, b, L);
  const int q0 = 128 * qt, tid = threadIdx.x, warp = tid >> 5;
  float s1 = 0.f, s2 = 0.f;
  const int nk = q0 >= len ? 0 : (causal ? min(q0 + 127, len - 1) / 128 + 1 : (len + 127) / 128);
  if (nk > 0) {
    if (tid == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      for (int i = 0; i < 5; ++i) mbar_init(bar(i), 1);
      fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(tslot), 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t tl = (uint32_t)(warp * 32) << 16;
    constexpr uint32_t ID = idesc_f16(128, 128, BF16, false, false);
    int k_iss[2] = {0, 0}, k_wt[2] = {0, 0}, s_iss[2] = {0, 0}, s_wt[2] = {0, 0};  // thread 0's books
    bool ok = true;
    auto issue_mma = [&](int j) -> bool {  // thread 0: S_(j % 2) = Q K_j^T once K_j has landed
      const int st = j & 1;
      if (!mbar_wait(bar(1 + st), k_wt[st] & 1, kSiteTrTma)) return false;
      ++k_wt[st];
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_f16(tmem + 128 * st, sdesc_sw128(smem_u32(sQ) + 32 * ks, 16, 1024),
                 sdesc_sw128(smem_u32(sK(st)) + 32 * ks, 16, 1024), ID, ks > 0 ? 1u : 0u);
      umma_commit(bar(3 + st));
      ++s_iss[st];
      return true;
    };
    if (tid == 0) {
      mbar_expect_tx(bar(0), (uint32_t)kTrTile);
      tma_load_3d(smem_u32(sQ), &tm_q, 0, q0, bh, bar(0));
      for (int j = 0; j < 2 && j < nk; ++j) {
        mbar_expect_tx(bar(1 + j), (uint32_t)kTrTile);
        tma_load_3d(smem_u32(sK(j)), &tm_k, 0, 128 * j, bh, bar(1 + j));
        ++k_iss[j];
      }
      ok = mbar_wait(bar(0), 0, kSiteTrTma) && issue_mma(0);
    }
    ok = __syncthreads_and(ok) != 0;
    const int qi = q0 + tid;
    for (int j = 0; j < nk && ok; ++j) {
      const int st = j & 1;
      if (tid == 0 && j + 1 < nk) ok = issue_mma(j + 1);
      const bool got = mbar_wait(bar(3 + st), (j >> 1) & 1, kSiteTrMma);
      if (tid == 0 && got) {
        ++s_wt[st];
        if (j + 2 < nk) {  // K stage st is free once S_j is complete
          mbar_expect_tx(bar(1 + st), (uint32_t)kTrTile);
          tma_load_3d(smem_u32(sK(st)), &tm_k, 0, 128 * (j + 2), bh, bar(1 + st));
          ++k_iss[st];
        }
      }
      ok = __syncthreads_and(ok && got) != 0;
      if (!ok) break;
      tc_fence_after();
      const int k0 = 128 * j;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + tl + 128 * st + 32 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (stat_valid(qi, k0 + 32 * c + e, len, causal)) {
            const float x = __uint_as_float(v[e]) * scale;
            s1 += x;
            s2 = fmaf(x, x, s2);
          }
        }
      }
      tc_fence_before();
      __syncthreads();  // S_(j % 2) read before S_(j + 2) overwrites it
    }
    if (tid == 0) {  // nothing may still be in flight when TMEM and the CTA go away (bounded)
      for (int st = 0; st < 2; ++st) {
        while (s_wt[st] < s_iss[st] && mbar_wait(bar(3 + st), s_wt[st] & 1, kSiteTrMma)) ++s_wt[st];
        while (k_wt[st] < k_iss[st] && mbar_wait(bar(1 + st), k_wt[st] & 1, kSiteTrTma)) ++k_wt[st];
      }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);
  }
  const double t1 = block_sum256<double, 4>((double)s1, red);
  const double t2 = block_sum256<double, 4>((double)s2, red);
  if (tid == 0) {
    const long long idx = ((long long)bh * gridDim.y + qt) * 2;
    part[idx] = t1;
    part[idx + 1] = t2;
  }
}

constexpr int kBtThreads = 256;
constexpr size_t kBtSmem = 1024 + 6 * kTrTile + 64;

template <typename T, int MODE>
__global__ void __launch_bounds__(kBtThreads, 1) sattn_train_bwd_tc_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
    const float* __restrict__ lg, const float* __restrict__ lse, const float* __restrict__ Di,
    const float* __restrict__ stats, const int64_t* __restrict__ lengths, int H, int L, float scale, int causal,
    T* __restrict__ outg, float* __restrict__ dlg, float* __restrict__ dkb, float* __restrict__ gk) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr bool KEYS = MODE == 0;  // the CTA's own tile is a key tile
  extern __shared__ uint8_t smraw[];
  uint8_t* base = align1024_shared(smraw);
  uint8_t* own1 = base;            // K (key-major) or Q
  uint8_t* own2 = base + kTrTile;  // V or dO
  auto oth1 = [&](int st) { return base + kTrTile * (2 + 2 * st); };  // Q or K
  auto oth2 = [&](int st) { return base + kTrTile * (3 + 2 * st); };  // dO or V
  __shared__ float colA[2][128], colB[2][128];  // per stage: lse, D_i of the queries (keys: log-gates)
  __shared__ float red[2][128];
  __shared__ uint64_t bars[4];  // own, other[2], mma
  __shared__ uint32_t tslot[1];
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int nt = (L + 127) / 128;
  // causal: the tiles with the most partners first (key tile 0, query tile nt - 1)
  const int bh = blockIdx.x, own = KEYS || !causal ? (int)blockIdx.y : nt - 1 - (int)blockIdx.y;
  const int b = bh / H, h = bh - b * H;
  const int len = row_len(lengths, b, L);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = (warp & 3) * 32 + lane, hc = warp >> 2;
  const uint32_t tl = (uint32_t)((warp & 3) * 32) << 16;
  const int o0 = 128 * own, o = o0 + r;
  const int t_begin = KEYS ? (causal ? own : 0) : 0;
  const int t_end = KEYS ? nt : (causal ? own + 1 : nt);
  const int cnt = t_end - t_begin;
  const float mean = stats[h * 4], c_st = stats[h * 4 + 3];
  const long long rowbase = (long long)bh * L;
  // this thread's row values
  const float g_row = KEYS && o < L ? lg[rowbase + o] : -INFINITY;
  const float lse_row = !KEYS && o < L ? lse[rowbase + o] : 0.f;
  const float di_row = !KEYS && o < L ? Di[rowbase + o] : 0.f;
  auto load_cols = [&](int st, int t) {  // per-column values of other tile t (threads < 128)
    if (tid < 128) {
      const int x = 128 * t + tid;
      if (KEYS) {
        colA[st][tid] = x < L ? lse[rowbase + x] : 0.f;
        colB[st][tid] = x < L ? Di[rowbase + x] : 0.f;
      } else {
        colA[st][tid] = x < L ? lg[rowbase + x] : -INFINITY;
      }
    }
  };
  if (tid == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_do);
    for (int i = 0; i < 4; ++i) mbar_init(bar(i), 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(smem_u32(tslot), 512);
  load_cols(0, t_begin);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // MODE 0: dv at T_ACC, the dk parts at T_DK, T_G; MODE 2: dS_total at T_W, dq at T_ACC
  constexpr uint32_t T_S = 0, T_DP = 128, T_W = 256, T_ACC = MODE == 0 ? 256 : 320, T_DK = 320, T_G = 384;
  constexpr uint32_t ID_SS = idesc_f16(128, 128, BF16, false, false);
  constexpr uint32_t ID_ACC = idesc_f16(128, 64, BF16, false, true);
  const CUtensorMap* m_own1 = KEYS ? &tm_k : &tm_q;
  const CUtensorMap* m_own2 = KEYS ? &tm_v : &tm_do;
  const CUtensorMap* m_oth1 = KEYS ? &tm_q : &tm_k;
  const CUtensorMap* m_oth2 = KEYS ? &tm_do : &tm_v;
  int ld_iss[2] = {0, 0}, ld_wt[2] = {0, 0}, mma_iss = 0, mma_wt = 0;  // thread 0's books
  if (tid == 0) {
    mbar_expect_tx(bar(0), 2u * kTrTile);
    tma_load_3d(smem_u32(own1), m_own1, 0, o0, bh, bar(0));
    tma_load_3d(smem_u32(own2), m_own2, 0, o0, bh, bar(0));
    mbar_expect_tx(bar(1), 2u * kTrTile);
    tma_load_3d(smem_u32(oth1(0)), m_oth1, 0, 128 * t_begin, bh, bar(1));
    tma_load_3d(smem_u32(oth2(0)), m_oth2, 0, 128 * t_begin, bh, bar(1));
    ++ld_iss[0];
  }
  bool ok = __syncthreads_and(mbar_wait(bar(0), 0, kSiteTrTma)) != 0;
  float dl = 0.f;
  for (int u = 0; u < cnt && ok; ++u) {
    const int st = u & 1, t = t_begin + u, x0 = 128 * t;
    if (u + 1 < cnt) {  // prefetch the next other tile into the stage MMA3(u - 1) released
      if (tid == 0) {
        const int sn = st ^ 1;
        mbar_expect_tx(bar(1 + sn), 2u * kTrTile);
        tma_load_3d(smem_u32(oth1(sn)), m_oth1, 0, x0 + 128, bh, bar(1 + sn));
        tma_load_3d(smem_u32(oth2(sn)), m_oth2, 0, x0 + 128, bh, bar(1 + sn));
        ++ld_iss[sn];
      }
      load_cols(st ^ 1, t + 1);
    }
    bool got = mbar_wait(bar(1 + st), (u >> 1) & 1, kSiteTrTma);
    if (tid == 0 && got) ++ld_wt[st];
    ok = __syncthreads_and(got) != 0;
    if (!ok) break;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        umma_f16(tmem + T_S, sdesc_sw128(smem_u32(own1) + 32 * ks, 16, 1024),
                 sdesc_sw128(smem_u32(oth1(st)) + 32 * ks, 16, 1024), ID_SS, ks > 0 ? 1u : 0u);
        umma_f16(tmem + T_DP, sdesc_sw128(smem_u32(own2) + 32 * ks, 16, 1024),
                 sdesc_sw128(smem_u32(oth2(st)) + 32 * ks, 16, 1024), ID_SS, ks > 0 ? 1u : 0u);
      }
      umma_commit(bar(3));
      ++mma_iss;
    }
    got = mbar_wait(bar(3), mma_wt & 1, kSiteTrMma);
    if (got) ++mma_wt;  // the same count in every thread while nothing fails
    ok = __syncthreads_and(got) != 0;
    if (!ok) break;
    tc_fence_after();
    // this thread's 64 columns, as 16-bit pairs into TMEM. MODE 0 writes three operands over
    // the S / dP columns it has already read (P and dS into its S half, the centred scores
    // into its dP half: chunk cc of half hc lands at S + 64 hc + 32 cc, dP + 64 hc + 16 cc);
    // MODE 2 writes dS_total into T_W.
#pragma unroll 1
    for (int cc = 0; cc < 2; ++cc) {
      const int c0 = 64 * hc + 32 * cc;
      uint32_t sv[32], pv[32];
      tmem_ld32(tmem + tl + T_S + c0, sv);
      tmem_ld32(tmem + tl + T_DP + c0, pv);
      tmem_wait_ld();
      uint32_t pk[16], pd[16], pg[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float wp[2], wd[2], wg[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int c = c0 + e + q, x = x0 + c;
          const int kj = KEYS ? o : x, qi = KEYS ? x : o;
          const float s = __uint_as_float(sv[e + q]) * scale;
          const float g = KEYS ? g_row : colA[st][c];
          const float lq = KEYS ? colA[st][c] : lse_row;
          const float dq = KEYS ? colB[st][c] : di_row;
          const float lgt = logit(s, qi, kj, g, L, causal);
          const float p = lgt == -INFINITY ? 0.f : __expf(lgt - lq);
          const float dsm = p * (__uint_as_float(pv[e + q]) - dq);
          const bool valid = stat_valid(qi, kj, len, causal);
          if (MODE == 0) {
            if (kj != qi) dl += dsm;
            wp[q] = p;
            wd[q] = dsm;
            wg[q] = valid ? s - mean : 0.f;
          } else {
            wp[q] = dsm + (valid ? c_st * (s - mean) : 0.f);
          }
        }
        pk[e >> 1] = pack2<T>(wp[0], wp[1]);
        if (MODE == 0) {
          pd[e >> 1] = pack2<T>(wd[0], wd[1]);
          pg[e >> 1] = pack2<T>(wg[0], wg[1]);
        }
      }
      if (MODE == 0) {
        tmem_st16(tmem + tl + T_S + (uint32_t)c0, pk);
        tmem_st16(tmem + tl + T_S + (uint32_t)c0 + 16, pd);
        tmem_st16(tmem + tl + T_DP + (uint32_t)(64 * hc + 16 * cc), pg);
      } else {
        tmem_st16(tmem + tl + T_W + (uint32_t)(c0 >> 1), pk);
      }
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      if (MODE == 0) {
        // K step ks covers other columns 16 ks .. 16 ks + 15: half ks / 4, chunk (ks / 2) % 2
        const uint32_t bo = smem_u32(oth2(st)), bq = smem_u32(oth1(st));
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t hh = ks >> 2, cq = (ks >> 1) & 1, sub = ks & 1;
          const uint32_t aP = T_S + 64 * hh + 32 * cq + 8 * sub, aG = T_DP + 64 * hh + 16 * cq + 8 * sub;
          const uint32_t acc = (u > 0 || ks > 0) ? 1u : 0u;
          umma_f16_ts(tmem + T_ACC, tmem + aP, sdesc_sw128(bo + 2048 * ks, 16, 1024), ID_ACC, acc);
          umma_f16_ts(tmem + T_DK, tmem + aP + 16, sdesc_sw128(bq + 2048 * ks, 16, 1024), ID_ACC, acc);
          umma_f16_ts(tmem + T_G, tmem + aG, sdesc_sw128(bq + 2048 * ks, 16, 1024), ID_ACC, acc);
        }
      } else {
        const uint32_t b3 = smem_u32(oth1(st));
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_f16_ts(tmem + T_ACC, tmem + T_W + 8 * ks, sdesc_sw128(b3 + 2048 * ks, 16, 1024), ID_ACC,
                      (u > 0 || ks > 0) ? 1u : 0u);
      }
      umma_commit(bar(3));
      ++mma_iss;
    }
    got = mbar_wait(bar(3), mma_wt & 1, kSiteTrMma);  // TMEM operands and the stage are free afterwards
    if (got) ++mma_wt;
    ok = __syncthreads_and(got) != 0;
    tc_fence_after();
  }
  if (ok) {
    uint32_t av[32];
    tmem_ld32(tmem + tl + T_ACC + 32 * hc, av);
    tmem_wait_ld();
    if (o < L) {
      const float mul = MODE == 0 ? 1.f : scale;
      uint4* dst = reinterpret_cast<uint4*>(outg + (rowbase + o) * 64 + 32 * hc);
#pragma unroll
      for (int e = 0; e < 32; e += 8)
        dst[e >> 3] = make_uint4(pack2<T>(__uint_as_float(av[e]) * mul, __uint_as_float(av[e + 1]) * mul),
                                 pack2<T>(__uint_as_float(av[e + 2]) * mul, __uint_as_float(av[e + 3]) * mul),
                                 pack2<T>(__uint_as_float(av[e + 4]) * mul, __uint_as_float(av[e + 5]) * mul),
                                 pack2<T>(__uint_as_float(av[e + 6]) * mul, __uint_as_float(av[e + 7]) * mul));
    }
    if (MODE == 0) {
      // dk's two fp32 parts (the softmax term and the statistics one, whose coefficient the
      // next kernel computes), then dlg
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        tmem_ld32(tmem + tl + (part ? T_G : T_DK) + 32 * hc, av);
        tmem_wait_ld();
        if (o < L) {
          float4* dst = reinterpret_cast<float4*>((part ? gk : dkb) + (rowbase + o) * 64 + 32 * hc);
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            dst[e >> 2] = make_float4(__uint_as_float(av[e]), __uint_as_float(av[e + 1]), __uint_as_float(av[e + 2]),
                                      __uint_as_float(av[e + 3]));
        }
      }
      red[hc][r] = dl;
      __syncthreads();
      if (hc == 0 && o < L) dlg[rowbase + o] = red[0][r] + red[1][r];
    }
  } else if (tid == 0) {  // let what is in flight land before TMEM and the CTA go away (bounded)
    while (mma_wt < mma_iss && mbar_wait(bar(3), mma_wt & 1, kSiteTrMma)) ++mma_wt;
    for (int st = 0; st < 2; ++st)
      while (ld_wt[st] < ld_iss[st] && mbar_wait(bar(1 + st), ld_wt[st] & 1, kSiteTrTma)) ++ld_wt[st];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// dk = scale (dk_s + c g) per element (head_dim 64; four elements a thread).
template <typename T>
__global__ void __launch_bounds__(256) sattn_train_dk_combine_kernel(const float* __restrict__ dkb,
                                                                     const float* __restrict__ gk,
                                                                     const float* __restrict__ stats, int H, int L,
                                                                     long long n4, float scale, T* __restrict__ dk) {
  const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
  if (i >= n4) return;
  const int h = (int)((i / (16ll * L)) % H);
  const float c = stats[h * 4 + 3];
  const float4 a = reinterpret_cast<const float4*>(dkb)[i];
  const float4 g = reinterpret_cast<const float4*>(gk)[i];
  const uint32_t lo = pack2<T>(scale * fmaf(c, g.x, a.x), scale * fmaf(c, g.y, a.y));
  const uint32_t hi = pack2<T>(scale * fmaf(c, g.z, a.z), scale * fmaf(c, g.w, a.w));
  reinterpret_cast<uint2*>(dk)[i] = make_uint2(lo, hi);
}

bool train_maps(CUtensorMap* m, const void* p, bool bf16, int L, long long bhn) {
  return make_map_3d(m, p, bf16, 64, (uint64_t)L, (uint64_t)bhn, 64, 128, 1);
}

template <typename T>
cudaError_t train_fwd_tc_t(const SattnTrainArgs& a, cudaStream_t s) {
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const long long bhn = (long long)a.B * a.H;
  const int nt = (a.L + 127) / 128;
  CUtensorMap mq, mk;
  if (!train_maps(&mq, a.q, bf16, a.L, bhn) || !train_maps(&mk, a.k, bf16, a.L, bhn)) return cudaErrorInvalidValue;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(sattn_train_stats_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kStSmem)))
    return e;
  sattn_train_stats_tc_kernel<T><<<dim3((unsigned)bhn, (unsigned)nt), 128, kStSmem, s>>>(mq, mk, a.lengths, a.H, a.L,
                                                                                         a.scale, a.causal, a.part);
  if ((e = cudaGetLastError())) return e;
  sattn_train_stats_fin_kernel<<<(unsigned)a.H, 256, 0, s>>>(a.part, a.lengths, a.B, a.H, a.L, nt, a.causal, a.stats);
  if ((e = cudaGetLastError())) return e;
  const long long n = bhn * a.L;
  sattn_train_gate_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, s>>>((const T*)a.gate, a.lengths, a.stats, a.H,
                                                                         a.L, n, a.penalty, a.lg);
  if ((e = cudaGetLastError())) return e;
  return launch_sattn_attn_fa(a.q, a.k, a.v, a.lg, a.out, a.lse, a.B, a.H, a.L, a.scale, a.dtype, a.causal, s);
}

template <typename T>
cudaError_t train_bwd_tc_t(const SattnTrainArgs& a, const void* dout, void* dq, void* dk, void* dv, void* dgate,
                           cudaStream_t s) {
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const long long bhn = (long long)a.B * a.H;
  const int nt = (a.L + 127) / 128;
  CUtensorMap mq, mk, mv, mo;
  if (!train_maps(&mq, a.q, bf16, a.L, bhn) || !train_maps(&mk, a.k, bf16, a.L, bhn) ||
      !train_maps(&mv, a.v, bf16, a.L, bhn) || !train_maps(&mo, dout, bf16, a.L, bhn))
    return cudaErrorInvalidValue;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(sattn_train_bwd_tc_kernel<T, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kBtSmem)) ||
      (e = cudaFuncSetAttribute(sattn_train_bwd_tc_kernel<T, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kBtSmem)))
    return e;
  const long long rows = bhn * a.L;
  sattn_train_rowdot_kernel<T><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>((const T*)dout, (const T*)a.out, rows, 64,
                                                                          a.Di);
  if ((e = cudaGetLastError())) return e;
  const dim3 grid((unsigned)bhn, (unsigned)nt);
  sattn_train_bwd_tc_kernel<T, 0><<<grid, kBtThreads, kBtSmem, s>>>(mq, mk, mv, mo, a.lg, a.lse, a.Di, a.stats,
                                                                    a.lengths, a.H, a.L, a.scale, a.causal, (T*)dv,
                                                                    a.dlg, a.dkb, a.gk);
  if ((e = cudaGetLastError())) return e;
  sattn_train_bwd_fin_kernel<T><<<(unsigned)a.H, 256, 0, s>>>((const T*)a.gate, a.lengths, a.dlg, a.B, a.H, a.L,
                                                              a.penalty, a.stats, (T*)dgate);
  if ((e = cudaGetLastError())) return e;
  const long long n4 = rows * 16;  // float4 groups of dk
  sattn_train_dk_combine_kernel<T><<<(unsigned)((n4 + 255) / 256), 256, 0, s>>>(a.dkb, a.gk, a.stats, a.H, a.L, n4,
                                                                                a.scale, (T*)dk);
  if ((e = cudaGetLastError())) return e;
  sattn_train_bwd_tc_kernel<T, 2><<<grid, kBtThreads, kBtSmem, s>>>(mq, mk, mv, mo, a.lg, a.lse, a.Di, a.stats,
                                                                    a.lengths, a.H, a.L, a.scale, a.causal, (T*)dq,
                                                                    nullptr, nullptr, nullptr);
  return cudaGetLastError();
}
}  // namespace

bool sattn_train_supported(int D) { return D == 16 || D == 32 || D == 64 || D == 128; }

bool sattn_train_tc_supported(int D, int dtype) { return D == 64 && dtype != SSD_F32; }

cudaError_t launch_sattn_train_fwd(const SattnTrainArgs& a, cudaStream_t s) {
  if (a.use_tc) {
    if (!sattn_train_tc_supported(a.D, a.dtype) || (long long)a.B * a.H > 0x7fffffffll || (a.L + 127) / 128 > 65535)
      return cudaErrorInvalidValue;
    return a.dtype == SSD_BF16 ? train_fwd_tc_t<__nv_bfloat16>(a, s) : train_fwd_tc_t<__half>(a, s);
  }
  switch (a.dtype) {
    case SSD_F32: return train_fwd_t<float>(a, s);
    case SSD_BF16: return train_fwd_t<__nv_bfloat16>(a, s);
    case SSD_F16: return train_fwd_t<__half>(a, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_sattn_train_bwd(const SattnTrainArgs& a, const void* dout, void* dq, void* dk, void* dv,
                                   void* dgate, cudaStream_t s) {
  if (a.use_tc) {
    if (!sattn_train_tc_supported(a.D, a.dtype) || (long long)a.B * a.H > 0x7fffffffll || (a.L + 127) / 128 > 65535)
      return cudaErrorInvalidValue;
    return a.dtype == SSD_BF16 ? train_bwd_tc_t<__nv_bfloat16>(a, dout, dq, dk, dv, dgate, s)
                               : train_bwd_tc_t<__half>(a, dout, dq, dk, dv, dgate, s);
  }
  switch (a.dtype) {
    case SSD_F32: return train_bwd_t<float>(a, dout, dq, dk, dv, dgate, s);
    case SSD_BF16: return train_bwd_t<__nv_bfloat16>(a, dout, dq, dk, dv, dgate, s);
    case SSD_F16: return train_bwd_t<__half>(a, dout, dq, dk, dv, dgate, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ssdb200
