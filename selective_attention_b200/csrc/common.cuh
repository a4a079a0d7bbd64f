// common.cuh - dtype helpers, the chunk map and the device error flag shared by
// the SSD / SSU kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/ssd_b200.h"

namespace ssdb200 {

// ---------------------------------------------------------------------------
// Device error flag. Each translation unit has its own copy; the host reads and
// clears every unit's copy in ssd_b200_device_error(). Kernels never trap: when a
// bounded wait gives up they record a site code here and return.
// ---------------------------------------------------------------------------
static __device__ unsigned int g_err_flag;

__device__ __forceinline__ void record_error(unsigned int code) {
  atomicCAS(&g_err_flag, 0u, code);
}

// ---------------------------------------------------------------------------
// Element loads/stores in fp32 registers.
// ---------------------------------------------------------------------------
template <typename T> struct Ld;
template <> struct Ld<float> {
  static __device__ __forceinline__ float f(const float* p) { return *p; }
};
template <> struct Ld<__nv_bfloat16> {
  static __device__ __forceinline__ float f(const __nv_bfloat16* p) { return __bfloat162float(*p); }
};
template <> struct Ld<__half> {
  static __device__ __forceinline__ float f(const __half* p) { return __half2float(*p); }
};

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// Two fp32 values packed as one 32-bit word of the 16-bit type T.
template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t w);
// bf16 is the upper half of an fp32 word: widening is an exact bit move (integer
// pipe), which keeps the transcendental / conversion pipe free for tanh and exp.
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<__half2*>(&w));
}

// ---------------------------------------------------------------------------
// dt transform: d = delta_raw (+ bias); softplus below 20; clamp; the reference's
// ssd_scan/forward_kernel.py:68-79 and ssu/forward_kernel.py:121-131.
// softplus is log(exp(x) + 1) as triton_kernels/softplus.py:8 writes it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float dt_transform(float d, int use_softplus, float dmin, float dmax) {
  if (use_softplus && d <= 20.0f) d = logf(expf(d) + 1.0f);
  return fminf(fmaxf(d, dmin), dmax);
}

__device__ __forceinline__ float silu(float z) { return z / (1.0f + expf(-z)); }
// Same function through the fast intrinsics, for epilogues that round to 16 bits.
__device__ __forceinline__ float silu_fast(float z) { return __fdividef(z, 1.0f + __expf(-z)); }

// ---------------------------------------------------------------------------
// Chunk map: chunk k of the scan -> (row, chunk-in-row, first token, limits).
// Padded mode: k = row * nc + c over a (b, L) batch. Packed mode: a device table
// built from cu_seqlens; chunks never straddle sequences.
// ---------------------------------------------------------------------------
struct ChunkEntry {      // packed-mode table entry
  int row;              // sequence index
  int c;                // chunk index within the sequence
  long long tok0;       // first token (flattened)
  int lim;              // tokens of this chunk that belong to the sequence (<= cs)
  int pad;
};

struct ChunkMap {
  int packed;           // 0 padded, 1 packed
  int cs;               // chunk size
  int nc;               // padded: chunks per row
  long long L;          // padded: seq_len
  const long long* length;  // padded: per-row valid length or null
  const ChunkEntry* table;  // packed
  const int* count;         // packed: number of chunks in the table
  const int2* rows;         // packed: per-sequence {first chunk, number of chunks}
};

struct ChunkInfo {
  int row, c;
  long long tok0;
  int lim;     // rows < lim are tokens of this row (the reference's seq_len limit)
  int vlim;    // rows < vlim have dt != 0 (the reference's `length` limit)
};

__device__ __forceinline__ bool chunk_info(const ChunkMap& m, int k, ChunkInfo& ci) {
  if (!m.packed) {
    ci.row = k / m.nc;
    ci.c = k - ci.row * m.nc;
    long long start = (long long)ci.c * m.cs;
    ci.tok0 = (long long)ci.row * m.L + start;
    long long lim = m.L - start;
    ci.lim = (int)(lim < m.cs ? lim : m.cs);
    long long len = m.length ? m.length[ci.row] : m.L;
    if (len > m.L) len = m.L;
    long long v = len - start;
    ci.vlim = (int)(v < 0 ? 0 : (v < ci.lim ? v : ci.lim));
    return true;
  }
  if (k >= *m.count) return false;
  ChunkEntry e = m.table[k];
  ci.row = e.row;
  ci.c = e.c;
  ci.tok0 = e.tok0;
  ci.lim = e.lim;
  ci.vlim = e.lim;
  return true;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace ssdb200

// Per-translation-unit host accessor for the error flag, defined once per .cu.
#define SSDB200_DEFINE_ERROR_FETCH(fn_name)                                     \
  unsigned int fn_name(cudaStream_t s) {                                        \
    unsigned int v = 0, zero = 0;                                               \
    if (cudaStreamSynchronize(s) != cudaSuccess) return 0xFFFFFFFFu;            \
    cudaMemcpyFromSymbol(&v, ssdb200::g_err_flag, sizeof(v));                   \
    if (v) cudaMemcpyToSymbol(ssdb200::g_err_flag, &zero, sizeof(zero));        \
    return v;                                                                   \
  }
