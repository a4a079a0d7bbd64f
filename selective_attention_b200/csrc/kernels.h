// kernels.h - host-side launch interface between the C ABI (api.cu) and the
// kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace ssdb200 {

struct LaunchCtx {
  cudaStream_t stream;
  ChunkMap cm;
  int nchunks_max;  // grid extent over chunks (exact in padded mode, an upper bound in packed mode)
  int nrows;        // batch rows (padded) or sequences (packed)
  int H, P, N, G, cs;
  long long T;      // total tokens (b * L)
  int use_sp;
  float dmin, dmax;
};

// ssd_simt.cu
cudaError_t launch_chunk_cumsum(const LaunchCtx& c, int dt_dtype, const float* A, const void* delta_raw,
                                const float* delta_bias, float* dt, float* cum);
cudaError_t launch_state_passing(const LaunchCtx& c, float* states, void* prev16, int prev_dtype,
                                 const float* cum, const float* h_init, float* h_last);
cudaError_t launch_build_chunk_table(cudaStream_t s, const void* cu, int cu64, int nseq, int cs, ChunkEntry* table,
                                     int2* rows, int* count);
cudaError_t launch_simt_chunk_state(const LaunchCtx& c, int x_dtype, const void* u, const void* B,
                                    const float* dt, const float* cum, float* states);
cudaError_t launch_simt_bmm_chunk(const LaunchCtx& c, int x_dtype, const void* B, const void* C, float* CB);
cudaError_t launch_simt_chunk_scan(const LaunchCtx& c, int x_dtype, int y_dtype, const void* u, const float* dt,
                                   const float* cum, const void* C, const float* prev, const float* CB,
                                   const float* D, const void* z, void* y);
unsigned int fetch_error_simt(cudaStream_t s);

// ssd_bwd.cu (CUDA-core backward; P <= 64, N <= 128 (multiples of 8), chunk 32..256 in steps of 32)
struct BwdArgs {
  int x_dtype, dt_dtype, y_dtype;
  const void* u;
  const float* A;
  const void* B;
  const void* C;
  const void* delta_raw;
  const float* delta_bias;
  const float* h_init;
  const void* y_grad;
  const float* h_last_grad;
  void* u_grad;
  float* A_grad;
  float* B_grad;
  float* C_grad;
  void* delta_raw_grad;
  float* delta_bias_grad;
  float* h_init_grad;
  // workspace
  float *dt, *cum, *states, *hg, *CB, *CBg, *accS, *gC, *dl_part, *A_part, *bias_part;
  float* rows4;  // (4, chunks, H, cs): ddt, gB, row and column decay sums of the tensor-core intra kernel
  // tensor-core path: 16-bit copies (the inputs' type) of prev and hg (chunks, H, P, N) and,
  // when y_grad is fp32, of y_grad (b, L, H, P)
  uint16_t *prev16, *hg16, *y16;
  // fp32 inputs at P 64, N 128, cs 256: B and C split into the bf16 hi / lo tiles of the
  // split-bf16 chunk_state (ssd_split.cu), which recomputes the chunk states and HG
  void *Bs_split, *Cs_split;
  float* accY;  // (chunks, H, cs, P): the intra-chunk product from split_bwd_accy
  float* Gyu;   // (chunks, H, cs, cs): y_grad u^T from split_bwd_g (lower blocks)
  cudaEvent_t ev[6];
};
bool bwd_supported(int P, int N, int cs);
size_t bwd_dl_slices(int P, int N);
cudaError_t launch_ssd_bwd(const LaunchCtx& c, const BwdArgs& a);
// ssd_bwd_tc.cu (the backward contractions on tcgen05: 16-bit u / B / C, P 64, N 128, chunk 256)
bool bwd_state_grad_tc_supported(int x_dtype, int y_dtype, int P, int N, int cs);
cudaError_t launch_bwd_chunk_states_tc(const LaunchCtx& c, const BwdArgs& a);  // same shapes
cudaError_t launch_bwd_intra_tc(const LaunchCtx& c, const BwdArgs& a);         // same shapes; fills rows4
// per (chunk, group, half) over the group's heads: B_grad / C_grad summed in TMEM (needs prev16,
// hg16 from the state pass and, for fp32 y_grad, y16 from the recompute)
cudaError_t launch_bwd_state_grad_grp_tc(const LaunchCtx& c, const BwdArgs& a);
cudaError_t launch_bwd_cb_tc(const LaunchCtx& c, const BwdArgs& a);   // CB = C B^T, lower 128-row blocks
cudaError_t launch_bwd_bmm_tc(const LaunchCtx& c, const BwdArgs& a);  // CB_grad products into B_grad / C_grad
unsigned int fetch_error_bwd_tc(cudaStream_t s);

// sattn.cu (selective-attention decode step; head_dim 8..256, a power of two)
bool sattn_decode_supported(int D);
cudaError_t launch_sattn_decode(const void* q, const void* k, const void* v, const float* lg, void* kc, void* vc,
                                float* lgc, long long widx, long long cap, void* out, long long bh, int D,
                                float scale, int dtype, cudaStream_t s);
bool sattn_prefill_supported(int D);
bool sattn_prefill_tc_supported(int D, int dtype);
// use_tc: tcgen05 kernel (16-bit inputs, D 64 or 128); otherwise the CUDA-core kernel.
cudaError_t launch_sattn_prefill(const void* q, const void* k, const void* v, const float* lg, void* out, int b, int H,
                                 int L, int D, float scale, int dtype, int use_tc, cudaStream_t s);
unsigned int fetch_error_sattn(cudaStream_t s);
// The pipelined tensor-core attention (16-bit, head_dim 64) with the row log-sum-exp written
// (lse may be null) and causal or bidirectional key ranges; used by the training forward.
cudaError_t launch_sattn_attn_fa(const void* q, const void* k, const void* v, const float* lg, void* out, float* lse,
                                 int b, int H, int L, float scale, int dtype, int causal, cudaStream_t s);

// sattn_train.cu (training-mode selective attention and its backward; CUDA cores)
struct SattnTrainArgs {
  int B, H, L, D, dtype, causal;
  int use_tc;  // tcgen05 kernels (16-bit inputs, head_dim 64)
  float scale, penalty;
  const void* q;
  const void* k;
  const void* v;
  const void* gate;
  const int64_t* lengths;
  void* out;
  float* lse;
  float* lg;
  float* stats;
  // workspace
  double* part;  // (B, H, L / 64, 2) per query tile (128 rows on tensor cores): sum, sum of squares
  float* Di;     // (B, H, L) dout . out
  float* dlg;    // (B, H, L) gradient of the log-gates
  float* dkb;    // (B, H, L, D) tensor-core path: the softmax part of dk (fp32)
  float* gk;     // (B, H, L, D) tensor-core path: sum_i (S - mean) q_i over the valid scores
};
bool sattn_train_supported(int D);
bool sattn_train_tc_supported(int D, int dtype);
cudaError_t launch_sattn_train_fwd(const SattnTrainArgs& a, cudaStream_t s);
cudaError_t launch_sattn_train_bwd(const SattnTrainArgs& a, const void* dout, void* dq, void* dk, void* dv,
                                   void* dgate, cudaStream_t s);

// ssd_tc.cu (tcgen05 + TMA; bf16/fp16 inputs, P = 64, N = 128, cs = 256; prev16 in the input type)
bool tc_supported(int x_dtype, int P, int N, int cs);
// delta_raw == NULL: dt / cum are inputs; otherwise chunk_cumsum is fused in and they are written.
cudaError_t launch_tc_chunk_state(const LaunchCtx& c, int x_dtype, int dt_dtype, const void* u, const void* B,
                                  const float* A, const void* delta_raw, const float* delta_bias, float* dt,
                                  float* cum, float* states, int* tmap_status);
// chunk_cumsum + chunk_state + state_passing in one kernel, one CTA per (row, head)
// chain: writes dt, cum, prev16 and h_last; the fp32 chunk states stay on chip.
cudaError_t launch_tc_state_pass(const LaunchCtx& c, int x_dtype, int dt_dtype, const void* u, const void* B,
                                 const float* A, const void* delta_raw, const float* delta_bias, float* dt,
                                 float* cum, void* prev16, const float* h_init, float* h_last, int* tmap_status);
cudaError_t launch_tc_chunk_scan(const LaunchCtx& c, int x_dtype, int y_dtype, const void* u, const float* A,
                                 const float* dt, const float* cum, const void* B, const void* C, const void* prev16,
                                 const float* D, const void* z, void* y, int* tmap_status);
unsigned int fetch_error_tc(cudaStream_t s);

// ssd_split.cu (tcgen05 with split-bf16 products for fp32 inputs and outputs, P = 64, N = 128,
// cs = 256). Operand tiles per (chunk, group), split into bf16 hi / lo and swizzled, read with
// bulk copies: split_b writes chunk_state's B tiles (4), bmm_chunk chunk_scan's masked CB (6)
// and C (4) tiles. chunk_state writes fp32 states, which state_passing turns into prev.
bool split_supported(int x_dtype, int y_dtype, int P, int N, int cs);
size_t split_operand_bytes_per_chunk_group();  // Bs + CBs + Cs
cudaError_t launch_split_b(const LaunchCtx& c, const float* B, void* Bs);
// mode 0: chunk states (the forward); mode 1: the backward's intra-chunk state gradient from
// y_grad (in place of u) and the C tiles (in place of B)
cudaError_t launch_split_chunk_state(const LaunchCtx& c, const float* u, const void* Bs, const float* dt,
                                     const float* cum, float* states, int mode = 0);
cudaError_t launch_split_bmm(const LaunchCtx& c, const float* B, const float* C, void* CBs, void* Cs);
cudaError_t launch_split_chunk_scan(const LaunchCtx& c, const float* u, const float* dt, const float* cum,
                                    const void* Cs, const float* prev, const void* CBs, const float* D,
                                    const float* z, float* y);
// The backward's state-side products for fp32 inputs (accS, B_grad / C_grad group sums by
// atomics, gC), as bwd_state_grad_kernel computes them
cudaError_t launch_split_state_grad(const LaunchCtx& c, const float* u, const float* B, const float* C,
                                    const float* y_grad, const float* dt, const float* cum, const float* prev,
                                    const float* hg, float* accS, float* B_grad, float* C_grad, float* gC);
// The backward's intra-chunk product accY for fp32 inputs (from the fp32 CB of bwd_cb), for
// bwd_intra_split
cudaError_t launch_split_bwd_accy(const LaunchCtx& c, const float* CB, const float* y_grad, const float* cum,
                                  float* accY);
// G = y_grad u^T per (chunk, head) for fp32 inputs, the lower 128 x 128 blocks, as fp32 rows
// [chunk][head][256][256] for bwd_intra_split
cudaError_t launch_split_bwd_g(const LaunchCtx& c, const float* u, const float* y_grad, float* G);
unsigned int fetch_error_split(cudaStream_t s);

// ssu.cu
cudaError_t launch_ssm_conv_prefill(const void* hbc, long long row_stride, const float* w, const float* bias,
                                    void* x, void* Bo, void* Co, void* ctx, const int64_t* lengths, int b, int L,
                                    int inner, int gn, int K, int dtype, cudaStream_t s);
cudaError_t launch_ssm_conv_decode(const void* hnew, long long row_stride, void* ctx, const float* w,
                                   const float* bias, void* x, void* Bo, void* Co, int b, int inner, int gn, int K,
                                   int dtype, cudaStream_t s);
cudaError_t launch_ssu(const void* u, const float* A, const void* B, const void* C, const void* delta_raw,
                       const float* delta_bias, void* h, void* y, const float* D, const void* z, int b, int H,
                       int P, int N, int G, int x_dtype, int dt_dtype, int h_dtype, int y_dtype, int use_sp,
                       float dmin, float dmax, cudaStream_t stream);
unsigned int fetch_error_ssu(cudaStream_t s);

}  // namespace ssdb200
