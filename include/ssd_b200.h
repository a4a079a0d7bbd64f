/*
 * ssd_b200.h - C ABI of the B200 (sm_100a) SSD chunked-scan forward and the
 * single-token selective state update (SSU).
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream and returns an
 * ssd_status_t. Nothing here allocates device memory: the fused SSD forward
 * takes a caller-provided workspace sized by ssd_scan_fwd_workspace_size().
 * Tensors are dense row-major ("contiguous") in the shapes given below.
 *
 * Reference interfaces replaced (nmquan1503/selective-attention, paths under
 * src/selective_attention/):
 *   ssd_scan_fwd           <- triton_kernels/ssd_scan/forward.py:223 ssd_scan_forward
 *                             (called from ops/ssd_scan.py:70 SSDScanFn.forward)
 *   ssd_scan_bwd           <- triton_kernels/ssd_scan/backward.py:467 ssd_scan_backward
 *                             (called from ops/ssd_scan.py:91 SSDScanFn.backward)
 *   ssd_chunk_cumsum_fwd   <- triton_kernels/ssd_scan/forward.py:14  chunk_cumsum_forward
 *   ssd_chunk_state_fwd    <- triton_kernels/ssd_scan/forward.py:62  chunk_state_forward
 *   ssd_state_passing_fwd  <- triton_kernels/ssd_scan/forward.py:102 state_passing_forward
 *   ssd_bmm_chunk_fwd      <- triton_kernels/ssd_scan/forward.py:139 bmm_chunk_forward
 *   ssd_chunk_scan_fwd     <- triton_kernels/ssd_scan/forward.py:175 chunk_scan_forward
 *   ssu_fwd                <- triton_kernels/ssu/forward.py:7 ssu_forward
 *                             (called from ops/ssu.py:61 SSUFn.forward)
 *   ssm_conv_prefill       <- modules/ssm.py:112-134 (SiLU, depthwise causal conv1d,
 *                             split into x, B, C) and inference/ssm_cache.py:10-36
 *                             SSMCache.build_conv_ctx
 *   sattn_decode_step      <- modules/selective_attention.py:390-404 (SelectiveMHA.step:
 *                             cache update and pos-mode gated softmax attention) and
 *                             inference/selective_attn_cache.py:27-42 SelectiveAttnCache.update_kv
 *   sattn_prefill_fwd      <- modules/selective_attention.py:27-144 _build_attn_matrix and
 *                             the seq-mode _gated_softmax, with the @ v of :270-280
 *                             (SelectiveMHA.forward in inference, compressed or not)
 *   sattn_train_fwd        <- modules/selective_attention.py:232-280 (SelectiveMHA.forward with
 *                             self.training: score statistics, std-scaled log-gates, gated
 *                             softmax, @ v)
 *   sattn_train_bwd        <- the autograd backward of the same lines (torch's, for the
 *                             reference), including the gradient through the score std
 *   ssm_conv_decode        <- modules/ssm.py:173-186 (decode step: cache update, SiLU,
 *                             weighted sum, split) and inference/ssm_cache.py:38-43
 *                             SSMCache.update
 * The reference crosses host->device only at Triton launches; these functions are
 * the same crossing for a C caller.
 */
#ifndef SSD_B200_H
#define SSD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SSD_OK = 0,
  SSD_ERR_INVALID_ARGUMENT = 1, /* bad size, null pointer, unsupported combination */
  SSD_ERR_UNSUPPORTED_DTYPE = 2,
  SSD_ERR_WORKSPACE_TOO_SMALL = 3,
  SSD_ERR_CUDA = 4,             /* a CUDA runtime call failed (launch, attribute, ...) */
  SSD_ERR_DEVICE_TIMEOUT = 5,   /* a kernel gave up on a bounded wait (see ssd_b200_device_error) */
  SSD_ERR_NO_TENSOR_MAP = 6,    /* the driver's tensor-map encoder could not be obtained */
  SSD_ERR_SCRATCH_LIMIT = 7     /* ssd_scan_fwd_noalloc: needs more than its fixed scratch */
} ssd_status_t;

typedef enum { SSD_F32 = 0, SSD_BF16 = 1, SSD_F16 = 2 } ssd_dtype_t;

typedef enum {
  SSD_IMPL_AUTO = 0,   /* tensor-core path when the shape/dtype allow it, else CUDA-core path;
                          on the tensor-core path chunk_state and state_passing are fused when
                          there are at least SSD_FUSED_MIN_CHAINS (row, head) chains; fp32
                          inputs with fp32 output take the split-bf16 tensor-core chain */
  SSD_IMPL_TC = 1,     /* tcgen05 + TMA kernels (bf16/fp16, headdim 64, dstate 128, chunk 256),
                          chunk_state and state_passing fused (one CTA per (row, head) chain) */
  SSD_IMPL_SIMT = 2,   /* CUDA-core FFMA kernels (any dtype; fp32-exact accumulation) */
  SSD_IMPL_TC_STAGED = 3 /* tensor-core kernels with chunk_state and state_passing as separate
                            launches and fp32 chunk states in the workspace */
} ssd_impl_t;

#define SSD_FUSED_MIN_CHAINS 128

/*
 * One parameter block for the SSD entry points. Fields an entry point does not
 * use are ignored. Shapes (b = batch, L = seqlen, H = nheads, P = headdim,
 * N = dstate, G = ngroups, cs = chunk_size, nc = ceil(L/cs)):
 *
 *   u          (b, L, H, P)   x_dtype          A          (H,)          fp32
 *   B, C       (b, L, G, N)   x_dtype          delta_raw  (b, L, H)     dt_dtype
 *   delta_bias (H,) fp32 or NULL               h_init     (b, H, P, N)  fp32 or NULL
 *   length     (b,) int64 or NULL (= L)        D          (H*P,) fp32 or NULL
 *   z          (b, L, H*P)    x_dtype or NULL  y          (b, L, H, P)  y_dtype
 *   h_last     (b, H, P, N)   fp32
 *
 * Packed variable-length mode (an extension; the reference only has padded rows
 * plus `length`): nseq > 0, b must be 1, L is the total token count and
 * cu_seqlens holds nseq+1 offsets (int32 or int64 per cu_dtype). Each sequence is
 * scanned as its own row with zero (or h_init[i]) initial state, exactly as the
 * reference computes a right-padded row with length = seqlen; h_last and h_init are
 * (nseq, H, P, N). `length` must be NULL in this mode.
 *
 * Stage buffers (chunk-major, k = b*nc + c in padded mode):
 *   dt, cum    (b, nc, H, cs) fp32   -- the reference's (b, H, nc, cs) with H and nc swapped
 *   states     (b, nc, H, P, N) fp32 -- same as the reference
 *   CB         (b, nc, G, cs, cs) fp32 -- same as the reference
 */
typedef struct ssd_params {
  int64_t batch, seqlen, nheads, headdim, dstate, ngroups, chunk_size;
  int64_t nseq;
  int32_t x_dtype, dt_dtype, y_dtype, cu_dtype; /* cu_dtype: 32 or 64 */
  int32_t use_delta_softplus;
  float delta_min, delta_max;
  int32_t impl;
  const void* u;
  const float* A;
  const void* B;
  const void* C;
  const void* delta_raw;
  const float* delta_bias;
  const float* h_init;
  const int64_t* length;
  const float* D;
  const void* z;
  const void* cu_seqlens;
  void* y;
  float* h_last;
  float* dt;
  float* cum;
  float* states;
  float* CB;
  void* workspace;
  size_t workspace_bytes;
  /* Optional cudaEvent_t handles recorded on the stream by ssd_scan_fwd: [0] before
     the first stage, then after chunk_cumsum [1] (on the split-bf16 chain also after the
     split of B for chunk_state), chunk_state [2], state_passing [3], bmm_chunk [4] (same
     point as [3] when bmm is fused) and chunk_scan [5]. NULL entries are skipped. */
  void* events[6];
} ssd_params;

/* Library version string and the status text of a code. */
const char* ssd_b200_version(void);
const char* ssd_b200_status_string(int status);

/*
 * Device-side error flag: kernels set it (instead of trapping) when a bounded
 * wait gives up. Synchronizes `stream`, returns the flag (0 = none) and clears it.
 */
int ssd_b200_device_error(void* stream);

/* Whether ssd_scan_fwd runs `p` on tensor cores (1: the 16-bit chains, or the split-bf16
 * chain of fp32 inputs) or on CUDA cores (0). */
int ssd_scan_uses_tensor_cores(const ssd_params* p);

/* The kernel chain ssd_scan_fwd runs for `p` (its impl field included): 0 CUDA-core
 * stages, 1 tensor-core stages with chunk_state and state_passing as separate launches,
 * 2 tensor-core with chunk_state and state_passing fused, 3 fp32 inputs and output on
 * tensor cores with split-bf16 products (hi = bf16(x), lo = bf16(x - hi); three products
 * per pair; chunk_state, bmm_chunk and chunk_scan; taken under SSD_IMPL_AUTO at headdim 64,
 * dstate 128, chunk 256 when u, B and C are 16-byte aligned); -1 for an invalid geometry.
 * No reference counterpart (host-side query). */
int ssd_scan_path(const ssd_params* p);

/* Bytes of workspace ssd_scan_fwd needs for `p` (sizes, dtypes, impl, nseq). */
size_t ssd_scan_fwd_workspace_size(const ssd_params* p);

/*
 * Fused SSD forward: chunk_cumsum -> chunk_state -> state_passing -> chunk_scan
 * (bmm_chunk fused into chunk_scan on the tensor-core path), with the optional
 * D-skip and z-gate epilogue y = (y + D*u) * silu(z) of modules/ssm.py:145-150.
 * Writes y and h_last. Uses p->workspace (>= ssd_scan_fwd_workspace_size(p)).
 */
int ssd_scan_fwd(const ssd_params* p, void* stream);

/*
 * ssd_scan_fwd without a caller workspace and without any allocation. It has no
 * counterpart in the reference (whose forward allocates its intermediates through
 * torch on every call). It is for callers that cannot allocate device memory when
 * they run the scan, e.g. a host whose device memory is fully reserved by another
 * runtime's pool, or a hot path that must not block on an allocation's device-wide
 * synchronisation. The library holds a fixed scratch array of
 * SSD_NOALLOC_SCRATCH_BYTES on every GPU that loads it, until the process exits;
 * p->workspace and p->workspace_bytes are ignored. A problem whose
 * ssd_scan_fwd_workspace_size() exceeds the array returns SSD_ERR_SCRATCH_LIMIT
 * (the fused tensor-core chain, the default from SSD_FUSED_MIN_CHAINS (row, head)
 * chains, needs about 18 KB per chunk and head: b=8, L=2048, H=24 takes about 28 MB
 * and fits; the staged chain (SSD_IMPL_TC_STAGED, or fewer chains under AUTO) needs
 * about 50 KB per chunk and head, so the same shape forced onto it, at 78 MB, is
 * rejected; b=2, L=2048, H=32 on the staged chain takes 26 MB and fits).
 * The first call on a device resolves the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture. A failed
 * lookup is not remembered: the next call on that device tries again. All calls
 * share the array: calls that overlap on the GPU (other streams or host threads)
 * race on it. Nothing in it needs to start at zero.
 */
#define SSD_NOALLOC_SCRATCH_BYTES (32u << 20)
int ssd_scan_fwd_noalloc(const ssd_params* p, void* stream);

/* Stage entry points (padded mode only). Each reads/writes the stage buffers. */
int ssd_chunk_cumsum_fwd(const ssd_params* p, void* stream);     /* -> dt, cum */
int ssd_chunk_state_fwd(const ssd_params* p, void* stream);      /* u, B, dt, cum -> states */
int ssd_state_passing_fwd(const ssd_params* p, void* stream);    /* states (in place), cum, h_init -> h_last */
int ssd_bmm_chunk_fwd(const ssd_params* p, void* stream);        /* B, C -> CB (lower-triangular tiles) */
int ssd_chunk_scan_fwd(const ssd_params* p, void* stream);       /* u, dt, cum, C, states, CB, D, z -> y */

/*
 * Gradients of the SSD scan (triton_kernels/ssd_scan/backward.py:467-555): the
 * forward intermediates are recomputed, then the reference's stages run with the
 * same maths and masking (rows at or past `length` get no gradient and their y_grad
 * is ignored; clamped dt gets zero gradient; softplus gets sigmoid below 20).
 * Inputs come from an ssd_params block that describes the forward call (u, A, B,
 * C, delta_raw, delta_bias, h_init, length or cu_seqlens, chunk size, dt options;
 * D, z and y are ignored) plus:
 *   y_grad       (b, L, H, P)  y_grad_dtype (fp32 or x_dtype)
 *   h_last_grad  (b, H, P, N)  fp32, or NULL for zero
 * and writes
 *   u_grad (b, L, H, P) x_dtype;  A_grad (H,) fp32;  B_grad, C_grad (b, L, G, N) fp32;
 *   delta_raw_grad (b, L, H) dt_dtype;  delta_bias_grad (H,) fp32 (required iff
 *   delta_bias is given);  h_init_grad (b, H, P, N) fp32 (required iff h_init is given)
 * (the reference's output dtypes: backward.py:90,144,200,254,439-441). Supported shapes:
 * headdim <= 64, dstate <= 128, both multiples of 8; chunk_size a multiple of 32 up
 * to 256. Uses p->workspace (>= ssd_scan_bwd_workspace_size(p)); p->events, when
 * set, are recorded before the first stage [0], after the state recompute [1], the
 * state passes and CB [2], the state-side products [3], the intra-chunk products [4].
 */
typedef struct ssd_bwd_params {
  const void* y_grad;
  int32_t y_grad_dtype;
  const float* h_last_grad;
  void* u_grad;
  float* A_grad;
  float* B_grad;
  float* C_grad;
  void* delta_raw_grad;
  float* delta_bias_grad;
  float* h_init_grad;
} ssd_bwd_params;

/* Bytes of device workspace ssd_scan_bwd needs for p's geometry and x_dtype (fp32 inputs at
 * headdim 64, dstate 128, chunk 256 add the buffers of the tensor-core fp32 path). */
size_t ssd_scan_bwd_workspace_size(const ssd_params* p);
int ssd_scan_bwd(const ssd_params* p, const ssd_bwd_params* g, void* stream);

/*
 * Selective state update, one token (triton_kernels/ssu/forward.py:7):
 *   dt = clamp(softplus?(delta_raw + delta_bias)), h <- h*exp(A*dt) + (B*dt) x u,
 *   y = h . C, then optionally y = (y + D*u) * silu(z).
 * u (b,H,P) x_dtype; A (H,) fp32; B, C (b,G,N) x_dtype; delta_raw (b,H) dt_dtype;
 * delta_bias (H,) fp32 or NULL; h (b,H,P,N) h_dtype, updated in place;
 * D (H*P,) fp32 or NULL; z (b,H*P) x_dtype or NULL; y (b,H,P) y_dtype.
 */
int ssu_fwd(const void* u, const float* A, const void* B, const void* C,
            const void* delta_raw, const float* delta_bias, void* h, void* y,
            const float* D, const void* z,
            int64_t batch, int64_t nheads, int64_t headdim, int64_t dstate, int64_t ngroups,
            int32_t x_dtype, int32_t dt_dtype, int32_t h_dtype, int32_t y_dtype,
            int32_t use_delta_softplus, float delta_min, float delta_max, void* stream);

/*
 * SSM prefill front end between the input projection and the scan
 * (modules/ssm.py:112-134, inference/ssm_cache.py:10-36):
 *   out = bias + depthwise causal conv_K( silu(hbc) )   (silu rounded to `dtype` first),
 *   x, B, C = out[..., :inner], out[..., inner:inner+gn], out[..., inner+gn:],
 *   conv_ctx[b, c, k] = hbc[b, len_b - K + k, c] (0 outside [0, len_b)), len_b = lengths[b] or L.
 * hbc (b, L, inner + 2*gn) with token stride row_stride (elements; the channels are
 * contiguous), dtype; weight (inner+2*gn, K) fp32; bias (inner+2*gn,) fp32 or NULL;
 * x (b, L, inner), B and C (b, L, gn) dtype; conv_ctx (b, inner+2*gn, K) dtype or NULL;
 * lengths (b,) int64 or NULL. 1 <= K <= 8.
 */
int ssm_conv_prefill(const void* hbc, int64_t row_stride, const float* weight, const float* bias,
                     void* x, void* B, void* C, void* conv_ctx, const int64_t* lengths,
                     int64_t batch, int64_t seqlen, int64_t inner, int64_t gn, int64_t kernel_size,
                     int32_t dtype, void* stream);

/*
 * SSM decode-step front end (modules/ssm.py:173-186, inference/ssm_cache.py:38-43): per
 * channel c of row b, conv_ctx[b, c, :] is shifted left by one and hbc_new[b, c] appended
 * (in place), then out = sum_k w[c,k] silu(conv_ctx[b,c,k]) + bias[c] with the reference's
 * roundings to `dtype` (silu, each product, the sum, the bias add), split into
 * x (b, inner), B and C (b, gn). hbc_new (b, inner + 2*gn) with row stride row_stride
 * (elements), dtype; conv_ctx (b, inner + 2*gn, K) dtype, updated in place; weight
 * (inner+2*gn, K) fp32; bias (inner+2*gn,) fp32 or NULL. 1 <= K <= 8.
 */
int ssm_conv_decode(const void* hbc_new, int64_t row_stride, void* conv_ctx, const float* weight, const float* bias,
                    void* x, void* B, void* C, int64_t batch, int64_t inner, int64_t gn, int64_t kernel_size,
                    int32_t dtype, void* stream);

/*
 * Selective-attention decode step (modules/selective_attention.py:390-404): writes the
 * token's key, value and log-gate at slot write_idx of the cache (as
 * SelectiveAttnCache.update_kv does), then with n = write_idx + 1 cached keys
 *   s_j = scale * q . k_j + (j < n-1 ? log_gate_j : 0),   out = softmax(s) . v
 * (the pos-mode gated softmax: every cached key but the token's own is gated; a key
 * whose log-gate is -inf drops out). The caller advances write_idx.
 *   q_rot, k_rot, v      (b, H, D)          dtype
 *   log_gate             (b, H)             fp32
 *   k_cache, v_cache     (b, H, cap, D)     dtype, updated in place
 *   log_gate_cache       (b, H, cap)        fp32, updated in place
 *   out                  (b, H, D)          dtype
 * head_dim D in {8, 16, 32, 64, 128, 256}; q_rot, k_cache, v_cache 16-byte aligned;
 * 0 <= write_idx < cap.
 */
int sattn_decode_step(const void* q_rot, const void* k_rot, const void* v, const float* log_gate,
                      void* k_cache, void* v_cache, float* log_gate_cache, int64_t write_idx, int64_t capacity,
                      void* out, int64_t batch, int64_t nheads, int64_t head_dim, float scale, int32_t dtype,
                      void* stream);

/*
 * Selective-attention prefill (inference): for every query i of a sequence
 *   s_ij = scale * q_i . k_j + (j < i ? log_gate_j : 0)  for j <= i,   out_i = softmax_j(s_i) . v
 * i.e. causal attention in which every earlier key adds its log-gate and the token's
 * own score is ungated (the seq-mode _gated_softmax). Keys whose gate is zero (log-gate
 * -inf; the reference compresses them away) and padding keys (log-gate -inf, as the
 * layer's masked_fill sets them) drop out.
 *   q_rot, k_rot, v, out  (b, H, L, D)  dtype, 16-byte aligned
 *   log_gate              (b, H, L)     fp32
 * head_dim D in {16, 32, 64, 128}. impl: SSD_IMPL_AUTO takes the tcgen05 kernel for
 * 16-bit inputs with D 64 or 128 (out 16-byte aligned) and the CUDA-core kernel
 * otherwise; SSD_IMPL_TC requires the former, SSD_IMPL_SIMT forces the latter.
 */
int sattn_prefill_fwd(const void* q_rot, const void* k_rot, const void* v, const float* log_gate, void* out,
                      int64_t batch, int64_t nheads, int64_t seqlen, int64_t head_dim, float scale, int32_t dtype,
                      int32_t impl, void* stream);

/*
 * Selective attention in training mode (modules/selective_attention.py:232-280 with
 * self.training) and its backward. Forward, per head h over the batch:
 *   S_ij      = scale * q_i . k_j  (j <= i when is_causal)
 *   mean, std = over the valid scores: i, j < lengths[b] (and j <= i when causal)
 *   log_gate  = log(select_gate) * (std * log_gate_penalty), -inf for j >= lengths[b]
 *   out_i     = softmax_j(S_ij + (j != i ? log_gate_j : 0)) . v
 *   q_rot, k_rot, v, out  (b, H, L, D)  dtype, 16-byte aligned
 *   select_gate           (b, H, L)     dtype (the sigmoid gate, transposed as :204)
 *   lengths               (b,)          int64, or NULL (every position valid)
 * and, saved for the backward (and for the layer's score_std_ema update, :252-256):
 *   lse       (b, H, L) fp32  row log-sum-exp of the gated scores
 *   log_gate  (b, H, L) fp32
 *   stats     (H, 4)    fp32  mean, std, count of valid scores, and a coefficient the
 *                             backward fills in
 * The backward takes dout (b, H, L, D) and writes dq, dk, dv (b, H, L, D) and
 * dselect_gate (b, H, L), all in dtype, including the path through std (the gates are
 * scaled by it). head_dim D in {16, 32, 64, 128}. impl: SSD_IMPL_AUTO runs 16-bit inputs
 * with head_dim 64 on tcgen05 (16-bit products, fp32 accumulation and softmax) and the rest
 * on CUDA cores in fp32; SSD_IMPL_TC requires the former, SSD_IMPL_SIMT forces the latter. Both
 * calls use p->workspace (>= sattn_train_workspace_size(p)); the backward needs the
 * forward's out, lse, log_gate and stats unchanged.
 */
typedef struct sattn_train_params {
  int64_t batch, nheads, seqlen, head_dim;
  int32_t dtype;
  int32_t is_causal;
  int32_t impl; /* SSD_IMPL_AUTO / SSD_IMPL_TC (16-bit, head_dim 64: tcgen05) / SSD_IMPL_SIMT */
  float scale;
  float log_gate_penalty;
  const void* q_rot;
  const void* k_rot;
  const void* v;
  const void* select_gate;
  const int64_t* lengths;
  void* out;
  float* lse;
  float* log_gate;
  float* stats;
  void* workspace;
  size_t workspace_bytes;
} sattn_train_params;

size_t sattn_train_workspace_size(const sattn_train_params* p);
int sattn_train_fwd(const sattn_train_params* p, void* stream);
int sattn_train_bwd(const sattn_train_params* p, const void* dout, void* dq, void* dk, void* dv,
                    void* dselect_gate, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SSD_B200_H */
