// api.cu - the C ABI declared in include/ssd_b200.h: argument checks, workspace
// layout, stage dispatch between the tensor-core and CUDA-core kernels.
#include <cstring>

#include "kernels.h"

using namespace ssdb200;

namespace {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t v) { return (v + kAlign - 1) & ~(kAlign - 1); }

bool dtype_ok(int d) { return d == SSD_F32 || d == SSD_BF16 || d == SSD_F16; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct Geometry {
  int b, H, P, N, G, cs;
  long long L, T;
  int nc;        // padded: chunks per row
  int nchunks;   // grid extent over chunks
  int nrows;     // rows (padded batch) or sequences (packed)
  bool packed;
};

int geometry(const ssd_params* p, Geometry& g) {
  if (!p) return SSD_ERR_INVALID_ARGUMENT;
  if (p->batch <= 0 || p->seqlen <= 0 || p->nheads <= 0 || p->headdim <= 0 || p->dstate <= 0 ||
      p->ngroups <= 0 || p->chunk_size <= 0)
    return SSD_ERR_INVALID_ARGUMENT;
  if (p->nheads % p->ngroups != 0) return SSD_ERR_INVALID_ARGUMENT;
  if (p->chunk_size > 256) return SSD_ERR_INVALID_ARGUMENT;  // chunk_cumsum: <= 8 tokens per lane
  if ((p->headdim * p->dstate) % 4 != 0) return SSD_ERR_INVALID_ARGUMENT;
  g.b = (int)p->batch;
  g.H = (int)p->nheads;
  g.P = (int)p->headdim;
  g.N = (int)p->dstate;
  g.G = (int)p->ngroups;
  g.cs = (int)p->chunk_size;
  g.L = p->seqlen;
  g.T = p->batch * p->seqlen;
  g.packed = p->nseq > 0;
  if (g.T > (1ll << 31) - 1) return SSD_ERR_INVALID_ARGUMENT;  // TMA coordinates are 32-bit
  if (g.packed) {
    if (p->batch != 1 || p->length || !p->cu_seqlens) return SSD_ERR_INVALID_ARGUMENT;
    if (p->cu_dtype != 32 && p->cu_dtype != 64) return SSD_ERR_INVALID_ARGUMENT;
    g.nc = 0;
    g.nrows = (int)p->nseq;
    g.nchunks = (int)((g.T + g.cs - 1) / g.cs + p->nseq);
  } else {
    g.nc = (int)((g.L + g.cs - 1) / g.cs);
    g.nrows = g.b;
    g.nchunks = g.b * g.nc;
  }
  return SSD_OK;
}

// The CUDA-core chunk_state stages 32 tokens of x*w and B in shared memory.
bool simt_fits(const Geometry& g) { return 32ll * (g.P + g.N) * 4 <= 200 * 1024; }

bool use_tc(const ssd_params* p, const Geometry& g) {
  if (p->impl == SSD_IMPL_SIMT) return false;
  return tc_supported(p->x_dtype, g.P, g.N, g.cs);
}

// fp32 inputs and output at P 64, N 128, cs 256 under AUTO: chunk_state, bmm_chunk and
// chunk_scan on tcgen05 with split-bf16 products (ssd_split.cu); SSD_IMPL_SIMT keeps the
// CUDA-core kernels. u, B, C, D, z and y are accessed with 16-byte loads and stores.
bool use_split(const ssd_params* p, const Geometry& g) {
  // grids of (.., chunk) with the chunk index in a y / z grid dimension (at most 65535)
  return p->impl == SSD_IMPL_AUTO && split_supported(p->x_dtype, p->y_dtype, g.P, g.N, g.cs) && g.nchunks <= 65535 &&
         aligned16(p->u) && aligned16(p->B) && aligned16(p->C) && aligned16(p->y) &&
         (!p->D || aligned16(p->D)) && (!p->z || aligned16(p->z));
}

// Tensor-core path with chunk_state and state_passing fused (one CTA per (row, head)
// chain): always under SSD_IMPL_TC, under AUTO when there are enough chains to fill
// the GPU.
bool use_fused(const ssd_params* p, const Geometry& g) {
  if (!use_tc(p, g) || p->impl == SSD_IMPL_TC_STAGED) return false;
  return p->impl == SSD_IMPL_TC || (long long)g.nrows * g.H >= SSD_FUSED_MIN_CHAINS;
}

struct Workspace {
  float* dt;
  float* cum;
  float* states;
  void* prev16;
  float* CB;
  void* Bs;   // split-bf16 chain: operand tiles of chunk_state (B rows) and chunk_scan
  void* CBs;  // (masked CB, C rows)
  void* Cs;
  ChunkEntry* table;
  int2* rows;
  int* count;
  size_t bytes;
};

Workspace carve(const ssd_params* p, const Geometry& g, bool tc, bool fused, uint8_t* base) {
  Workspace w{};
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* ptr = base ? base + off : nullptr;
    off += align_up(n);
    return ptr;
  };
  const size_t nk = (size_t)g.nchunks;
  w.dt = (float*)take(nk * g.H * g.cs * sizeof(float));
  w.cum = (float*)take(nk * g.H * g.cs * sizeof(float));
  if (!fused) w.states = (float*)take(nk * g.H * (size_t)g.P * g.N * sizeof(float));
  if (tc) w.prev16 = take(nk * g.H * (size_t)g.P * g.N * 2);
  else if (use_split(p, g)) {
    const size_t tile = split_operand_bytes_per_chunk_group() / 14;  // 4 B + 6 CB + 4 C tiles
    w.Bs = take(nk * g.G * 4 * tile);
    w.CBs = take(nk * g.G * 6 * tile);
    w.Cs = take(nk * g.G * 4 * tile);
  } else w.CB = (float*)take(nk * g.G * (size_t)g.cs * g.cs * sizeof(float));
  if (g.packed) {
    w.table = (ChunkEntry*)take(nk * sizeof(ChunkEntry));
    w.rows = (int2*)take((size_t)g.nrows * sizeof(int2));
    w.count = (int*)take(sizeof(int));
  }
  w.bytes = off;
  return w;
}

LaunchCtx make_ctx(const ssd_params* p, const Geometry& g, cudaStream_t s, const Workspace* w) {
  LaunchCtx c{};
  c.stream = s;
  c.cm.packed = g.packed ? 1 : 0;
  c.cm.cs = g.cs;
  c.cm.nc = g.nc;
  c.cm.L = g.L;
  c.cm.length = reinterpret_cast<const long long*>(p->length);
  if (g.packed && w) {
    c.cm.table = w->table;
    c.cm.count = w->count;
    c.cm.rows = w->rows;
  }
  c.nchunks_max = g.nchunks;
  c.nrows = g.nrows;
  c.H = g.H;
  c.P = g.P;
  c.N = g.N;
  c.G = g.G;
  c.cs = g.cs;
  c.T = g.T;
  c.use_sp = p->use_delta_softplus ? 1 : 0;
  c.dmin = p->delta_min;
  c.dmax = p->delta_max;
  return c;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? SSD_OK : SSD_ERR_CUDA; }

int check_common_inputs(const ssd_params* p, bool need_y) {
  if (!dtype_ok(p->x_dtype) || !dtype_ok(p->dt_dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  if (need_y && !dtype_ok(p->y_dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  return SSD_OK;
}

void record(const ssd_params* p, int i, cudaStream_t s) {
  if (p->events[i]) cudaEventRecord(reinterpret_cast<cudaEvent_t>(p->events[i]), s);
}

}  // namespace

extern "C" {

const char* ssd_b200_version(void) { return "ssd_b200 0.1.0 sm_100a"; }

const char* ssd_b200_status_string(int status) {
  switch (status) {
    case SSD_OK: return "ok";
    case SSD_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SSD_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case SSD_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case SSD_ERR_CUDA: return "CUDA runtime error";
    case SSD_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case SSD_ERR_NO_TENSOR_MAP: return "tensor-map encoder unavailable";
    case SSD_ERR_SCRATCH_LIMIT: return "problem needs more scratch than ssd_scan_fwd_noalloc holds";
  }
  return "unknown status";
}

int ssd_b200_device_error(void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned int a = fetch_error_simt(s);
  const unsigned int b = fetch_error_tc(s);
  const unsigned int c = fetch_error_ssu(s);
  const unsigned int d = fetch_error_sattn(s);
  const unsigned int e = fetch_error_bwd_tc(s);
  const unsigned int f = fetch_error_split(s);
  return (int)(a ? a : (b ? b : (c ? c : (d ? d : (e ? e : f)))));
}

int ssd_scan_uses_tensor_cores(const ssd_params* p) {
  Geometry g;
  if (geometry(p, g) != SSD_OK) return 0;
  return (use_tc(p, g) || use_split(p, g)) ? 1 : 0;
}

int ssd_scan_path(const ssd_params* p) {
  Geometry g;
  if (geometry(p, g) != SSD_OK) return -1;
  if (use_fused(p, g)) return 2;
  if (use_split(p, g)) return 3;
  return use_tc(p, g) ? 1 : 0;
}

size_t ssd_scan_fwd_workspace_size(const ssd_params* p) {
  Geometry g;
  if (geometry(p, g) != SSD_OK) return 0;
  return carve(p, g, use_tc(p, g), use_fused(p, g), nullptr).bytes;
}

int ssd_scan_fwd(const ssd_params* p, void* stream) {
  Geometry g;
  int st = geometry(p, g);
  if (st) return st;
  if ((st = check_common_inputs(p, true))) return st;
  if (!p->u || !p->A || !p->B || !p->C || !p->delta_raw || !p->y || !p->h_last || !p->workspace)
    return SSD_ERR_INVALID_ARGUMENT;
  const bool want_tc = p->impl == SSD_IMPL_TC || p->impl == SSD_IMPL_TC_STAGED;
  if (want_tc && !tc_supported(p->x_dtype, g.P, g.N, g.cs)) return SSD_ERR_INVALID_ARGUMENT;
  const bool tc = use_tc(p, g);
  if (!tc && !simt_fits(g)) return SSD_ERR_INVALID_ARGUMENT;
  if (tc && p->y_dtype != SSD_F32 && p->y_dtype != p->x_dtype) return SSD_ERR_UNSUPPORTED_DTYPE;
  if (!aligned16(p->h_last) || (p->h_init && !aligned16(p->h_init))) return SSD_ERR_INVALID_ARGUMENT;
  if (tc && (!aligned16(p->u) || !aligned16(p->B) || !aligned16(p->C) || !aligned16(p->y) ||
             (p->z && !aligned16(p->z)) || (p->D && !aligned16(p->D))))
    return SSD_ERR_INVALID_ARGUMENT;
  const bool fused = use_fused(p, g);
  Workspace w = carve(p, g, tc, fused, reinterpret_cast<uint8_t*>(p->workspace));
  if (p->workspace_bytes < w.bytes) return SSD_ERR_WORKSPACE_TOO_SMALL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LaunchCtx c = make_ctx(p, g, s, &w);
  record(p, 0, s);
  if (g.packed) {
    st = cuda_status(launch_build_chunk_table(s, p->cu_seqlens, p->cu_dtype == 64, (int)p->nseq, g.cs, w.table,
                                              w.rows, w.count));
    if (st) return st;
  }
  int tms = 0;
  if (fused) {
    // chunk_cumsum, chunk_state and state_passing in one kernel (events [1]..[3] coincide).
    record(p, 1, s);
    record(p, 2, s);
    cudaError_t e = launch_tc_state_pass(c, p->x_dtype, p->dt_dtype, p->u, p->B, p->A, p->delta_raw,
                                         p->delta_bias, w.dt, w.cum, w.prev16, p->h_init, p->h_last, &tms);
    if (tms) return SSD_ERR_NO_TENSOR_MAP;
    if ((st = cuda_status(e))) return st;
    record(p, 3, s);
    record(p, 4, s);
    e = launch_tc_chunk_scan(c, p->x_dtype, p->y_dtype, p->u, p->A, w.dt, w.cum, p->B, p->C, w.prev16, p->D, p->z,
                             p->y, &tms);
    if (tms) return SSD_ERR_NO_TENSOR_MAP;
    if ((st = cuda_status(e))) return st;
    record(p, 5, s);
  } else if (tc) {
    // chunk_cumsum is fused into the tensor-core chunk_state (events [1] and [2] coincide).
    record(p, 1, s);
    cudaError_t e = launch_tc_chunk_state(c, p->x_dtype, p->dt_dtype, p->u, p->B, p->A, p->delta_raw,
                                          p->delta_bias, w.dt, w.cum, w.states, &tms);
    if (tms) return SSD_ERR_NO_TENSOR_MAP;
    if ((st = cuda_status(e))) return st;
    record(p, 2, s);
    if ((st = cuda_status(launch_state_passing(c, w.states, w.prev16, p->x_dtype, w.cum, p->h_init, p->h_last))))
      return st;
    record(p, 3, s);
    record(p, 4, s);
    e = launch_tc_chunk_scan(c, p->x_dtype, p->y_dtype, p->u, p->A, w.dt, w.cum, p->B, p->C, w.prev16, p->D, p->z,
                             p->y, &tms);
    if (tms) return SSD_ERR_NO_TENSOR_MAP;
    if ((st = cuda_status(e))) return st;
    record(p, 5, s);
  } else {
    const bool split = use_split(p, g);
    const float *u32 = static_cast<const float*>(p->u), *B32 = static_cast<const float*>(p->B),
                *C32 = static_cast<const float*>(p->C);
    if ((st = cuda_status(launch_chunk_cumsum(c, p->dt_dtype, p->A, p->delta_raw, p->delta_bias, w.dt, w.cum))))
      return st;
    // split chain: chunk_state's B tiles are written here too (inside events [0, 1])
    if (split && (st = cuda_status(launch_split_b(c, B32, w.Bs)))) return st;
    record(p, 1, s);
    if ((st = cuda_status(split ? launch_split_chunk_state(c, u32, w.Bs, w.dt, w.cum, w.states)
                                : launch_simt_chunk_state(c, p->x_dtype, p->u, p->B, w.dt, w.cum, w.states))))
      return st;
    record(p, 2, s);
    if ((st = cuda_status(launch_state_passing(c, w.states, nullptr, SSD_F32, w.cum, p->h_init, p->h_last))))
      return st;
    record(p, 3, s);
    if ((st = cuda_status(split ? launch_split_bmm(c, B32, C32, w.CBs, w.Cs)
                                : launch_simt_bmm_chunk(c, p->x_dtype, p->B, p->C, w.CB))))
      return st;
    record(p, 4, s);
    if ((st = cuda_status(split ? launch_split_chunk_scan(c, u32, w.dt, w.cum, w.Cs, w.states, w.CBs, p->D,
                                                          static_cast<const float*>(p->z), static_cast<float*>(p->y))
                                : launch_simt_chunk_scan(c, p->x_dtype, p->y_dtype, p->u, w.dt, w.cum, p->C,
                                                         w.states, w.CB, p->D, p->z, p->y))))
      return st;
    record(p, 5, s);
  }
  return SSD_OK;
}

// ------------------------------------------------------------- backward
namespace {

// x32: fp32 u / B / C, whose backward (at the split path's shape) also needs the split operand
// tiles, accY and G = y_grad u^T
size_t carve_bwd(const Geometry& g, bool x32, uint8_t* base, BwdArgs* a, ChunkEntry** table, int2** rows,
                 int** count) {
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* ptr = base ? base + off : nullptr;
    off += align_up(n);
    return reinterpret_cast<float*>(ptr);
  };
  const size_t nk = (size_t)g.nchunks, H = (size_t)g.H, PN = (size_t)g.P * g.N, cs = (size_t)g.cs;
  BwdArgs dummy{};
  BwdArgs& w = a ? *a : dummy;
  w.dt = take(nk * H * cs * 4);
  w.cum = take(nk * H * cs * 4);
  w.states = take(nk * H * PN * 4);
  w.hg = take(nk * H * PN * 4);
  w.CB = take(nk * g.G * cs * cs * 4);
  w.CBg = take(nk * g.G * cs * cs * 4);
  w.accS = take(nk * H * cs * g.P * 4);
  w.gC = take(nk * H * cs * 4);
  w.dl_part = take(nk * H * bwd_dl_slices(g.P, g.N) * 4);
  w.A_part = take(nk * H * 4);
  w.bias_part = take(nk * H * 4);
  w.rows4 = take(4 * nk * H * cs * 4);
  w.prev16 = reinterpret_cast<uint16_t*>(take(nk * H * PN * 2));
  w.hg16 = reinterpret_cast<uint16_t*>(take(nk * H * PN * 2));
  w.y16 = reinterpret_cast<uint16_t*>(take((size_t)g.T * H * g.P * 2));
  if (x32 && split_supported(SSD_F32, SSD_F32, g.P, g.N, g.cs)) {
    const size_t tiles = nk * g.G * (split_operand_bytes_per_chunk_group() / 14) * 4;
    w.Bs_split = take(tiles);
    w.Cs_split = take(tiles);
    w.accY = take(nk * H * cs * g.P * 4);
    w.Gyu = take(nk * H * cs * cs * 4);
  }
  ChunkEntry* t = nullptr;
  int2* r = nullptr;
  int* c = nullptr;
  if (g.packed) {
    t = reinterpret_cast<ChunkEntry*>(take(nk * sizeof(ChunkEntry)));
    r = reinterpret_cast<int2*>(take((size_t)g.nrows * sizeof(int2)));
    c = reinterpret_cast<int*>(take(sizeof(int)));
  }
  if (table) *table = t;
  if (rows) *rows = r;
  if (count) *count = c;
  return off;
}

}  // namespace

extern "C" size_t ssd_scan_bwd_workspace_size(const ssd_params* p) {
  Geometry g;
  if (geometry(p, g) != SSD_OK || !bwd_supported(g.P, g.N, g.cs)) return 0;
  return carve_bwd(g, p->x_dtype == SSD_F32, nullptr, nullptr, nullptr, nullptr, nullptr);
}

extern "C" int ssd_scan_bwd(const ssd_params* p, const ssd_bwd_params* gr, void* stream) {
  Geometry g;
  int st = geometry(p, g);
  if (st) return st;
  if (!gr) return SSD_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(p->x_dtype) || !dtype_ok(p->dt_dtype) || !dtype_ok(gr->y_grad_dtype))
    return SSD_ERR_UNSUPPORTED_DTYPE;
  if (!bwd_supported(g.P, g.N, g.cs)) return SSD_ERR_INVALID_ARGUMENT;
  if (!p->u || !p->A || !p->B || !p->C || !p->delta_raw || !p->workspace || !gr->y_grad || !gr->u_grad ||
      !gr->A_grad || !gr->B_grad || !gr->C_grad || !gr->delta_raw_grad)
    return SSD_ERR_INVALID_ARGUMENT;
  if (!p->delta_bias != !gr->delta_bias_grad || !p->h_init != !gr->h_init_grad) return SSD_ERR_INVALID_ARGUMENT;
  if (!aligned16(gr->B_grad) || !aligned16(gr->C_grad) || (p->h_init && !aligned16(p->h_init)) ||
      (gr->h_init_grad && !aligned16(gr->h_init_grad)) || (gr->h_last_grad && !aligned16(gr->h_last_grad)))
    return SSD_ERR_INVALID_ARGUMENT;
  if ((long long)g.nchunks > 65535 || g.H > 65535 || g.nrows > 65535) return SSD_ERR_INVALID_ARGUMENT;
  BwdArgs a{};
  ChunkEntry* table;
  int2* rows;
  int* count;
  const size_t need = carve_bwd(g, p->x_dtype == SSD_F32, reinterpret_cast<uint8_t*>(p->workspace), &a, &table, &rows, &count);
  if (p->workspace_bytes < need) return SSD_ERR_WORKSPACE_TOO_SMALL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  Workspace w{};
  w.table = table;
  w.rows = rows;
  w.count = count;
  LaunchCtx c = make_ctx(p, g, s, &w);
  record(p, 0, s);
  if (g.packed) {
    st = cuda_status(launch_build_chunk_table(s, p->cu_seqlens, p->cu_dtype == 64, (int)p->nseq, g.cs, table, rows,
                                              count));
    if (st) return st;
  }
  a.x_dtype = p->x_dtype;
  a.dt_dtype = p->dt_dtype;
  a.y_dtype = gr->y_grad_dtype;
  a.u = p->u;
  a.A = p->A;
  a.B = p->B;
  a.C = p->C;
  a.delta_raw = p->delta_raw;
  a.delta_bias = p->delta_bias;
  a.h_init = p->h_init;
  a.y_grad = gr->y_grad;
  a.h_last_grad = gr->h_last_grad;
  a.u_grad = gr->u_grad;
  a.A_grad = gr->A_grad;
  a.B_grad = gr->B_grad;
  a.C_grad = gr->C_grad;
  a.delta_raw_grad = gr->delta_raw_grad;
  a.delta_bias_grad = gr->delta_bias_grad;
  a.h_init_grad = gr->h_init_grad;
  for (int i = 0; i < 6; ++i) a.ev[i] = reinterpret_cast<cudaEvent_t>(p->events[i]);
  if ((st = cuda_status(launch_ssd_bwd(c, a)))) return st;
  record(p, 5, s);
  return SSD_OK;
}

// ------------------------------------------------------------- stage entries
static int stage_prologue(const ssd_params* p, Geometry& g) {
  int st = geometry(p, g);
  if (st) return st;
  if (g.packed) return SSD_ERR_INVALID_ARGUMENT;
  return SSD_OK;
}

int ssd_chunk_cumsum_fwd(const ssd_params* p, void* stream) {
  Geometry g;
  int st = stage_prologue(p, g);
  if (st) return st;
  if (!dtype_ok(p->dt_dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  if (!p->A || !p->delta_raw || !p->dt || !p->cum) return SSD_ERR_INVALID_ARGUMENT;
  LaunchCtx c = make_ctx(p, g, reinterpret_cast<cudaStream_t>(stream), nullptr);
  return cuda_status(launch_chunk_cumsum(c, p->dt_dtype, p->A, p->delta_raw, p->delta_bias, p->dt, p->cum));
}

int ssd_chunk_state_fwd(const ssd_params* p, void* stream) {
  Geometry g;
  int st = stage_prologue(p, g);
  if (st) return st;
  if ((st = check_common_inputs(p, false))) return st;
  if (!p->u || !p->B || !p->dt || !p->cum || !p->states) return SSD_ERR_INVALID_ARGUMENT;
  LaunchCtx c = make_ctx(p, g, reinterpret_cast<cudaStream_t>(stream), nullptr);
  if (use_tc(p, g)) {
    if (!aligned16(p->u) || !aligned16(p->B)) return SSD_ERR_INVALID_ARGUMENT;
    int tms = 0;
    cudaError_t e = launch_tc_chunk_state(c, p->x_dtype, SSD_F32, p->u, p->B, nullptr, nullptr, nullptr, p->dt,
                                          p->cum, p->states, &tms);
    if (tms) return SSD_ERR_NO_TENSOR_MAP;
    return cuda_status(e);
  }
  if (p->impl == SSD_IMPL_TC || p->impl == SSD_IMPL_TC_STAGED || !simt_fits(g)) return SSD_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_simt_chunk_state(c, p->x_dtype, p->u, p->B, p->dt, p->cum, p->states));
}

int ssd_state_passing_fwd(const ssd_params* p, void* stream) {
  Geometry g;
  int st = stage_prologue(p, g);
  if (st) return st;
  if (!p->states || !p->cum || !p->h_last) return SSD_ERR_INVALID_ARGUMENT;
  if (!aligned16(p->states) || !aligned16(p->h_last) || (p->h_init && !aligned16(p->h_init)))
    return SSD_ERR_INVALID_ARGUMENT;
  LaunchCtx c = make_ctx(p, g, reinterpret_cast<cudaStream_t>(stream), nullptr);
  return cuda_status(launch_state_passing(c, p->states, nullptr, SSD_F32, p->cum, p->h_init, p->h_last));
}

int ssd_bmm_chunk_fwd(const ssd_params* p, void* stream) {
  Geometry g;
  int st = stage_prologue(p, g);
  if (st) return st;
  if (!dtype_ok(p->x_dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  if (!p->B || !p->C || !p->CB) return SSD_ERR_INVALID_ARGUMENT;
  LaunchCtx c = make_ctx(p, g, reinterpret_cast<cudaStream_t>(stream), nullptr);
  return cuda_status(launch_simt_bmm_chunk(c, p->x_dtype, p->B, p->C, p->CB));
}

int ssd_chunk_scan_fwd(const ssd_params* p, void* stream) {
  Geometry g;
  int st = stage_prologue(p, g);
  if (st) return st;
  if ((st = check_common_inputs(p, true))) return st;
  if (!p->u || !p->C || !p->dt || !p->cum || !p->states || !p->CB || !p->y) return SSD_ERR_INVALID_ARGUMENT;
  LaunchCtx c = make_ctx(p, g, reinterpret_cast<cudaStream_t>(stream), nullptr);
  return cuda_status(launch_simt_chunk_scan(c, p->x_dtype, p->y_dtype, p->u, p->dt, p->cum, p->C, p->states, p->CB,
                                            p->D, p->z, p->y));
}

// ------------------------------------------------------------- SSU
int ssu_fwd(const void* u, const float* A, const void* B, const void* C, const void* delta_raw,
            const float* delta_bias, void* h, void* y, const float* D, const void* z, int64_t batch,
            int64_t nheads, int64_t headdim, int64_t dstate, int64_t ngroups, int32_t x_dtype, int32_t dt_dtype,
            int32_t h_dtype, int32_t y_dtype, int32_t use_delta_softplus, float delta_min, float delta_max,
            void* stream) {
  if (!u || !A || !B || !C || !delta_raw || !h || !y) return SSD_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || nheads <= 0 || headdim <= 0 || dstate <= 0 || ngroups <= 0) return SSD_ERR_INVALID_ARGUMENT;
  if (nheads % ngroups != 0 || dstate > 1024) return SSD_ERR_INVALID_ARGUMENT;
  if (batch * nheads > 0x7fffffffll) return SSD_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(x_dtype) || !dtype_ok(dt_dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  if (h_dtype != SSD_F32 && h_dtype != SSD_BF16) return SSD_ERR_UNSUPPORTED_DTYPE;
  if (y_dtype != x_dtype) return SSD_ERR_UNSUPPORTED_DTYPE;
  return cuda_status(launch_ssu(u, A, B, C, delta_raw, delta_bias, h, y, D, z, (int)batch, (int)nheads,
                                (int)headdim, (int)dstate, (int)ngroups, x_dtype, dt_dtype, h_dtype, y_dtype,
                                use_delta_softplus, delta_min, delta_max, reinterpret_cast<cudaStream_t>(stream)));
}

int ssm_conv_prefill(const void* hbc, int64_t row_stride, const float* weight, const float* bias, void* x, void* B,
                     void* C, void* conv_ctx, const int64_t* lengths, int64_t batch, int64_t seqlen, int64_t inner,
                     int64_t gn, int64_t kernel_size, int32_t dtype, void* stream) {
  if (!hbc || !weight || !x || !B || !C) return SSD_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || seqlen <= 0 || inner <= 0 || gn <= 0 || kernel_size < 1 || kernel_size > 8)
    return SSD_ERR_INVALID_ARGUMENT;
  if (row_stride < inner + 2 * gn) return SSD_ERR_INVALID_ARGUMENT;
  if (batch > 65535 || seqlen > 0x7fffffffll || inner + 2 * gn > 0x7fffffffll) return SSD_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  return cuda_status(launch_ssm_conv_prefill(hbc, (long long)row_stride, weight, bias, x, B, C, conv_ctx, lengths,
                                             (int)batch, (int)seqlen, (int)inner, (int)gn, (int)kernel_size, dtype,
                                             reinterpret_cast<cudaStream_t>(stream)));
}

int ssm_conv_decode(const void* hbc_new, int64_t row_stride, void* conv_ctx, const float* weight, const float* bias,
                    void* x, void* B, void* C, int64_t batch, int64_t inner, int64_t gn, int64_t kernel_size,
                    int32_t dtype, void* stream) {
  if (!hbc_new || !conv_ctx || !weight || !x || !B || !C) return SSD_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || inner <= 0 || gn <= 0 || kernel_size < 1 || kernel_size > 8) return SSD_ERR_INVALID_ARGUMENT;
  if (row_stride < inner + 2 * gn || batch * (inner + 2 * gn) > 0x7fffffffffll) return SSD_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  return cuda_status(launch_ssm_conv_decode(hbc_new, (long long)row_stride, conv_ctx, weight, bias, x, B, C,
                                            (int)batch, (int)inner, (int)gn, (int)kernel_size, dtype,
                                            reinterpret_cast<cudaStream_t>(stream)));
}

int sattn_decode_step(const void* q_rot, const void* k_rot, const void* v, const float* log_gate, void* k_cache,
                      void* v_cache, float* log_gate_cache, int64_t write_idx, int64_t capacity, void* out,
                      int64_t batch, int64_t nheads, int64_t head_dim, float scale, int32_t dtype, void* stream) {
  if (!q_rot || !k_rot || !v || !log_gate || !k_cache || !v_cache || !log_gate_cache || !out)
    return SSD_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || nheads <= 0 || capacity <= 0 || write_idx < 0 || write_idx >= capacity)
    return SSD_ERR_INVALID_ARGUMENT;
  if (!sattn_decode_supported((int)head_dim) || batch * nheads > 0x7fffffffll || capacity > 0x7fffffffll)
    return SSD_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  if (!aligned16(q_rot) || !aligned16(k_cache) || !aligned16(v_cache)) return SSD_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_sattn_decode(q_rot, k_rot, v, log_gate, k_cache, v_cache, log_gate_cache,
                                         (long long)write_idx, (long long)capacity, out, batch * nheads,
                                         (int)head_dim, scale, dtype, reinterpret_cast<cudaStream_t>(stream)));
}

int sattn_prefill_fwd(const void* q_rot, const void* k_rot, const void* v, const float* log_gate, void* out,
                      int64_t batch, int64_t nheads, int64_t seqlen, int64_t head_dim, float scale, int32_t dtype,
                      int32_t impl, void* stream) {
  if (!q_rot || !k_rot || !v || !log_gate || !out) return SSD_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || nheads <= 0 || seqlen <= 0 || batch > 65535 || nheads > 65535 || seqlen > 0x7fffffffll)
    return SSD_ERR_INVALID_ARGUMENT;
  if (!sattn_prefill_supported((int)head_dim)) return SSD_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  if (!aligned16(q_rot) || !aligned16(k_rot) || !aligned16(v)) return SSD_ERR_INVALID_ARGUMENT;
  const bool tc_ok = sattn_prefill_tc_supported((int)head_dim, dtype);
  if (impl == SSD_IMPL_TC && (!tc_ok || !aligned16(out))) return SSD_ERR_INVALID_ARGUMENT;
  const int use_tc = impl != SSD_IMPL_SIMT && tc_ok && aligned16(out);
  return cuda_status(launch_sattn_prefill(q_rot, k_rot, v, log_gate, out, (int)batch, (int)nheads, (int)seqlen,
                                          (int)head_dim, scale, dtype, use_tc,
                                          reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"

namespace {

// Checks the training-attention parameters and carves the workspace (base NULL: size only).
int train_args(const sattn_train_params* p, SattnTrainArgs* a, size_t* need) {
  if (!p) return SSD_ERR_INVALID_ARGUMENT;
  if (p->batch <= 0 || p->nheads <= 0 || p->seqlen <= 0 || p->batch > 65535 || p->nheads > 65535 ||
      p->seqlen > (1ll << 30))
    return SSD_ERR_INVALID_ARGUMENT;
  if (!sattn_train_supported((int)p->head_dim)) return SSD_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(p->dtype)) return SSD_ERR_UNSUPPORTED_DTYPE;
  const size_t B = (size_t)p->batch, H = (size_t)p->nheads, L = (size_t)p->seqlen;
  const size_t nt = (L + 63) / 64;
  uint8_t* base = reinterpret_cast<uint8_t*>(p->workspace);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* ptr = base ? base + off : nullptr;
    off += align_up(n);
    return ptr;
  };
  a->part = reinterpret_cast<double*>(take(B * H * nt * 2 * sizeof(double)));
  a->Di = reinterpret_cast<float*>(take(B * H * L * sizeof(float)));
  a->dlg = reinterpret_cast<float*>(take(B * H * L * sizeof(float)));
  a->dkb = reinterpret_cast<float*>(take(B * H * L * (size_t)p->head_dim * sizeof(float)));
  a->gk = reinterpret_cast<float*>(take(B * H * L * (size_t)p->head_dim * sizeof(float)));
  *need = off;
  a->B = (int)B;
  a->H = (int)H;
  a->L = (int)L;
  a->D = (int)p->head_dim;
  a->dtype = p->dtype;
  a->causal = p->is_causal ? 1 : 0;
  const bool tc_ok = sattn_train_tc_supported((int)p->head_dim, p->dtype);
  if (p->impl == SSD_IMPL_TC && !tc_ok) return SSD_ERR_INVALID_ARGUMENT;
  a->use_tc = p->impl != SSD_IMPL_SIMT && tc_ok;
  a->scale = p->scale;
  a->penalty = p->log_gate_penalty;
  a->q = p->q_rot;
  a->k = p->k_rot;
  a->v = p->v;
  a->gate = p->select_gate;
  a->lengths = p->lengths;
  a->out = p->out;
  a->lse = p->lse;
  a->lg = p->log_gate;
  a->stats = p->stats;
  return SSD_OK;
}

int train_common_checks(const sattn_train_params* p, const SattnTrainArgs& a, size_t need) {
  if (!p->q_rot || !p->k_rot || !p->v || !p->select_gate || !p->out || !p->lse || !p->log_gate || !p->stats ||
      !p->workspace)
    return SSD_ERR_INVALID_ARGUMENT;
  if (!aligned16(p->q_rot) || !aligned16(p->k_rot) || !aligned16(p->v) || !aligned16(p->out))
    return SSD_ERR_INVALID_ARGUMENT;
  if (p->workspace_bytes < need) return SSD_ERR_WORKSPACE_TOO_SMALL;
  (void)a;
  return SSD_OK;
}

}  // namespace

extern "C" {

size_t sattn_train_workspace_size(const sattn_train_params* p) {
  SattnTrainArgs a{};
  size_t need = 0;
  sattn_train_params q = p ? *p : sattn_train_params{};
  q.workspace = nullptr;
  return train_args(&q, &a, &need) == SSD_OK ? need : 0;
}

int sattn_train_fwd(const sattn_train_params* p, void* stream) {
  SattnTrainArgs a{};
  size_t need = 0;
  int st = train_args(p, &a, &need);
  if (st) return st;
  if ((st = train_common_checks(p, a, need))) return st;
  return cuda_status(launch_sattn_train_fwd(a, reinterpret_cast<cudaStream_t>(stream)));
}

int sattn_train_bwd(const sattn_train_params* p, const void* dout, void* dq, void* dk, void* dv, void* dselect_gate,
                    void* stream) {
  SattnTrainArgs a{};
  size_t need = 0;
  int st = train_args(p, &a, &need);
  if (st) return st;
  if ((st = train_common_checks(p, a, need))) return st;
  if (!dout || !dq || !dk || !dv || !dselect_gate) return SSD_ERR_INVALID_ARGUMENT;
  if (!aligned16(dout)) return SSD_ERR_INVALID_ARGUMENT;
  return cuda_status(launch_sattn_train_bwd(a, dout, dq, dk, dv, dselect_gate, reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"
