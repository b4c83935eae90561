// C ABI of the EMA scan library: argument validation, TMA tensor maps,
// workspace carving and kernel dispatch.  Nothing here allocates memory.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <mutex>
#include <string>

#include "ema_scan_dispatch.h"
#include "ema_ssd_b200.h"

namespace emab {

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// The driver's tensor-map encoder needs a current context on the calling
// thread.  A thread that has made no runtime call that binds one (an autograd
// worker whose first CUDA work is this launch, for instance) has none, and
// the encoder then fails with CUDA_ERROR_INVALID_CONTEXT: bind the current
// device's primary context first (once per thread and device).
int bind_thread_context() {
  thread_local int bound = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (bound == dev) return EMA_OK;
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
  bound = dev;
  return EMA_OK;
}

int elem_size(int dtype) { return dtype == EMA_DTYPE_F32 ? 4 : 2; }

CUtensorMapDataType map_dtype(int dtype) {
  switch (dtype) {
    case EMA_DTYPE_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case EMA_DTYPE_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  }
}

// A (B, L, H, P) tensor written with vector stores: 16-byte aligned base and
// strides that are multiples of 16 bytes (channel stride 1).
int check_tile_tensor(const void* ptr, int dtype, const int64_t st[3], const char* name) {
  const int es = elem_size(dtype);
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "%s: base address must be 16-byte aligned", name);
  for (int i = 0; i < 3; ++i) {
    if (st[i] <= 0 || (st[i] * es) % 16 != 0)
      return fail(EMA_ERR_INVALID_ARGUMENT,
                  "%s: stride %d (%lld elements) must be positive and a multiple of 16 bytes", name, i,
                  static_cast<long long>(st[i]));
  }
  return EMA_OK;
}

// 4-D map over a (B, L, H, P) tensor with unit channel stride; box = one
// (chunk, batch, head) tile of BP channels x Q tokens.
int make_tile_map(CUtensorMap* m, const void* ptr, int dtype, int64_t B, int64_t L, int64_t H,
                  int64_t P, const int64_t st[3], int BP, int Q, const char* name) {
  const int es = elem_size(dtype);
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "%s: base address must be 16-byte aligned", name);
  for (int i = 0; i < 3; ++i) {
    if (st[i] <= 0 || (st[i] * es) % 16 != 0)
      return fail(EMA_ERR_INVALID_ARGUMENT,
                  "%s: stride %d (%lld elements) must be positive and a multiple of 16 bytes", name, i,
                  static_cast<long long>(st[i]));
  }
  if (int r = bind_thread_context()) return r;
  auto enc = encode_fn();
  if (!enc) return fail(EMA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(P), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(L), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(st[2] * es), static_cast<cuuint64_t>(st[1] * es),
                           static_cast<cuuint64_t>(st[0] * es)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(BP), 1u, static_cast<cuuint32_t>(Q), 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = enc(m, map_dtype(dtype), 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EMA_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return EMA_OK;
}

int block_p_for(int64_t P) {
  if (P <= 64) return 64;
  if (P <= 128) return 128;
  return 0;
}

// Workspace: 256-byte header | dA partials [tiles][32] f32 | aggregate records
// [tiles][BP + 1] u64 | inclusive records [tiles][BP] u64.
struct WsLayout {
  size_t partial, agg, incl, total;
};

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

WsLayout ws_layout(int64_t tiles, int BP) {
  WsLayout l;
  size_t off = static_cast<size_t>(kHdrWords) * 4;
  l.partial = off;
  off = align256(off + static_cast<size_t>(tiles) * 32 * 4);
  l.agg = off;
  off = align256(off + static_cast<size_t>(tiles) * (BP + 1) * 8);
  l.incl = off;
  off = align256(off + static_cast<size_t>(tiles) * BP * 8);
  l.total = off;
  return l;
}

int carve_workspace(void* ws, size_t bytes, int64_t tiles, int BP, ScanWorkspace* out) {
  if (ws == nullptr) return fail(EMA_ERR_WORKSPACE, "workspace is NULL");
  if (reinterpret_cast<uintptr_t>(ws) % 256 != 0)
    return fail(EMA_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  const WsLayout l = ws_layout(tiles, BP);
  if (bytes < l.total)
    return fail(EMA_ERR_WORKSPACE, "workspace too small: %zu bytes given, %zu needed", bytes, l.total);
  char* base = static_cast<char*>(ws);
  out->hdr = reinterpret_cast<uint32_t*>(base);
  out->partial = reinterpret_cast<float*>(base + l.partial);
  out->agg = reinterpret_cast<uint64_t*>(base + l.agg);
  out->incl = reinterpret_cast<uint64_t*>(base + l.incl);
  out->rec_end = reinterpret_cast<uint64_t*>(base + (bytes & ~static_cast<size_t>(7)));
  return EMA_OK;
}

int num_sms_of_current_device(int* n) {
  static int cache[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev >= 0 && dev < 64 && cache[dev] > 0) {
    *n = cache[dev];
    return EMA_OK;
  }
  e = cudaDeviceGetAttribute(n, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "SM count: %s", cudaGetErrorString(e));
  if (dev >= 0 && dev < 64) cache[dev] = *n;
  return EMA_OK;
}

int check_shape(int64_t B, int64_t L, int64_t H, int64_t P, int64_t Q, int dtype) {
  if (B < 0 || L < 0 || H <= 0 || P <= 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "bad shape batch=%lld seqlen=%lld nheads=%lld headdim=%lld",
                (long long)B, (long long)L, (long long)H, (long long)P);
  if (Q != 64 && Q != 128 && Q != 256)
    return fail(EMA_ERR_UNSUPPORTED, "chunk_size must be 64, 128 or 256 (got %lld)", (long long)Q);
  if (dtype != EMA_DTYPE_F32 && dtype != EMA_DTYPE_BF16 && dtype != EMA_DTYPE_F16)
    return fail(EMA_ERR_INVALID_ARGUMENT, "unknown dtype code %d", dtype);
  if (block_p_for(P) == 0)
    return fail(EMA_ERR_UNSUPPORTED, "headdim must be <= 128 (got %lld)", (long long)P);
  if ((P * elem_size(dtype)) % 16 != 0)
    return fail(EMA_ERR_UNSUPPORTED, "headdim * element size must be a multiple of 16 bytes (headdim=%lld)",
                (long long)P);
  const int64_t nc = (L + Q - 1) / Q;
  if (B > INT32_MAX || L > INT32_MAX || H > INT32_MAX || B * H * nc > INT32_MAX)
    return fail(EMA_ERR_UNSUPPORTED, "problem too large for 32-bit tile indices");
  return EMA_OK;
}

// dt (B, L, H) -> (B, H, L) through a 32 x 33 shared tile: each warp reads
// 32 heads of one token (one 128-byte row) and writes 32 tokens of one head.
// Grid (ceil(L/32), ceil(H/32), B), 256 threads.
__global__ void __launch_bounds__(256) dt_rows_kernel(const float* __restrict__ dt, float* __restrict__ rows, int L,
                                                      int H) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z, t0 = blockIdx.x * 32, h0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const float* src = dt + static_cast<size_t>(b) * L * H;
  grid_dep_wait();
#pragma unroll
  for (int r = ty; r < 32; r += 8) {
    const int t = t0 + r, h = h0 + tx;
    if (t < L && h < H) tile[r][tx] = src[static_cast<size_t>(t) * H + h];
  }
  __syncthreads();
  float* dst = rows + static_cast<size_t>(b) * H * L;
#pragma unroll
  for (int r = ty; r < 32; r += 8) {
    const int h = h0 + r, t = t0 + tx;
    if (t < L && h < H) dst[static_cast<size_t>(h) * L + t] = tile[tx][r];
  }
  grid_dep_release();
}

// dt (B, L, H) -> (B, H, L): one contiguous row per (batch, head), so each
// scan tile loads its dt with one bulk copy.
int launch_dt_rows(const float* dt, float* rows, int64_t B, int64_t L, int64_t H, cudaStream_t s) {
  if (reinterpret_cast<uintptr_t>(rows) % 16 != 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "dt_rows must be 16-byte aligned");
  if (B > 65535 || (H + 31) / 32 > 65535)
    return fail(EMA_ERR_UNSUPPORTED, "dt_rows: batch or nheads too large for the transpose grid");
  dim3 grid(static_cast<unsigned>((L + 31) / 32), static_cast<unsigned>((H + 31) / 32), static_cast<unsigned>(B));
  cudaError_t e = launch_programmatic(dt_rows_kernel, grid, dim3(256), 0, s, dt, rows, static_cast<int>(L),
                                      static_cast<int>(H));
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "dt_rows: launch failed: %s", cudaGetErrorString(e));
  return EMA_OK;
}

int map_dispatch_result(int r, const char* what) {
  if (r == 0) return EMA_OK;
  if (r == -1) return fail(EMA_ERR_UNSUPPORTED, "%s: no kernel for this combination", what);
  if (r == -2) return fail(EMA_ERR_UNSUPPORTED, "%s: tile needs more shared memory than a CTA has", what);
  return fail(EMA_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(static_cast<cudaError_t>(r)));
}

}  // namespace

void set_last_error(const char* msg) { g_last_error = msg; }

namespace {
// bit 0: the tensor-core backward, bit 1: the tensor-core forward.  Off by
// default: both agree with the CUDA-core kernels within the bf16 tolerance but
// are slower on the benchmark shape.
std::atomic<int> g_tensor_core_path{0};
}
bool tensor_core_path_enabled() { return (g_tensor_core_path.load(std::memory_order_relaxed) & 1) != 0; }
bool fwd_tensor_core_path_enabled() { return (g_tensor_core_path.load(std::memory_order_relaxed) & 2) != 0; }

int encode_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* ptr, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128) {
  if (int r = bind_thread_context()) return r;
  auto enc = encode_fn();
  if (!enc) return fail(EMA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return fail(EMA_ERR_INVALID_ARGUMENT, "TMA base not 16-byte aligned");
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1u;
    if (i + 1 < rank) {
      if (strides_bytes[i] % 16 != 0) return fail(EMA_ERR_INVALID_ARGUMENT, "TMA stride not a multiple of 16 bytes");
      st[i] = strides_bytes[i];
    }
  }
  CUresult r = enc(m, dt, rank, const_cast<void*>(ptr), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(EMA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return EMA_OK;
}

int ensure_smem_attr(const void* fn, int bytes, unsigned long long* device_mask) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  const unsigned long long bit = (dev < 64) ? (1ull << dev) : 0ull;
  auto* m = reinterpret_cast<std::atomic<unsigned long long>*>(device_mask);
  if (bit && (m->load(std::memory_order_acquire) & bit)) return 0;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (bit) m->fetch_or(bit, std::memory_order_acq_rel);
  return 0;
}

}  // namespace emab

using namespace emab;

extern "C" {

size_t ema_scan_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads, int64_t headdim,
                               int64_t chunk_size) {
  if (batch <= 0 || seqlen <= 0 || nheads <= 0 || headdim <= 0 || chunk_size <= 0) return 256;
  const int BP = block_p_for(headdim) ? block_p_for(headdim) : 128;
  const int64_t nc = (seqlen + chunk_size - 1) / chunk_size;
  return ws_layout(batch * nheads * nc, BP).total;
}

int ema_fwd_launch(const EmaFwdArgs* a, void* stream) {
  if (a == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "args is NULL");
  int r = check_shape(a->batch, a->seqlen, a->nheads, a->headdim, a->chunk_size, a->dtype);
  if (r) return r;
  if (a->batch == 0 || a->seqlen == 0) return EMA_OK;
  if (a->x == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "x is required");
  if (a->out == nullptr && a->final_state == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "out is required (a state-only forward needs final_state)");
  const bool ref_form = a->dA != nullptr;
  const bool dt_form = a->dt != nullptr || a->A != nullptr;
  if (ref_form == dt_form || (dt_form && (a->dt == nullptr || a->A == nullptr)))
    return fail(EMA_ERR_INVALID_ARGUMENT, "give either dA, or both dt and A");
  if (dt_form && (a->da_cs != nullptr || a->da_cs_sum != nullptr))
    return fail(EMA_ERR_INVALID_ARGUMENT, "da_cs / da_cs_sum are outputs of the dA form only");
  const bool seq = a->seq_idx != nullptr;
  if (seq && (a->seq_idx_type < EMA_IDX_I8 || a->seq_idx_type > EMA_IDX_I64))
    return fail(EMA_ERR_INVALID_ARGUMENT, "seq_idx_type must be EMA_IDX_I8/I32/I64");
  if (seq && dt_form) return fail(EMA_ERR_UNSUPPORTED, "seq_idx is supported with the dA form only");

  const int Q = static_cast<int>(a->chunk_size);
  const int BP = block_p_for(a->headdim);
  const int64_t nc = (a->seqlen + Q - 1) / Q;
  const int64_t tiles = a->batch * a->nheads * nc;

  FwdLaunch l{};
  FwdParams& p = l.params;
  r = carve_workspace(a->workspace, a->workspace_bytes, tiles, BP, &p.ws);
  if (r) return r;
  CUtensorMap mx;
  r = make_tile_map(&mx, a->x, a->dtype, a->batch, a->seqlen, a->nheads, a->headdim, a->x_stride, BP, Q, "x");
  if (r) return r;
  if (a->out != nullptr) {
    r = check_tile_tensor(a->out, a->dtype, a->out_stride, "out");
    if (r) return r;
  }
  p.B = static_cast<int>(a->batch);
  p.L = static_cast<int>(a->seqlen);
  p.H = static_cast<int>(a->nheads);
  p.P = static_cast<int>(a->headdim);
  p.nc = static_cast<int>(nc);
  p.div_bh = make_fast_div(static_cast<uint32_t>(a->batch * a->nheads));
  p.div_h = make_fast_div(static_cast<uint32_t>(a->nheads));
  p.rows = a->dA;
  p.dt = a->dt;
  p.A = a->A;
  p.dt_rows = 0;
  if (a->dt_rows != nullptr) {
    if (!dt_form) return fail(EMA_ERR_INVALID_ARGUMENT, "dt_rows: dt form only");
    r = launch_dt_rows(a->dt, a->dt_rows, a->batch, a->seqlen, a->nheads, static_cast<cudaStream_t>(stream));
    if (r) return r;
    p.dt = a->dt_rows;
    p.dt_rows = 1;
  }
  p.seq_idx = a->seq_idx;
  p.seq_idx_type = a->seq_idx_type;
  p.init = a->initial_state;
  p.states = a->states;
  p.st_b = a->states_stride[0];
  p.st_c = a->states_stride[1];
  p.st_h = a->states_stride[2];
  p.st_p = a->states_stride[3];
  if (a->mid_states != nullptr) {
    if (!dt_form || seq) return fail(EMA_ERR_UNSUPPORTED, "mid_states: dt form without seq_idx only");
    if (Q % 2 != 0 || (Q / 2) % fwd_segment_tokens(BP) != 0)
      return fail(EMA_ERR_UNSUPPORTED, "mid_states: chunk_size / 2 must be a multiple of %d", fwd_segment_tokens(BP));
  }
  p.mid_states = a->mid_states;
  p.sm_b = a->mid_states_stride[0];
  p.sm_c = a->mid_states_stride[1];
  p.sm_h = a->mid_states_stride[2];
  p.sm_p = a->mid_states_stride[3];
  p.da_cs = a->da_cs;
  p.da_cs_sum = a->da_cs_sum;
  p.final_state = a->final_state;
  p.y = a->out;
  p.sy_b = a->out_stride[0];
  p.sy_l = a->out_stride[1];
  p.sy_h = a->out_stride[2];
  l.map_x = &mx;
  l.block_p = BP;
  l.chunk = Q;
  l.mode = ref_form ? kFwdLog2 : kFwdDt;
  l.seq = seq;
  l.tiles = tiles;
  r = num_sms_of_current_device(&l.num_sms);
  if (r) return r;
  l.stream = static_cast<cudaStream_t>(stream);
  if (fwd_tensor_core_path_enabled()) {
    r = fwd_tc_launch(l, a->dtype, a->x, a->x_stride, a->out, a->out_stride);
    if (r == 0) return EMA_OK;
    if (r == -3) return EMA_ERR_CUDA;
    if (r != 1) return map_dispatch_result(r, "ema_fwd (tensor cores)");
  }
  switch (a->dtype) {
    case EMA_DTYPE_BF16: r = fwd_dispatch_bf16(l); break;
    case EMA_DTYPE_F16: r = fwd_dispatch_f16(l); break;
    default: r = fwd_dispatch_f32(l); break;
  }
  return map_dispatch_result(r, "ema_fwd");
}

int ema_bwd_launch(const EmaBwdArgs* a, void* stream) {
  if (a == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "args is NULL");
  int r = check_shape(a->batch, a->seqlen, a->nheads, a->headdim, a->chunk_size, a->dtype);
  if (r) return r;
  if (a->batch == 0 || a->seqlen == 0) return EMA_OK;
  if (a->x == nullptr || a->dout == nullptr || a->states == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "x, dout and states are required");
  const bool state_only = a->dx == nullptr;
  if (state_only && a->d_initial_state == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "dx is required (a state-only backward needs d_initial_state)");
  const bool ref_form = a->da_cs != nullptr;
  const bool dt_form = a->dt != nullptr || a->A != nullptr;
  if (ref_form == dt_form || (dt_form && (a->dt == nullptr || a->A == nullptr)))
    return fail(EMA_ERR_INVALID_ARGUMENT, "give either da_cs, or both dt and A");
  if (!state_only && ref_form && a->dl == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "dl output is required with da_cs");
  if (!state_only && dt_form && (a->ddt == nullptr || a->dA_out == nullptr))
    return fail(EMA_ERR_INVALID_ARGUMENT, "ddt and dA_out outputs are required with dt/A");

  const int Q = static_cast<int>(a->chunk_size);
  const int BP = block_p_for(a->headdim);
  const int64_t nc = (a->seqlen + Q - 1) / Q;
  const int64_t tiles = a->batch * a->nheads * nc;

  BwdLaunch l{};
  BwdParams& p = l.params;
  r = carve_workspace(a->workspace, a->workspace_bytes, tiles, BP, &p.ws);
  if (r) return r;
  CUtensorMap mx, mdy;
  r = make_tile_map(&mx, a->x, a->dtype, a->batch, a->seqlen, a->nheads, a->headdim, a->x_stride, BP, Q, "x");
  if (r) return r;
  r = make_tile_map(&mdy, a->dout, a->dtype, a->batch, a->seqlen, a->nheads, a->headdim, a->dout_stride, BP,
                    Q, "dout");
  if (r) return r;
  CUtensorMap mdx = mdy;  // a state-only pass stores no dx
  if (!state_only) {
    r = make_tile_map(&mdx, a->dx, a->dtype, a->batch, a->seqlen, a->nheads, a->headdim, a->dx_stride, BP,
                      bwd_segment_tokens(BP), "dx");
    if (r) return r;
  }
  p.B = static_cast<int>(a->batch);
  p.L = static_cast<int>(a->seqlen);
  p.H = static_cast<int>(a->nheads);
  p.P = static_cast<int>(a->headdim);
  p.nc = static_cast<int>(nc);
  p.div_bh = make_fast_div(static_cast<uint32_t>(a->batch * a->nheads));
  p.div_h = make_fast_div(static_cast<uint32_t>(a->nheads));
  p.rows = a->da_cs;
  p.dt = a->dt;
  p.A = a->A;
  p.dt_rows = 0;  // the rows copy is switched in below, for the CUDA-core kernel only
  if (a->dt_rows != nullptr && !dt_form) return fail(EMA_ERR_INVALID_ARGUMENT, "dt_rows: dt form only");
  p.states = a->states;
  p.st_b = a->states_stride[0];
  p.st_c = a->states_stride[1];
  p.st_h = a->states_stride[2];
  p.st_p = a->states_stride[3];
  p.d_final = a->d_final_state;
  p.d_last = a->d_last_token;
  p.dl = a->dl;
  p.ddt = a->ddt;
  p.dA_out = a->dA_out;
  p.d_init = a->d_initial_state;
  p.dx = a->dx;
  p.sdx_b = a->dx_stride[0];
  p.sdx_l = a->dx_stride[1];
  p.sdx_h = a->dx_stride[2];
  l.map_x = &mx;
  l.map_dy = &mdy;
  l.map_dx = &mdx;
  l.block_p = BP;
  l.chunk = Q;
  l.mode = ref_form ? kBwdCumsum : kBwdDt;
  l.tiles = tiles;
  r = num_sms_of_current_device(&l.num_sms);
  if (r) return r;
  l.stream = static_cast<cudaStream_t>(stream);
  if (tensor_core_path_enabled()) {
    r = bwd_tc_launch(l, a->dtype, a->x, a->x_stride, a->dout, a->dout_stride, a->dx, a->dx_stride);
    if (r == 0) return EMA_OK;
    if (r == -3) return EMA_ERR_CUDA;
    if (r != 1) return map_dispatch_result(r, "ema_bwd (tensor cores)");
  }
  if (a->dt_rows != nullptr) {
    p.dt = a->dt_rows;
    p.dt_rows = 1;
  }
  switch (a->dtype) {
    case EMA_DTYPE_BF16: r = bwd_dispatch_bf16(l); break;
    case EMA_DTYPE_F16: r = bwd_dispatch_f16(l); break;
    default: r = bwd_dispatch_f32(l); break;
  }
  return map_dispatch_result(r, "ema_bwd");
}

int chunk_cumsum_launch(const float* dA, const int64_t dA_stride[3], float* dA_cs, const int64_t cs_stride[3],
                        float* dA_cs_rev, const int64_t rev_stride[3], int64_t batch, int64_t nheads,
                        int64_t seqlen, int64_t chunk_size, int32_t exp2, void* stream) {
  if (dA == nullptr || dA_cs == nullptr || dA_cs_rev == nullptr || dA_stride == nullptr ||
      cs_stride == nullptr || rev_stride == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "chunk_cumsum: NULL argument");
  if (batch < 0 || nheads < 0 || seqlen < 0 || chunk_size <= 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "chunk_cumsum: bad shape");
  if (chunk_size > 1024) return fail(EMA_ERR_UNSUPPORTED, "chunk_cumsum: chunk_size must be <= 1024");
  if (batch == 0 || nheads == 0 || seqlen == 0) return EMA_OK;
  const int64_t nc = (seqlen + chunk_size - 1) / chunk_size;
  if (nc > INT32_MAX || nheads > 65535 || batch > 65535)
    return fail(EMA_ERR_UNSUPPORTED, "chunk_cumsum: grid too large");
  dim3 grid(static_cast<unsigned>(nc), static_cast<unsigned>(nheads), static_cast<unsigned>(batch));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int L = static_cast<int>(seqlen), Q = static_cast<int>(chunk_size);
#define EMA_CC_LAUNCH(NTH)                                                                            \
  chunk_cumsum_kernel<NTH><<<grid, NTH, 0, s>>>(dA, dA_stride[0], dA_stride[1], dA_stride[2], dA_cs,  \
                                                cs_stride[0], cs_stride[1], cs_stride[2], dA_cs_rev,  \
                                                rev_stride[0], rev_stride[1], rev_stride[2], L, Q, exp2)
  if (Q <= 64) EMA_CC_LAUNCH(64);
  else if (Q <= 128) EMA_CC_LAUNCH(128);
  else if (Q <= 256) EMA_CC_LAUNCH(256);
  else if (Q <= 512) EMA_CC_LAUNCH(512);
  else EMA_CC_LAUNCH(1024);
#undef EMA_CC_LAUNCH
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "chunk_cumsum: launch failed: %s", cudaGetErrorString(e));
  return EMA_OK;
}

int ema_dt_rows_launch(const float* dt, float* dt_rows, int64_t batch, int64_t seqlen, int64_t nheads, void* stream) {
  if (dt == nullptr || dt_rows == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "dt_rows: NULL argument");
  if (batch < 0 || seqlen < 0 || nheads < 0) return fail(EMA_ERR_INVALID_ARGUMENT, "dt_rows: bad shape");
  if (batch == 0 || seqlen == 0 || nheads == 0) return EMA_OK;
  if (seqlen > INT32_MAX || nheads > INT32_MAX) return fail(EMA_ERR_UNSUPPORTED, "dt_rows: shape too large");
  return launch_dt_rows(dt, dt_rows, batch, seqlen, nheads, static_cast<cudaStream_t>(stream));
}

int ema_workspace_status(const void* workspace, uint32_t* status, void* stream) {
  if (workspace == nullptr || status == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "NULL argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t* word = static_cast<const uint32_t*>(workspace) + kHdrStatus;
  cudaError_t e = cudaMemcpyAsync(status, word, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "status read failed: %s", cudaGetErrorString(e));
  return EMA_OK;
}

int ema_workspace_clear_status(void* workspace, void* stream) {
  if (workspace == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "NULL workspace");
  uint32_t* word = static_cast<uint32_t*>(workspace) + kHdrStatus;
  cudaError_t e = cudaMemsetAsync(word, 0, sizeof(uint32_t), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "status clear failed: %s", cudaGetErrorString(e));
  return EMA_OK;
}

int ema_set_tensor_core_path(int32_t enable) {
  const int prev = g_tensor_core_path.exchange(enable & 3);
  return prev;
}

const char* ema_last_error(void) { return g_last_error.c_str(); }

const char* ema_version(void) { return "ema_ssd_b200 0.1.0 (sm_100a)"; }

}  // extern "C"
