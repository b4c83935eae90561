// State-only passes of the sequence-parallel EMA (kernels/ema_sp.py) as
// weighted column sums.
//
// For one row (a sub-span) of the dt-form recurrence z_t = exp(dt_t A_h)
// z_{t-1} + dt_t x_t, with cs_t = A_h sum_{u <= t} dt_u:
//
//   direction 0  end state from a zero start   out = sum_t exp(cs_end - cs_t) dt_t x_t
//   direction 1  gradient w.r.t. the start      out = sum_t exp(cs_t) dy_t
//                state, from the row's own dy
//
// Neither needs the recurrence's sequential scan or a look-back between
// tiles: every token's weight follows from the within-row cumsum of dt A, and
// the sum over tokens is a reduction.  One CTA of 8 warps per (row, head) walks
// its row in 1024-token blocks: a block scan of dt A (the block's first x loads
// and the next block's dt in flight meanwhile), then the block's tokens stream
// in sub-blocks: each lane issues sixteen 16-byte loads before its FMAs, a warp
// load covering 512 bytes of whole token rows (lane l: 16 bytes of channels of
// one row); a lane's running sum combines over the blocks through the block decay (direction 0:
// S <- exp(ld_block) S + block sum; direction 1: G <- G + block sum, the
// weights carrying exp(cs before the block)), and the lanes' and warps' sums --
// disjoint tokens -- add up at the end.  fp32 arithmetic, as the scan kernels;
// optionally the row's log decay A_h sum dt, summed in float64, for the folds.
// HBM-bound: x (or dy) is read once, coalesced.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "ema_common.cuh"
#include "ema_scan_dispatch.h"
#include "ema_ssd_b200.h"

namespace emab {
void set_last_error(const char* msg);

namespace spstate {

constexpr int kBlock = 1024;  // tokens per block
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTPT = kBlock / kThreads;  // tokens per thread in the block scan

struct Params {
  int L, H;
  const void* x;
  long long sr, sl, sh;  // element strides of row, token, head
  const float* dt;       // (rows, L, H)
  const float* A;
  float* out;            // (rows, H, P)
  double* ld;            // (rows, H) A_h sum dt, or null
  int dir;
};

template <typename T, int P>
__global__ void __launch_bounds__(kThreads, 2) span_state_kernel(const Params p) {
  constexpr int EPL = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte lane load
  constexpr int LPR = P / EPL;                           // lanes per token row
  constexpr int RPW = 32 / LPR;                          // token rows per warp load
  constexpr int NL = 16;                                 // loads in flight per lane
  constexpr int SUB = kWarps * RPW * NL;                 // tokens per sub-block
  static_assert(LPR >= 1 && LPR <= 32 && 32 % LPR == 0, "headdim");
  static_assert(kBlock % SUB == 0, "sub-blocks tile the block");
  __shared__ float s_w[kBlock];          // the block's per-token weights
  __shared__ float s_wsum[kWarps];       // per-warp scan totals
  __shared__ float s_red[kWarps][P];     // per-warp sums, reduced at the end
  __shared__ double s_dsum[kWarps];      // per-warp float64 sums of dt
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = blockIdx.x / p.H, h = blockIdx.x % p.H;
  const float Ah = p.A[h];
  const int rsub = lane / LPR;  // this lane's token within a warp load
  const T* xbase = static_cast<const T*>(p.x) + row * p.sr + h * p.sh + EPL * (lane % LPR);
  const float* dtbase = p.dt + static_cast<size_t>(row) * p.L * p.H + h;
  float acc[EPL];  // this lane's tokens, weighted, combined over the blocks so far
#pragma unroll
  for (int k = 0; k < EPL; ++k) acc[k] = 0.f;
  float before = 0.f;  // direction 1: the cumsum of dt A before the block
  double dsum = 0.0;   // this thread's dt, summed in float64 (the row's log decay)
  float dn[kTPT];      // dt of the next block, fetched while this block's x streams
#pragma unroll
  for (int k = 0; k < kTPT; ++k) {
    const int t = tid * kTPT + k;
    dn[k] = (t < p.L) ? dtbase[static_cast<size_t>(t) * p.H] : 0.f;
  }
  uint4 raw[NL];
  auto load_sub = [&](int t0, int s0, int n) {
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      const int t = s0 + (i * kWarps + warp) * RPW + rsub;
      raw[i] = (t < n) ? __ldg(reinterpret_cast<const uint4*>(xbase + static_cast<long long>(t0 + t) * p.sl))
                       : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  for (int t0 = 0; t0 < p.L; t0 += kBlock) {
    const int n = min(kBlock, p.L - t0);
    load_sub(t0, 0, n);  // the block's first x in flight through the scan
    // ---- block scan of dt A -------------------------------------------------------
    float d[kTPT], v[kTPT];
    float run = 0.f;
#pragma unroll
    for (int k = 0; k < kTPT; ++k) {
      d[k] = dn[k];
      dsum += static_cast<double>(d[k]);
      run += d[k] * Ah;
      v[k] = run;
    }
#pragma unroll
    for (int k = 0; k < kTPT; ++k) {  // the next block's dt
      const int t = t0 + kBlock + tid * kTPT + k;
      dn[k] = (t < p.L) ? dtbase[static_cast<size_t>(t) * p.H] : 0.f;
    }
    float incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    float wpre = 0.f, total = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float sw = s_wsum[w];
      if (w < warp) wpre += sw;
      total += sw;
    }
    const float excl = wpre + incl - run;  // cumsum before this thread's first token
#pragma unroll
    for (int k = 0; k < kTPT; ++k) {
      const int t = tid * kTPT + k;
      const float cs = excl + v[k];  // within the block, through token t
      s_w[t] = (t >= n) ? 0.f : (p.dir == 0 ? __expf(total - cs) * d[k] : __expf(before + cs));
    }
    __syncthreads();
    // ---- weighted column sums: NL 16-byte loads in flight per lane, then the FMAs ----
    float bs[EPL];
#pragma unroll
    for (int k = 0; k < EPL; ++k) bs[k] = 0.f;
    for (int s0 = 0; s0 < n; s0 += SUB) {
      if (s0 > 0) load_sub(t0, s0, n);
#pragma unroll
      for (int i = 0; i < NL; ++i) {
        const float w = s_w[s0 + (i * kWarps + warp) * RPW + rsub];  // 0 past the row's end
        const T* e = reinterpret_cast<const T*>(&raw[i]);
#pragma unroll
        for (int k = 0; k < EPL; ++k) bs[k] = fmaf(w, to_f32(e[k]), bs[k]);
      }
    }
    if (p.dir == 0) {
      const float dec = __expf(total);
#pragma unroll
      for (int k = 0; k < EPL; ++k) acc[k] = fmaf(dec, acc[k], bs[k]);
    } else {
#pragma unroll
      for (int k = 0; k < EPL; ++k) acc[k] += bs[k];
      before += total;
    }
    __syncthreads();  // s_w / s_wsum are rewritten by the next block
  }
  // ---- the lanes' and warps' sums (linear combinations of disjoint tokens) ----------
#pragma unroll
  for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
    for (int k = 0; k < EPL; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
  if (lane < LPR)
#pragma unroll
    for (int k = 0; k < EPL; ++k) s_red[warp][EPL * lane + k] = acc[k];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
  if (lane == 0) s_dsum[warp] = dsum;
  __syncthreads();
  if (p.ld != nullptr && tid == 0) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += s_dsum[w];
    p.ld[static_cast<size_t>(row) * p.H + h] = t * static_cast<double>(Ah);
  }
  for (int c = tid; c < P; c += kThreads) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) sum += s_red[w][c];
    p.out[(static_cast<size_t>(row) * p.H + h) * P + c] = sum;
  }
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_last_error(buf);
  return code;
}

template <typename T, int P>
int launch_t(const Params& p, long long rows, cudaStream_t s) {
  span_state_kernel<T, P><<<static_cast<unsigned>(rows * p.H), kThreads, 0, s>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ema_span_state launch failed: %s", cudaGetErrorString(e));
  return EMA_OK;
}

template <typename T>
int launch_p(const Params& p, long long rows, int P, cudaStream_t s) {
  switch (P) {
    case 32: return launch_t<T, 32>(p, rows, s);
    case 64: return launch_t<T, 64>(p, rows, s);
    case 128: return launch_t<T, 128>(p, rows, s);
    default: return fail(EMA_ERR_UNSUPPORTED, "ema_span_state: headdim 32, 64 or 128");
  }
}

}  // namespace spstate
}  // namespace emab

extern "C" EMA_API int ema_span_state_launch(const EmaSpanStateArgs* a, void* stream) {
  using namespace emab::spstate;
  if (a == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_state: args is NULL");
  if (a->rows < 0 || a->seqlen < 0 || a->nheads <= 0 || a->headdim <= 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_state: bad shape");
  if (a->direction != 0 && a->direction != 1)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_state: direction 0 or 1");
  if (a->x == nullptr || a->dt == nullptr || a->A == nullptr || a->out == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_state: x, dt, A and out are required");
  if (a->rows * a->nheads > 2147483647LL || a->seqlen > 2147483647LL)
    return fail(EMA_ERR_UNSUPPORTED, "ema_span_state: shape too large");
  const int es = a->dtype == EMA_DTYPE_F32 ? 4 : 2;
  if (a->dtype != EMA_DTYPE_F32 && a->dtype != EMA_DTYPE_BF16 && a->dtype != EMA_DTYPE_F16)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_state: unknown dtype %d", a->dtype);
  if (reinterpret_cast<uintptr_t>(a->x) % 16u != 0u)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_state: x must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if ((a->x_stride[i] * es) % 16 != 0)
      return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_state: x strides must be multiples of 16 bytes");
  if (a->rows == 0 || a->seqlen == 0) {
    const size_t n = static_cast<size_t>(a->rows) * a->nheads;
    cudaError_t e = n ? cudaMemsetAsync(a->out, 0, n * a->headdim * sizeof(float), static_cast<cudaStream_t>(stream))
                      : cudaSuccess;
    if (e == cudaSuccess && n && a->log_decay != nullptr)
      e = cudaMemsetAsync(a->log_decay, 0, n * sizeof(double), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EMA_OK : fail(EMA_ERR_CUDA, "ema_span_state: %s", cudaGetErrorString(e));
  }
  Params p{static_cast<int>(a->seqlen), static_cast<int>(a->nheads), a->x, a->x_stride[0], a->x_stride[1],
           a->x_stride[2], a->dt, a->A, a->out, a->log_decay, a->direction};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int P = static_cast<int>(a->headdim);
  switch (a->dtype) {
    case EMA_DTYPE_F32: return launch_p<float>(p, a->rows, P, s);
    case EMA_DTYPE_BF16: return launch_p<__nv_bfloat16>(p, a->rows, P, s);
    default: return launch_p<__half>(p, a->rows, P, s);
  }
}
