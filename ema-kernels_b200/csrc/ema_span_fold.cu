// Sub-span folds of the sequence-parallel EMA (kernels/ema_sp.py).
//
// A rank's span of every (batch, head) chain is cut into K sub-spans run as
// batch rows.  With ld_k = A_h sum_{t in k} dt_t the log of sub-span k's decay,
// cl_k = sum_{j<k} ld_j and tot = sum_k ld_k, and V_k the sub-span's boundary
// value from its own inputs:
//
//   forward  (V_k: end state from a zero start)
//     summary   Vspan  = sum_k exp(tot - cl_k - ld_k) V_k          (the span's end state from zero)
//     expand    out_k  = exp(cl_k) Sin + sum_{q<k} exp(cl_k - cl_q - ld_q) V_q
//                                                                 (state entering sub-span k)
//   backward (V_k: gradient w.r.t. the sub-span's start from its own dy)
//     summary   Vspan  = sum_k exp(cl_k) V_k                      (the span's start gradient)
//     expand    out_k  = exp(tot - cl_k - ld_k) Gin + sum_{q>k} exp(cl_q - cl_k - ld_k) V_q
//                                                                 (gradient arriving at sub-span k's end)
//   summary also  Dspan = exp(tot).
//
// Every exponent is a sum of log decays over the sub-spans between two
// boundaries, so no term overflows and no quotient of decays appears; the
// folds run in float64 (a few values per (batch, head, channel)); the weights
// depend only on (batch, head, sub-spans), so each CTA computes them once in
// shared memory.  Summary: one CTA per (batch, head), threads over the channels;
// expansion: a thread per (sub-span, channel) output.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "ema_scan_dispatch.h"
#include "ema_ssd_b200.h"

namespace emab {
void set_last_error(const char* msg);

namespace spfold {

constexpr int kMaxSub = 64;
constexpr int kSumThreads = 128;
constexpr int kExpThreads = 256;  // expansion outputs (sub-span, channel) per CTA

struct Params {
  int B, K, H, P, dir;
  const double* ld;  // (B, K, H)
  const float* V;    // (B K, H, P)
  const float* bnd;  // (B, H, P)  expansion input
  float* out;        // summary: (B, H, P); expansion: (B K, H, P)
  float* dspan;      // (B, H) summary output, or null
};

// s_cl[k] = cl_k for k = 0..K (s_cl[K] = tot): the sub-spans' log decays are
// loaded in parallel, then summed in order by one thread (K <= 64 adds).
__device__ __forceinline__ void load_logs(const Params& p, int b, int h, double* s_ld, double* s_cl) {
  if (threadIdx.x < p.K) s_ld[threadIdx.x] = p.ld[(static_cast<size_t>(b) * p.K + threadIdx.x) * p.H + h];
  __syncthreads();
  if (threadIdx.x == 0) {
    double c = 0.0;
    for (int k = 0; k < p.K; ++k) {
      s_cl[k] = c;
      c += s_ld[k];
    }
    s_cl[p.K] = c;
  }
  __syncthreads();
}

// One CTA per (batch, head): the K weights once, then a K-term float64 dot per channel.
__global__ void __launch_bounds__(kSumThreads) summary_kernel(const Params p) {
  __shared__ double s_ld[kMaxSub], s_cl[kMaxSub + 1], s_w[kMaxSub];
  const int b = blockIdx.x / p.H, h = blockIdx.x % p.H;
  load_logs(p, b, h, s_ld, s_cl);
  const int K = p.K;
  if (threadIdx.x < K)
    s_w[threadIdx.x] = p.dir == 0 ? exp(s_cl[K] - s_cl[threadIdx.x + 1]) : exp(s_cl[threadIdx.x]);
  __syncthreads();
  const size_t kstride = static_cast<size_t>(p.H) * p.P;
  for (int c = threadIdx.x; c < p.P; c += blockDim.x) {
    const float* v = p.V + (static_cast<size_t>(b) * K * p.H + h) * p.P + c;
    double acc = 0.0;
#pragma unroll 8
    for (int k = 0; k < K; ++k) acc = fma(s_w[k], static_cast<double>(__ldg(v + k * kstride)), acc);
    p.out[(static_cast<size_t>(b) * p.H + h) * p.P + c] = static_cast<float>(acc);
  }
  if (threadIdx.x == 0 && p.dspan != nullptr) p.dspan[static_cast<size_t>(b) * p.H + h] = static_cast<float>(exp(s_cl[K]));
}

// grid (B H, ceil(K P / 256)): thread = one output (sub-span k, channel c).  The
// CTA's rows of pairwise weights (direction 0: W[k][q] = exp(cl_k - cl_{q+1}),
// q < k; direction 1: W[k][q] = exp(cl_q - cl_{k+1}), q > k -- exponents <= 0
// for decaying chains) and boundary weights are computed once in shared memory.
__global__ void __launch_bounds__(kExpThreads) expand_kernel(const Params p) {
  __shared__ double s_ld[kMaxSub], s_cl[kMaxSub + 1];
  __shared__ double s_W[kMaxSub * kMaxSub];
  __shared__ double s_bw[kMaxSub];
  const int b = blockIdx.x / p.H, h = blockIdx.x % p.H;
  load_logs(p, b, h, s_ld, s_cl);
  const int K = p.K, P = p.P;
  const int o0 = blockIdx.y * kExpThreads;
  const int k_lo = o0 / P, k_hi = min(K - 1, (o0 + kExpThreads - 1) / P);
  const int nr = k_hi - k_lo + 1;  // rows of weights this CTA's outputs use (<= K)
  for (int i = threadIdx.x; i < nr * K; i += blockDim.x) {
    const int k = k_lo + i / K, q = i % K;
    double w = 0.0;
    if (p.dir == 0 && q < k) w = exp(s_cl[k] - s_cl[q + 1]);
    if (p.dir == 1 && q > k) w = exp(s_cl[q] - s_cl[k + 1]);
    s_W[i] = w;
  }
  for (int r = threadIdx.x; r < nr; r += blockDim.x) {
    const int k = k_lo + r;
    s_bw[r] = p.dir == 0 ? exp(s_cl[k]) : exp(s_cl[K] - s_cl[k + 1]);
  }
  __syncthreads();
  const int o = o0 + threadIdx.x;
  if (o >= K * P) return;
  const int k = o / P, c = o % P, r = k - k_lo;
  const size_t kstride = static_cast<size_t>(p.H) * P;
  const float* v = p.V + (static_cast<size_t>(b) * K * p.H + h) * P + c;
  double acc = s_bw[r] * static_cast<double>(p.bnd[(static_cast<size_t>(b) * p.H + h) * P + c]);
  const double* w = s_W + r * K;
  const int q0 = p.dir == 0 ? 0 : k + 1, q1 = p.dir == 0 ? k : K;
#pragma unroll 4
  for (int q = q0; q < q1; ++q) acc = fma(w[q], static_cast<double>(__ldg(v + q * kstride)), acc);
  p.out[((static_cast<size_t>(b) * K + k) * p.H + h) * P + c] = static_cast<float>(acc);
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

int check(const EmaSpanFoldArgs* a, const char* what, bool expand) {
  if (a == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "%s: args is NULL", what);
  if (a->batch <= 0 || a->subspans <= 0 || a->nheads <= 0 || a->headdim <= 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "%s: bad shape", what);
  if (a->subspans > kMaxSub) return fail(EMA_ERR_UNSUPPORTED, "%s: at most %d sub-spans", what, kMaxSub);
  if (a->batch * a->nheads > 2147483647LL || a->subspans * a->headdim > 65535LL * kExpThreads)
    return fail(EMA_ERR_UNSUPPORTED, "%s: shape too large", what);
  if (a->direction != 0 && a->direction != 1) return fail(EMA_ERR_INVALID_ARGUMENT, "%s: direction 0 or 1", what);
  if (a->log_decay == nullptr || a->values == nullptr || a->out == nullptr ||
      (expand && a->boundary == nullptr))
    return fail(EMA_ERR_INVALID_ARGUMENT, "%s: log_decay, values, %sout are required", what,
                expand ? "boundary, " : "");
  return EMA_OK;
}

int launch(const EmaSpanFoldArgs* a, cudaStream_t s, bool expand) {
  const char* what = expand ? "ema_span_expand" : "ema_span_summary";
  int r = check(a, what, expand);
  if (r) return r;
  Params p{static_cast<int>(a->batch), static_cast<int>(a->subspans), static_cast<int>(a->nheads),
           static_cast<int>(a->headdim), a->direction, a->log_decay, a->values, a->boundary, a->out,
           expand ? nullptr : a->span_decay};
  const unsigned grid = static_cast<unsigned>(a->batch * a->nheads);
  if (expand) {
    const unsigned parts = static_cast<unsigned>((a->subspans * a->headdim + kExpThreads - 1) / kExpThreads);
    expand_kernel<<<dim3(grid, parts), kExpThreads, 0, s>>>(p);
  } else {
    summary_kernel<<<grid, kSumThreads, 0, s>>>(p);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return EMA_OK;
}

}  // namespace spfold
}  // namespace emab

extern "C" EMA_API int ema_span_summary(const EmaSpanFoldArgs* args, void* stream) {
  return emab::spfold::launch(args, static_cast<cudaStream_t>(stream), false);
}

extern "C" EMA_API int ema_span_expand(const EmaSpanFoldArgs* args, void* stream) {
  return emab::spfold::launch(args, static_cast<cudaStream_t>(stream), true);
}
