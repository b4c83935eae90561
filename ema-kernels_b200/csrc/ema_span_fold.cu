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
// folds run in float64 (a few values per (batch, head, channel)).  One CTA per
// (batch, head), threads over the channels.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "ema_scan_dispatch.h"
#include "ema_ssd_b200.h"

namespace emab {
void set_last_error(const char* msg);

namespace spfold {

constexpr int kMaxSub = 64;
constexpr int kThreads = 128;

struct Params {
  int B, K, H, P, dir;
  const double* ld;  // (B, K, H)
  const float* V;    // (B K, H, P)
  const float* bnd;  // (B, H, P)  expansion input
  float* out;        // summary: (B, H, P); expansion: (B K, H, P)
  float* dspan;      // (B, H) summary output, or null
};

__device__ __forceinline__ void load_logs(const Params& p, int b, int h, double* s_ld, double* s_cl,
                                          double* s_tot) {
  if (threadIdx.x == 0) {
    double c = 0.0;
    for (int k = 0; k < p.K; ++k) {
      const double l = p.ld[(static_cast<size_t>(b) * p.K + k) * p.H + h];
      s_ld[k] = l;
      s_cl[k] = c;
      c += l;
    }
    *s_tot = c;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads) summary_kernel(const Params p) {
  __shared__ double s_ld[kMaxSub], s_cl[kMaxSub], s_tot;
  const int b = blockIdx.x / p.H, h = blockIdx.x % p.H;
  load_logs(p, b, h, s_ld, s_cl, &s_tot);
  const double tot = s_tot;
  for (int c = threadIdx.x; c < p.P; c += blockDim.x) {
    double acc = 0.0;
    for (int k = 0; k < p.K; ++k) {
      const double w = p.dir == 0 ? exp(tot - s_cl[k] - s_ld[k]) : exp(s_cl[k]);
      acc += w * static_cast<double>(p.V[((static_cast<size_t>(b) * p.K + k) * p.H + h) * p.P + c]);
    }
    p.out[(static_cast<size_t>(b) * p.H + h) * p.P + c] = static_cast<float>(acc);
  }
  if (threadIdx.x == 0 && p.dspan != nullptr) p.dspan[static_cast<size_t>(b) * p.H + h] = static_cast<float>(exp(tot));
}

__global__ void __launch_bounds__(kThreads) expand_kernel(const Params p) {
  __shared__ double s_ld[kMaxSub], s_cl[kMaxSub], s_tot;
  const int b = blockIdx.x / p.H, h = blockIdx.x % p.H;
  load_logs(p, b, h, s_ld, s_cl, &s_tot);
  const double tot = s_tot;
  for (int c = threadIdx.x; c < p.P; c += blockDim.x) {
    const double bv = static_cast<double>(p.bnd[(static_cast<size_t>(b) * p.H + h) * p.P + c]);
    double v[kMaxSub];
#pragma unroll 1
    for (int k = 0; k < p.K; ++k)
      v[k] = static_cast<double>(p.V[((static_cast<size_t>(b) * p.K + k) * p.H + h) * p.P + c]);
#pragma unroll 1
    for (int k = 0; k < p.K; ++k) {
      double acc;
      if (p.dir == 0) {
        acc = exp(s_cl[k]) * bv;
        for (int q = 0; q < k; ++q) acc += exp(s_cl[k] - s_cl[q] - s_ld[q]) * v[q];
      } else {
        acc = exp(tot - s_cl[k] - s_ld[k]) * bv;
        for (int q = k + 1; q < p.K; ++q) acc += exp(s_cl[q] - s_cl[k] - s_ld[k]) * v[q];
      }
      p.out[((static_cast<size_t>(b) * p.K + k) * p.H + h) * p.P + c] = static_cast<float>(acc);
    }
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

int check(const EmaSpanFoldArgs* a, const char* what, bool expand) {
  if (a == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "%s: args is NULL", what);
  if (a->batch <= 0 || a->subspans <= 0 || a->nheads <= 0 || a->headdim <= 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "%s: bad shape", what);
  if (a->subspans > kMaxSub) return fail(EMA_ERR_UNSUPPORTED, "%s: at most %d sub-spans", what, kMaxSub);
  if (a->batch * a->nheads > 2147483647LL) return fail(EMA_ERR_UNSUPPORTED, "%s: shape too large", what);
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
  if (expand) expand_kernel<<<grid, kThreads, 0, s>>>(p);
  else summary_kernel<<<grid, kThreads, 0, s>>>(p);
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
