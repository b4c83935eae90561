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
// the sum over tokens is a reduction.  One CTA per (row, head) walks its row in
// 256-token blocks: a block scan of dt A, then warp c accumulates channels
// [8 c, 8 c + 8) (one 16-byte vector per token) over the block's tokens, one
// token per lane, and reduces over the lanes with shuffles; blocks combine
// through the block decay (direction 0: S <- exp(ld_block) S + block sum;
// direction 1: G <- G + exp(cs before the block) block sum).  fp32 arithmetic,
// as the scan kernels.  HBM-bound: x (or dy) is read once, 8 KB per CTA in
// flight per 256 threads.
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

constexpr int kBlock = 256;  // tokens per block (one per thread in the scan)

struct Params {
  int L, H;
  const void* x;
  long long sr, sl, sh;  // element strides of row, token, head
  const float* dt;       // (rows, L, H)
  const float* A;
  float* out;            // (rows, H, P)
  int dir;
};

template <typename T, int P>
__global__ void __launch_bounds__(32 * (P / 8)) span_state_kernel(const Params p) {
  constexpr int NW = P / 8;  // warps: one per 8-channel group
  constexpr int NT = 32 * NW;
  __shared__ float s_w[kBlock];   // the block's per-token weights
  __shared__ float s_wsum[32];    // per-warp scan totals
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = blockIdx.x / p.H, h = blockIdx.x % p.H;
  const float Ah = p.A[h];
  const T* xbase = static_cast<const T*>(p.x) + row * p.sr + h * p.sh + 8 * warp;
  const float* dtbase = p.dt + static_cast<size_t>(row) * p.L * p.H + h;
  float acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.f;
  float before = 0.f;  // direction 1: the cumsum of dt A before the block
  for (int t0 = 0; t0 < p.L; t0 += kBlock) {
    const int n = min(kBlock, p.L - t0);
    // ---- block scan of dt A (kBlock tokens over NT threads, kBlock / NT per thread) ----
    constexpr int TPT = (kBlock + NT - 1) / NT;
    float d[TPT], v[TPT];
    float run = 0.f;
#pragma unroll
    for (int k = 0; k < TPT; ++k) {
      const int t = tid * TPT + k;
      d[k] = (t < n) ? dtbase[static_cast<size_t>(t0 + t) * p.H] : 0.f;
      run += d[k] * Ah;
      v[k] = run;  // inclusive within this thread's tokens
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
    for (int w = 0; w < NW; ++w) {
      const float sw = s_wsum[w];
      if (w < warp) wpre += sw;
      total += sw;
    }
    const float excl = wpre + incl - run;  // cumsum before this thread's first token
#pragma unroll
    for (int k = 0; k < TPT; ++k) {
      const int t = tid * TPT + k;
      if (t < kBlock) {
        const float cs = excl + v[k];  // within the block, through token t
        s_w[t] = (t >= n) ? 0.f : (p.dir == 0 ? __expf(total - cs) * d[k] : __expf(before + cs));
      }
    }
    __syncthreads();
    // ---- weighted column sums: warp = 8-channel group, lane = token ----------------
    float bs[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) bs[k] = 0.f;
#pragma unroll 4
    for (int t = lane; t < n; t += 32) {
      float xv[8];
      load_pack<T, 8>(xbase + static_cast<long long>(t0 + t) * p.sl, xv);
      const float w = s_w[t];
#pragma unroll
      for (int k = 0; k < 8; ++k) bs[k] = fmaf(w, xv[k], bs[k]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) bs[k] += __shfl_xor_sync(0xffffffffu, bs[k], o);
    }
    if (p.dir == 0) {
      const float dec = __expf(total);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = fmaf(dec, acc[k], bs[k]);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += bs[k];
      before += total;
    }
    __syncthreads();  // s_w / s_wsum are rewritten by the next block
  }
  if (lane == 0) {
    float* o = p.out + (static_cast<size_t>(row) * p.H + h) * P + 8 * warp;
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = acc[k];
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
  span_state_kernel<T, P><<<static_cast<unsigned>(rows * p.H), 32 * (P / 8), 0, s>>>(p);
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
    const size_t bytes = static_cast<size_t>(a->rows) * a->nheads * a->headdim * sizeof(float);
    const cudaError_t e = bytes ? cudaMemsetAsync(a->out, 0, bytes, static_cast<cudaStream_t>(stream)) : cudaSuccess;
    return e == cudaSuccess ? EMA_OK : fail(EMA_ERR_CUDA, "ema_span_state: %s", cudaGetErrorString(e));
  }
  Params p{static_cast<int>(a->seqlen), static_cast<int>(a->nheads), a->x, a->x_stride[0], a->x_stride[1],
           a->x_stride[2], a->dt, a->A, a->out, a->direction};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int P = static_cast<int>(a->headdim);
  switch (a->dtype) {
    case EMA_DTYPE_F32: return launch_p<float>(p, a->rows, P, s);
    case EMA_DTYPE_BF16: return launch_p<__nv_bfloat16>(p, a->rows, P, s);
    default: return launch_p<__half>(p, a->rows, P, s);
  }
}
