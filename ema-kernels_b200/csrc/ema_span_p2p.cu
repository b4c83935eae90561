// Span exchange of the sequence-parallel EMA (kernels/ema_sp.py) over NVLink
// peer memory: one kernel per direction does what the summary fold, the NCCL
// exchange and the expansion fold do otherwise.
//
// Every rank owns one exchange buffer (ema_p2p_alloc, once per process group
// and shape) and maps every peer's buffer through CUDA IPC (ema_p2p_handle on
// the owner, ema_p2p_open on the others).  A launch runs one CTA per (batch,
// head), a thread per channel, all arithmetic in float64:
//   1. the span summary from the rank's K sub-spans, with e_k = exp(ld_k) the
//      decay of sub-span k:
//        forward   S = (s <- e_k s + V_k for k = 0 .. K-1, from s = 0)
//        backward  G = (g <- e_k g + V_k for k = K-1 .. 0, from g = 0)
//        D = exp(sum_k ld_k); rank 0 (forward) / the last rank (backward)
//        folds in the sequence's boundary value: S <- D b + S;
//   2. (S, D) into slot [parity][rank] of every rank's buffer (plain stores
//      over NVLink), a system-scope fence, then this CTA's flag word for this
//      rank in every rank's buffer set to the launch's tag (a release store);
//   3. waits until every rank's flag for this CTA has reached the tag
//      (acquire loads of its own buffer, bounded: after 1 s it sets a status
//      bit and goes on, so a missing rank ends in an error, not a hang);
//   4. folds the summaries of the spans before it (forward, s <- D_q s + S_q
//      in rank order from 0 or, on rank 0, the initial state) or after it
//      (backward, from the last rank down), the value at the span's boundary;
//   5. expands it into every sub-span's boundary value (the same recurrence
//      over the sub-spans, seeded with that value).
// Every factor is a decay e <= 1, so nothing overflows and no quotient of
// decays appears.  The tag is the buffer's launch counter (advanced by the
// launch's last CTA); slots alternate by its parity.  Every rank waits for
// every rank, so a rank that reaches launch e + 1 has seen all ranks start
// launch e, i.e. finish launch e - 1 and its reads of the slots launch e + 1
// rewrites.  Flags compare as "reached" (later tags count), so a fast peer's
// next tag does not strand a slow reader.  Calls are collective: every rank
// of the group calls with the same shapes, in the same order.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "ema_common.cuh"
#include "ema_scan_dispatch.h"
#include "ema_ssd_b200.h"

namespace emab {
void set_last_error(const char* msg);

namespace spx {

constexpr int kMaxSub = 64;
constexpr int kMaxRanks = EMA_SPAN_EXCHANGE_MAX_RANKS;
constexpr int kThreads = 128;  // one channel per thread: headdim <= 128
constexpr uint32_t kStatusExchangeTimeout = 1u;

// Buffer layout (bytes): header (epoch, done count, status; 256 bytes), then
// flags [kMaxRanks][bh] uint32, then slots [2][world][bh][P + 1] float.
constexpr size_t kHeaderBytes = 256;
__host__ __device__ inline size_t flags_bytes(long long bh) {
  return ((static_cast<size_t>(kMaxRanks) * bh * sizeof(uint32_t)) + 255) & ~static_cast<size_t>(255);
}
__host__ __device__ inline size_t slot_floats(long long P) { return static_cast<size_t>(P) + 1; }
__host__ inline size_t buffer_bytes(long long world, long long bh, long long P) {
  return kHeaderBytes + flags_bytes(bh) + 2 * static_cast<size_t>(world) * bh * slot_floats(P) * sizeof(float);
}

struct Params {
  int B, K, H, P, dir, rank, world;
  const double* ld;   // (B, K, H)
  const float* V;     // (B K, H, P)
  const float* bnd;   // (B, H, P) or null
  float* span_in;     // (B, H, P)
  float* out;         // (B K, H, P)
  unsigned char* buf[kMaxRanks];
};

__device__ __forceinline__ uint32_t* flag_ptr(unsigned char* buf, int src, int cta, int bh) {
  return reinterpret_cast<uint32_t*>(buf + kHeaderBytes) + static_cast<size_t>(src) * bh + cta;
}
__device__ __forceinline__ float* slot_ptr(unsigned char* buf, int par, int src, int cta, int bh, int world, int P) {
  float* slots = reinterpret_cast<float*>(buf + kHeaderBytes + flags_bytes(bh));
  return slots + ((static_cast<size_t>(par) * world + src) * bh + cta) * slot_floats(P);
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ld_relaxed_sys(const float* p) {
  float v;
  asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) exchange_kernel(const Params p) {
  __shared__ double s_e[kMaxSub];  // exp(ld_k)
  __shared__ double s_ld[kMaxSub];
  __shared__ double s_D;
  __shared__ uint32_t s_tag;
  const int cta = blockIdx.x, bh = gridDim.x, tid = threadIdx.x;
  const int b = cta / p.H, h = cta % p.H, K = p.K, P = p.P;
  unsigned char* own = p.buf[p.rank];
  uint32_t* hdr = reinterpret_cast<uint32_t*>(own);
  if (tid == 0) s_tag = ld_volatile_u32(&hdr[0]) + 1u;
  if (tid < K) {
    const double l = p.ld[(static_cast<size_t>(b) * K + tid) * p.H + h];
    s_ld[tid] = l;
    s_e[tid] = exp(l);
  }
  __syncthreads();
  if (tid == 0) {
    double t = 0.0;
    for (int k = 0; k < K; ++k) t += s_ld[k];
    s_D = exp(t);
  }
  __syncthreads();
  const uint32_t tag = s_tag;
  const int par = static_cast<int>(tag & 1u);
  const bool ch = tid < P;
  const int c = ch ? tid : 0;
  const size_t kstride = static_cast<size_t>(p.H) * P;
  const float* v = p.V + (static_cast<size_t>(b) * K * p.H + h) * P + c;  // sub-span k at v[k * kstride]
  const double D = s_D;
  // 1. the span summary
  double s = 0.0;
  if (p.dir == 0) {
#pragma unroll 4
    for (int k = 0; k < K; ++k) s = fma(s_e[k], s, static_cast<double>(__ldg(v + k * kstride)));
  } else {
#pragma unroll 4
    for (int k = K - 1; k >= 0; --k) s = fma(s_e[k], s, static_cast<double>(__ldg(v + k * kstride)));
  }
  const bool edge = p.dir == 0 ? p.rank == 0 : p.rank == p.world - 1;
  const double bv = (edge && p.bnd != nullptr && ch)
                        ? static_cast<double>(p.bnd[(static_cast<size_t>(b) * p.H + h) * P + c])
                        : 0.0;
  if (edge) s = fma(D, bv, s);
  // 2. into slot [par][rank] of every rank's buffer, then the flags
  for (int q = 0; q < p.world; ++q) {
    float* slot = slot_ptr(p.buf[q], par, p.rank, cta, bh, p.world, P);
    if (ch) slot[c] = static_cast<float>(s);
    if (tid == 0) slot[P] = static_cast<float>(D);
  }
  __threadfence_system();
  __syncthreads();
  if (tid < p.world) st_release_sys(flag_ptr(p.buf[tid], p.rank, cta, bh), tag);
  // 3. every rank's flag for this CTA (bounded)
  if (tid < p.world) {
    const uint32_t* f = flag_ptr(own, tid, cta, bh);
    if (static_cast<int>(ld_acquire_sys(f) - tag) < 0) {
      const unsigned long long t0 = global_timer_ns();
      uint32_t sleep = 32;
      while (static_cast<int>(ld_acquire_sys(f) - tag) < 0) {
        __nanosleep(sleep);
        sleep = sleep < 256 ? sleep * 2 : 256;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          atomicOr(&hdr[2], kStatusExchangeTimeout);
          break;
        }
      }
    }
  }
  __syncthreads();
  // 4. the value at this span's boundary
  double in = edge ? bv : 0.0;
  if (!edge) {
    if (p.dir == 0) {
      for (int q = 0; q < p.rank; ++q) {
        const float* slot = slot_ptr(own, par, q, cta, bh, p.world, P);
        in = fma(static_cast<double>(ld_relaxed_sys(slot + P)), in, static_cast<double>(ld_relaxed_sys(slot + c)));
      }
    } else {
      for (int q = p.world - 1; q > p.rank; --q) {
        const float* slot = slot_ptr(own, par, q, cta, bh, p.world, P);
        in = fma(static_cast<double>(ld_relaxed_sys(slot + P)), in, static_cast<double>(ld_relaxed_sys(slot + c)));
      }
    }
  }
  // 5. every sub-span's boundary value
  if (ch) {
    p.span_in[(static_cast<size_t>(b) * p.H + h) * P + c] = static_cast<float>(in);
    float* o = p.out + (static_cast<size_t>(b) * K * p.H + h) * P + c;
    double r = in;
    if (p.dir == 0) {  // the state entering sub-span k
      for (int k = 0; k < K; ++k) {
        o[k * kstride] = static_cast<float>(r);
        r = fma(s_e[k], r, static_cast<double>(__ldg(v + k * kstride)));
      }
    } else {  // the gradient arriving at sub-span k's end
      for (int k = K - 1; k >= 0; --k) {
        o[k * kstride] = static_cast<float>(r);
        r = fma(s_e[k], r, static_cast<double>(__ldg(v + k * kstride)));
      }
    }
  }
  // the launch's last CTA advances the tag
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&hdr[1], 1u) == gridDim.x - 1) {
      hdr[1] = 0u;
      __threadfence();
      hdr[0] = tag;
    }
  }
}

int fail(int code, const char* fmt, ...) {
  char msg[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  set_last_error(msg);
  return code;
}

}  // namespace spx
}  // namespace emab

using namespace emab::spx;

extern "C" EMA_API size_t ema_span_exchange_bytes(int64_t world, int64_t batch_heads, int64_t headdim) {
  if (world <= 0 || world > kMaxRanks || batch_heads <= 0 || headdim <= 0) return 0;
  return buffer_bytes(world, batch_heads, headdim);
}

extern "C" EMA_API int ema_p2p_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return fail(EMA_ERR_INVALID_ARGUMENT, "ema_p2p_alloc: bad arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ema_p2p_alloc: %s", cudaGetErrorString(e));
  return EMA_OK;
}

extern "C" EMA_API int ema_p2p_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? EMA_OK : fail(EMA_ERR_CUDA, "ema_p2p_free: %s", cudaGetErrorString(e));
}

extern "C" EMA_API int ema_p2p_handle(void* ptr, unsigned char* handle) {
  if (ptr == nullptr || handle == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "ema_p2p_handle: bad arguments");
  cudaIpcMemHandle_t hd;
  const cudaError_t e = cudaIpcGetMemHandle(&hd, ptr);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ema_p2p_handle: %s", cudaGetErrorString(e));
  static_assert(sizeof(hd) == EMA_P2P_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &hd, sizeof(hd));
  return EMA_OK;
}

extern "C" EMA_API int ema_p2p_open(const unsigned char* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "ema_p2p_open: bad arguments");
  cudaIpcMemHandle_t hd;
  std::memcpy(&hd, handle, sizeof(hd));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, hd, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ema_p2p_open: %s", cudaGetErrorString(e));
  return EMA_OK;
}

extern "C" EMA_API int ema_p2p_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? EMA_OK : fail(EMA_ERR_CUDA, "ema_p2p_close: %s", cudaGetErrorString(e));
}

extern "C" EMA_API int ema_span_exchange_status(void* own_buffer, uint32_t* status, int32_t clear) {
  if (own_buffer == nullptr || status == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_exchange_status: bad arguments");
  uint32_t* word = reinterpret_cast<uint32_t*>(own_buffer) + 2;
  cudaError_t e = cudaMemcpy(status, word, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear) e = cudaMemset(word, 0, sizeof(uint32_t));
  return e == cudaSuccess ? EMA_OK : fail(EMA_ERR_CUDA, "ema_span_exchange_status: %s", cudaGetErrorString(e));
}

extern "C" EMA_API int ema_span_exchange(const EmaSpanExchangeArgs* a, void* stream) {
  if (a == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_exchange: args is NULL");
  if (a->batch <= 0 || a->subspans <= 0 || a->nheads <= 0 || a->headdim <= 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_exchange: bad shape");
  if (a->subspans > kMaxSub) return fail(EMA_ERR_UNSUPPORTED, "ema_span_exchange: at most %d sub-spans", kMaxSub);
  if (a->headdim > kThreads) return fail(EMA_ERR_UNSUPPORTED, "ema_span_exchange: headdim <= %d", kThreads);
  if (a->world < 1 || a->world > kMaxRanks || a->rank < 0 || a->rank >= a->world)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_exchange: rank %d of %d (at most %d ranks)", a->rank, a->world,
                kMaxRanks);
  if (a->direction != 0 && a->direction != 1)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_exchange: direction 0 or 1");
  if (a->log_decay == nullptr || a->values == nullptr || a->span_in == nullptr || a->out == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_exchange: log_decay, values, span_in and out are required");
  const long long bh = a->batch * a->nheads;
  if (bh > 2147483647LL) return fail(EMA_ERR_UNSUPPORTED, "ema_span_exchange: shape too large");
  const size_t need = buffer_bytes(a->world, bh, a->headdim);
  if (a->buffer_bytes < need)
    return fail(EMA_ERR_WORKSPACE, "ema_span_exchange: buffers hold %zu bytes, the shape needs %zu",
                static_cast<size_t>(a->buffer_bytes), need);
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, exchange_kernel, kThreads, 0);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ema_span_exchange: %s", cudaGetErrorString(e));
  // CTA i waits for CTA i of every other rank: all CTAs must be resident at once
  if (bh > static_cast<long long>(sms) * per_sm)
    return fail(EMA_ERR_UNSUPPORTED, "ema_span_exchange: %lld CTAs (batch x heads) exceed the %d the GPU holds at once",
                bh, sms * per_sm);
  Params p{static_cast<int>(a->batch), static_cast<int>(a->subspans), static_cast<int>(a->nheads),
           static_cast<int>(a->headdim), a->direction, a->rank, a->world, a->log_decay, a->values,
           a->boundary, a->span_in, a->out, {}};
  for (int q = 0; q < kMaxRanks; ++q) {
    if (q < a->world && a->buffers[q] == nullptr)
      return fail(EMA_ERR_INVALID_ARGUMENT, "ema_span_exchange: buffer of rank %d is NULL", q);
    p.buf[q] = static_cast<unsigned char*>(q < a->world ? a->buffers[q] : nullptr);
  }
  exchange_kernel<<<static_cast<unsigned>(bh), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ema_span_exchange launch failed: %s", cudaGetErrorString(e));
  return EMA_OK;
}
