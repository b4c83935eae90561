// Device-side helpers shared by the EMA / SSD scan kernels (sm_100a).
//
//  * mbarrier + TMA (cp.async.bulk.tensor) wrappers, CTA-local forms only;
//  * acquire/release accessors for the inter-CTA look-back protocol;
//  * bounded waits: every spin gives up after a wall-clock limit, sets a bit
//    in the workspace status word and returns, so a lost producer can never
//    hang the GPU;
//  * float <-> element-type packs for bf16 / fp16 / fp32 tiles.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

namespace emab {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---- workspace header words (uint32 each) --------------------------------
constexpr int kHdrEpoch = 0;   // launch generation; tags look-back flags
constexpr int kHdrTicket = 1;  // dynamic tile counter (reset by the last CTA)
constexpr int kHdrDone = 2;    // finished-CTA counter (reset by the last CTA)
constexpr int kHdrStatus = 3;  // sticky error bits, read by the host
constexpr int kHdrWords = 64;  // header occupies 256 bytes

constexpr uint32_t kStatusLookbackTimeout = 1u;
constexpr uint32_t kStatusTmaTimeout = 2u;
constexpr uint32_t kStatusBadTicket = 4u;  // workspace counters were not reset (misuse)

constexpr uint32_t kFlagAgg = 1u;   // tile aggregate published
constexpr uint32_t kFlagIncl = 2u;  // inclusive prefix published
constexpr uint32_t kEpochMask = 0x3fffffffu;

// Wall-clock limit of every spin-wait (nanoseconds).
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch.  The scan kernels are launched with
// programmatic stream serialisation, so a kernel's CTAs may start while the
// previous kernel on the stream is still finishing.  grid_dep_wait() blocks
// until that kernel has completed and its writes are visible: nothing before
// it may read global memory that an earlier kernel writes (inputs, outputs,
// the shared look-back workspace).  grid_dep_release() lets the next kernel's
// CTAs be scheduled as SMs free up.  Both are no-ops for a plain launch.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Test a phase; a thread whose phase is not complete is suspended in hardware
// (issuing nothing) until it completes or about `hint_ns` pass.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase, uint32_t hint_ns = 1000000u) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait on an mbarrier phase; returns false (and sets the status bit)
// when the limit passes.  Between polls the thread sleeps with exponential
// backoff up to `max_sleep_ns`, so a waiting warp issues almost nothing.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase, uint32_t* status,
                                                  uint32_t max_sleep_ns = 256) {
  if (mbar_try_wait(bar, phase)) return true;
  const unsigned long long t0 = global_timer_ns();
  uint32_t sleep = 16;
  while (!mbar_try_wait(bar, phase)) {
    __nanosleep(sleep);
    sleep = sleep < max_sleep_ns ? sleep * 2 : max_sleep_ns;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      atomicOr(status, kStatusTmaTimeout);
      return false;
    }
  }
  return true;
}

// ---- TMA (tensor) copies; plain CTA-local forms only ---------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1,
                                             int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
      : "memory");
}
// L2 prefetch of a tensor-map box (no shared memory, no completion tracking).
__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
// L2 prefetch of a contiguous range: 16-byte aligned address, size a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Make generic-proxy shared-memory writes visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One bulk (non-tensor) copy global -> shared, completing on `bar` by bytes.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst_smem)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ---- cp.async (4-byte element gathers into shared memory) ----------------
__device__ __forceinline__ void cp_async_4(void* dst_smem, const void* src_gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst_smem)), "l"(src_gmem)
               : "memory");
}
// Arrive on `bar` once all prior cp.async of this thread have landed; counts
// against the barrier's expected arrivals (.noinc).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Barrier over the first `nthreads` threads (the consumer warps) only.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- acquire / release ----------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float ld_relaxed_gpu(const float* p) {
  float v;
  asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}
// Self-validating look-back words: {float value, uint32 tag} in one 64-bit
// single-copy-atomic access, so a reader that sees the tag sees the value.
__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t tag_word(float v, uint32_t tag) {
  return (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ uint32_t word_tag(uint64_t w) { return static_cast<uint32_t>(w >> 32); }
__device__ __forceinline__ float word_val(uint64_t w) { return __uint_as_float(static_cast<uint32_t>(w)); }

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

// ---- the SSD's dt map ---------------------------------------------------------
// dt <- clamp(softplus(dt + bias[h]), lo, hi), each step optional (Mamba-2's
// dt_bias / dt_softplus / dt_limit).  softplus(v) = log1p(exp(v)), v itself
// above 20 (torch's default threshold).  *deriv (if given) receives d dt / d
// (dt given): sigmoid(v) for the softplus, times 0 where the clamp is active.
struct DtMap {
  const float* bias;  // (H,) or null
  int softplus;
  int clamp;
  float lo, hi;
};
__device__ __forceinline__ bool dt_map_active(const DtMap& m) {
  return m.bias != nullptr || m.softplus != 0 || m.clamp != 0;
}
__device__ __forceinline__ float dt_map(const DtMap& m, int h, float raw, float* deriv) {
  float v = (m.bias != nullptr) ? raw + m.bias[h] : raw;
  float d = 1.f;
  if (m.softplus) {
    if (v <= 20.f) {
      d = 1.f / (1.f + expf(-v));
      v = log1pf(expf(v));
    }
  }
  if (m.clamp) {
    if (v < m.lo || v > m.hi) d = 0.f;
    v = fminf(fmaxf(v, m.lo), m.hi);
  }
  if (deriv != nullptr) *deriv = d;
  return v;
}
// The map an SsdFwdArgs / SsdBwdArgs asks for.
template <class Args>
inline DtMap dt_map_of(const Args* a) {
  return DtMap{a->dt_bias, a->dt_softplus, a->dt_clamp, a->dt_min, a->dt_max};
}

// ---- element packs --------------------------------------------------------
template <int BYTES>
struct RawVec;
template <>
struct RawVec<2> { using type = uint16_t; };
template <>
struct RawVec<4> { using type = uint32_t; };
template <>
struct RawVec<8> { using type = uint2; };
template <>
struct RawVec<16> { using type = uint4; };
template <>
struct RawVec<32> { struct type { uint4 a, b; }; };

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Load N consecutive elements (N * sizeof(T) bytes, naturally aligned) as floats.
template <typename T, int N>
__device__ __forceinline__ void load_pack(const T* p, float (&f)[N]) {
  using R = typename RawVec<sizeof(T) * N>::type;
  R r = *reinterpret_cast<const R*>(p);
  const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
  for (int k = 0; k < N; ++k) f[k] = to_f32(e[k]);
}
// Store N elements to global memory with the evict-first ("streaming") policy:
// outputs are written once and not re-read by this path.  The __stcs
// intrinsics (not inline asm) leave address arithmetic to the compiler.
__device__ __forceinline__ void st_cs(uint16_t* p, uint16_t v) { __stcs(reinterpret_cast<unsigned short*>(p), v); }
__device__ __forceinline__ void st_cs(uint32_t* p, uint32_t v) { __stcs(reinterpret_cast<unsigned int*>(p), v); }
__device__ __forceinline__ void st_cs(uint2* p, uint2 v) { __stcs(p, v); }
__device__ __forceinline__ void st_cs(uint4* p, uint4 v) { __stcs(p, v); }
template <typename T, int N>
__device__ __forceinline__ void store_pack_global_cs(T* p, const float (&f)[N]) {
  using R = typename RawVec<sizeof(T) * N>::type;
  R r;
  T* e = reinterpret_cast<T*>(&r);
#pragma unroll
  for (int k = 0; k < N; ++k) e[k] = from_f32<T>(f[k]);
  st_cs(reinterpret_cast<R*>(p), r);
}

// ---- packed fp32x2 (sm_100 FFMA2 / FMUL2 / FADD2) -------------------------
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 f2_bcast(float a) { return make_float2(a, a); }

// 2*NP consecutive elements as NP float pairs.
template <typename T, int NP>
__device__ __forceinline__ void load_pairs(const T* p, float2 (&v)[NP]) {
  float f[2 * NP];
  load_pack<T, 2 * NP>(p, f);
#pragma unroll
  for (int k = 0; k < NP; ++k) v[k] = make_float2(f[2 * k], f[2 * k + 1]);
}
template <typename T, int NP>
__device__ __forceinline__ void store_pairs_global_cs(T* p, const float2 (&v)[NP]) {
  float f[2 * NP];
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    f[2 * k] = v[k].x;
    f[2 * k + 1] = v[k].y;
  }
  store_pack_global_cs<T, 2 * NP>(p, f);
}

// ---- groups of 8 channels as 4 float pairs ----------------------------------
// One lane's channel group: 16 bytes of bf16 / f16, 32 bytes of f32.
struct U32x8 {
  uint4 a, b;
};
template <typename T>
__device__ __forceinline__ float2 cvt_pair(uint32_t w);
template <>
__device__ __forceinline__ float2 cvt_pair<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 cvt_pair<__half>(uint32_t w) {
  __half2 h;
  memcpy(&h, &w, 4);
  return __half22float2(h);
}
template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float2 v);
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float2 v) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
  uint32_t w;
  memcpy(&w, &h, 4);
  return w;
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(float2 v) {
  const __half2 h = __floats2half2_rn(v.x, v.y);
  uint32_t w;
  memcpy(&w, &h, 4);
  return w;
}
// 8 consecutive elements (16-byte aligned for 2-byte types, 32-byte for f32).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float2 (&v)[4]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    v[0] = make_float2(a.x, a.y);
    v[1] = make_float2(a.z, a.w);
    v[2] = make_float2(b.x, b.y);
    v[3] = make_float2(b.z, b.w);
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    v[0] = cvt_pair<T>(u.x);
    v[1] = cvt_pair<T>(u.y);
    v[2] = cvt_pair<T>(u.z);
    v[3] = cvt_pair<T>(u.w);
  }
}
// Streaming store of the first `n` (8, or 4 for f32) of 8 elements.
template <typename T>
__device__ __forceinline__ void store8_cs(T* p, const float2 (&v)[4], int n) {
  if constexpr (sizeof(T) == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0].x, v[0].y, v[1].x, v[1].y));
    if (n > 4) __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(v[2].x, v[2].y, v[3].x, v[3].y));
  } else {
    __stcs(reinterpret_cast<uint4*>(p),
           make_uint4(pack_pair<T>(v[0]), pack_pair<T>(v[1]), pack_pair<T>(v[2]), pack_pair<T>(v[3])));
  }
}

// NPR float pairs of consecutive elements (NPR = 2 or 4).
template <typename T, int NPR>
__device__ __forceinline__ void load_grp(const T* p, float2 (&v)[NPR]) {
  if constexpr (NPR == 4) {
    load8<T>(p, v);
  } else if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = make_float2(a.x, a.y);
    v[1] = make_float2(a.z, a.w);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    v[0] = cvt_pair<T>(u.x);
    v[1] = cvt_pair<T>(u.y);
  }
}
// Streaming store of the first `n` of 2 * NPR elements (n is 2 * NPR, or 4
// for an f32 group of 8 straddling the channel count).
template <typename T, int NPR>
__device__ __forceinline__ void store_grp_cs(T* p, const float2 (&v)[NPR], int n) {
  if constexpr (NPR == 4) {
    store8_cs<T>(p, v, n);
  } else if constexpr (sizeof(T) == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0].x, v[0].y, v[1].x, v[1].y));
  } else {
    __stcs(reinterpret_cast<uint2*>(p), make_uint2(pack_pair<T>(v[0]), pack_pair<T>(v[1])));
  }
}

// Plain (shared-memory) store of 2 * NPR elements as T.
template <typename T, int NPR>
__device__ __forceinline__ void store_grp(T* p, const float2 (&v)[NPR]) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int q = 0; q < NPR; q += 2)
      reinterpret_cast<float4*>(p)[q / 2] = make_float4(v[q].x, v[q].y, v[q + 1].x, v[q + 1].y);
  } else if constexpr (NPR == 2) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_pair<T>(v[0]), pack_pair<T>(v[1]));
  } else {
    *reinterpret_cast<uint4*>(p) =
        make_uint4(pack_pair<T>(v[0]), pack_pair<T>(v[1]), pack_pair<T>(v[2]), pack_pair<T>(v[3]));
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_pack(T* p, const float (&f)[N]) {
  using R = typename RawVec<sizeof(T) * N>::type;
  R r;
  T* e = reinterpret_cast<T*>(&r);
#pragma unroll
  for (int k = 0; k < N; ++k) e[k] = from_f32<T>(f[k]);
  *reinterpret_cast<R*>(p) = r;
}

}  // namespace emab
