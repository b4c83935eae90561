// The output gate of a Mamba-2 SSD layer call, out = y * silu(z)
// (mamba_chunk_scan_combined's `z` argument), and its gradient, each as one
// pass over (batch, seqlen, nheads, headdim) in HBM.
//
//   forward:   out = y * z * sigmoid(z)
//   backward:  dy  = dout * z * sigmoid(z)
//              dz  = dout * y * sigmoid(z) * (1 + z * (1 - sigmoid(z)))
//
// fp32 arithmetic on y, z, dout of one element type (bf16 / fp16 / fp32),
// results rounded once to that type.  Memory-bound: each thread moves groups
// of 8 consecutive channels (16-byte vectors for 2-byte types) where the
// headdim, strides and pointers allow it, single elements otherwise; the
// grid is a multiple of the SM count with a grid-stride loop.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "ema_common.cuh"
#include "ema_scan_dispatch.h"
#include "ssd_b200.h"

namespace emab {
void set_last_error(const char* msg);

namespace ssdgate {

struct View {
  long long sb, sl, sh;  // element strides of batch, token, head (channel stride 1)
};

struct Params {
  long long rows;  // batch * seqlen * nheads
  int L, H, P;
  const void* y;
  View vy;
  const void* z;
  View vz;
  const void* dout;
  View vd;
  void* out;  // forward: out; backward: dy
  View vo;
  void* dz;   // backward only
  View vdz;
};

__device__ __forceinline__ float sigmoidf(float v) { return 1.f / (1.f + expf(-v)); }

template <class T, int V>
__device__ __forceinline__ void load_vec(const T* p, float (&f)[V]) {
  load_pack<T, V>(p, f);
}
// V elements; 32-byte groups (8 fp32) as two 16-byte stores
template <class T, int V>
__device__ __forceinline__ void store_vec(T* p, const float (&f)[V]) {
  if constexpr (sizeof(T) * V == 32) {
    float a[V / 2], b[V / 2];
#pragma unroll
    for (int k = 0; k < V / 2; ++k) {
      a[k] = f[k];
      b[k] = f[V / 2 + k];
    }
    store_pack_global_cs<T, V / 2>(p, a);
    store_pack_global_cs<T, V / 2>(p + V / 2, b);
  } else {
    store_pack_global_cs<T, V>(p, f);
  }
}

template <class T, int V, bool BWD>
__global__ void __launch_bounds__(256) gate_kernel(const Params p) {
  const int vpr = p.P / V;  // vectors per row
  const long long nvec = p.rows * vpr;
  const long long lh = static_cast<long long>(p.L) * p.H;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < nvec;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / vpr;
    const int c = static_cast<int>(i - row * vpr) * V;
    const long long b = row / lh, r2 = row - b * lh;
    const long long l = r2 / p.H, h = r2 - l * p.H;
    auto at = [&](const View& v) { return b * v.sb + l * v.sl + h * v.sh + c; };
    float yv[V], zv[V], dv[V];
    load_vec<T, V>(static_cast<const T*>(p.y) + at(p.vy), yv);
    load_vec<T, V>(static_cast<const T*>(p.z) + at(p.vz), zv);
    if (BWD) load_vec<T, V>(static_cast<const T*>(p.dout) + at(p.vd), dv);
    float o[V], g[V];
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float s = sigmoidf(zv[k]);
      const float silu = zv[k] * s;
      if (BWD) {
        o[k] = dv[k] * silu;
        g[k] = dv[k] * yv[k] * s * (1.f + zv[k] * (1.f - s));
      } else {
        o[k] = yv[k] * silu;
      }
    }
    store_vec<T, V>(static_cast<T*>(p.out) + at(p.vo), o);
    if (BWD) store_vec<T, V>(static_cast<T*>(p.dz) + at(p.vdz), g);
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

View view(const int64_t (&s)[3]) { return View{s[0], s[1], s[2]}; }

bool vec_ok(const void* ptr, const int64_t (&s)[3], int esize) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16u != 0u) return false;
  for (int i = 0; i < 3; ++i)
    if ((s[i] * esize) % 16 != 0) return false;
  return true;
}

template <class T, bool BWD>
int launch_t(const Params& p, bool vec, cudaStream_t stream) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int V = vec ? 8 : 1;
  const long long nvec = p.rows * (p.P / V);
  long long blocks = (nvec + 255) / 256;
  const long long cap = static_cast<long long>(sms) * 8;  // 8 resident blocks of 256 threads per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (vec) gate_kernel<T, 8, BWD><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
  else gate_kernel<T, 1, BWD><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ssd_gate launch failed: %s", cudaGetErrorString(e));
  return EMA_OK;
}

template <bool BWD>
int launch(const SsdGateArgs* a, cudaStream_t stream) {
  const char* what = BWD ? "ssd_gate_bwd" : "ssd_gate_fwd";
  if (a == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "%s: args is NULL", what);
  if (a->batch < 0 || a->seqlen < 0 || a->nheads <= 0 || a->headdim <= 0)
    return fail(EMA_ERR_INVALID_ARGUMENT, "%s: bad shape", what);
  if (a->seqlen > 2147483647 || a->nheads > 2147483647 || a->headdim > 2147483647)
    return fail(EMA_ERR_UNSUPPORTED, "%s: shape too large", what);
  const int esize = a->dtype == EMA_DTYPE_F32 ? 4 : 2;
  if (a->dtype != EMA_DTYPE_F32 && a->dtype != EMA_DTYPE_BF16 && a->dtype != EMA_DTYPE_F16)
    return fail(EMA_ERR_INVALID_ARGUMENT, "%s: unknown dtype %d", what, a->dtype);
  if (a->y == nullptr || a->z == nullptr || a->out == nullptr || (BWD && (a->dout == nullptr || a->dz == nullptr)))
    return fail(EMA_ERR_INVALID_ARGUMENT, "%s: y, z and %s are required", what, BWD ? "dout, dy, dz" : "out");
  if (a->batch == 0 || a->seqlen == 0) return EMA_OK;
  Params p{};
  p.rows = a->batch * a->seqlen * a->nheads;
  p.L = static_cast<int>(a->seqlen);
  p.H = static_cast<int>(a->nheads);
  p.P = static_cast<int>(a->headdim);
  p.y = a->y;
  p.vy = view(a->y_stride);
  p.z = a->z;
  p.vz = view(a->z_stride);
  p.out = a->out;
  p.vo = view(a->out_stride);
  bool vec = (a->headdim % 8 == 0) && vec_ok(a->y, a->y_stride, esize) && vec_ok(a->z, a->z_stride, esize) &&
             vec_ok(a->out, a->out_stride, esize);
  if (BWD) {
    p.dout = a->dout;
    p.vd = view(a->dout_stride);
    p.dz = a->dz;
    p.vdz = view(a->dz_stride);
    vec = vec && vec_ok(a->dout, a->dout_stride, esize) && vec_ok(a->dz, a->dz_stride, esize);
  }
  switch (a->dtype) {
    case EMA_DTYPE_F32: return launch_t<float, BWD>(p, vec, stream);
    case EMA_DTYPE_BF16: return launch_t<__nv_bfloat16, BWD>(p, vec, stream);
    default: return launch_t<__half, BWD>(p, vec, stream);
  }
}

}  // namespace ssdgate
}  // namespace emab

extern "C" EMA_API int ssd_gate_fwd_launch(const SsdGateArgs* args, void* stream) {
  return emab::ssdgate::launch<false>(args, static_cast<cudaStream_t>(stream));
}

extern "C" EMA_API int ssd_gate_bwd_launch(const SsdGateArgs* args, void* stream) {
  return emab::ssdgate::launch<true>(args, static_cast<cudaStream_t>(stream));
}
