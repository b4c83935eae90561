// Self-test of the tcgen05 conventions in tc_common.cuh: one 128-row bf16
// GEMM per call, operands brought into shared memory by 128-byte-swizzled TMA
// loads (or written by threads in the same layout), D accumulated in tensor
// memory and read back with tcgen05.ld.  The SSD kernels rely on exactly these
// operand forms, so the GPU tests run this first.
//
//   mode 0: D[128x128] = A B^T,  A (128 x 128) and B (128 x 128) row-major, K contiguous (K-major)
//   mode 1: D[128x64]  = A X,    X (128 x 64) row-major: N contiguous (MN-major B)
//   mode 2: D[128x128] = X^T Y,  X, Y (128 x 128) row-major: M / N contiguous (MN-major A and B)
//   mode 3: mode 0 with A written into shared memory by the threads
//   mode 4: an M = 64 MMA, D[64x64] = A B^T (A, B 64 x 128, K-major), written
//           into zeroed tensor memory; all 128 lanes x 64 columns are read
//           back, which shows where the 64 rows of D live
//
// Test infrastructure: built by ema-kernels_b200/build.py into
// tests/native/libema_selftest_b200.so, apart from the product library, and
// loaded only by tests/test_tcgen05_gpu.py.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <string>

#include "ema_common.cuh"
#include "ema_selftest_b200.h"
#include "tc_common.cuh"

namespace emab {
namespace {

thread_local std::string g_error;

void set_last_error(const char* msg) { g_error = msg; }

// Tiled 2-D bf16 tensor map with 128-byte swizzle (this library's own copy of
// the product library's encoder).
int encode_map(CUtensorMap* m, const void* ptr, const uint64_t* dims, const uint64_t* stride_bytes,
               const uint32_t* box) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  if (enc == nullptr) {
    set_last_error("cuTensorMapEncodeTiled is not available from the driver");
    return EMA_ERR_CUDA;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) {  // bind the context
    set_last_error("no current device");
    return EMA_ERR_CUDA;
  }
  cuuint64_t d[2] = {dims[0], dims[1]};
  cuuint64_t st[1] = {stride_bytes[0]};
  cuuint32_t b[2] = {box[0], box[1]}, e[2] = {1u, 1u};
  if (enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed");
    return EMA_ERR_CUDA;
  }
  return EMA_OK;
}

constexpr int kRegion = 128 * 128;  // one 128-row x 64-column bf16 region, bytes

__global__ void __launch_bounds__(128, 1)
    tc_selftest_kernel(const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mb, int mode,
                       const __nv_bfloat16* a_plain, float* d, uint32_t* status) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sa = smem;                // 2 regions
  unsigned char* sb = smem + 2 * kRegion;  // 2 regions
  __shared__ uint64_t full, done;
  __shared__ uint32_t s_taddr;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = (mode == 1 || mode == 4) ? 64 : 128;
  const int R = (mode == 4) ? 64 : 128;  // operand rows
  const int reg = R * 128;               // bytes of one 64-column region
  if (tid == 0) {
    mbar_init(&full, 1);
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(&s_taddr, 128);
  if (mode == 3) {
    // A by the threads: element (r, k) -> region k / 64, swizzled (r, k % 64)
    for (int i = tid; i < 128 * 128; i += 128) {
      const int r = i / 128, k = i % 128;
      *reinterpret_cast<__nv_bfloat16*>(sa + (k / 64) * kRegion + tc::sw128_offset(r, k % 64)) = a_plain[i];
    }
    fence_proxy_async_smem();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = s_taddr;
  {  // zero the accumulator columns of every lane
    float z[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) z[i] = 0.f;
    for (int c0 = 0; c0 < 128; c0 += 16) tc::tmem_st16(tc::tmem_at(tbase, 32 * warp, c0), z);
    tc::tmem_wait_st();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (tid == 0) {
    const uint32_t bytes = (mode == 3 ? 0u : 2u * reg) + (mode == 1 ? 1u * kRegion : 2u * reg);
    mbar_arrive_expect_tx(&full, bytes);
    if (mode != 3) {
      tc::tma_load_2d(sa, &ma, &full, 0, 0);
      tc::tma_load_2d(sa + reg, &ma, &full, 64, 0);
    }
    if (mode == 1) {
      tc::tma_load_2d(sb, &mb, &full, 0, 0);  // 128 rows x 64 columns: one region of 16 KB
    } else {
      tc::tma_load_2d(sb, &mb, &full, 0, 0);
      tc::tma_load_2d(sb + reg, &mb, &full, 64, 0);
    }
    if (mbar_wait_bounded(&full, 0, status)) {
      tc::fence_after_sync();
      const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb);
      uint32_t idesc;
      if (mode == 1) idesc = tc::idesc_bf16(128, 64, false, true);
      else if (mode == 2) idesc = tc::idesc_bf16(128, 128, true, true);
      else if (mode == 4) idesc = tc::idesc_bf16(64, 64, false, false);
      else idesc = tc::idesc_bf16(128, 128, false, false);
#pragma unroll 1
      for (int s = 0; s < 8; ++s) {  // K = 128 in steps of 16
        uint64_t da, db;
        if (mode == 2) {
          da = tc::smem_desc_sw128(a0 + s * 2048, kRegion, 1024);
          db = tc::smem_desc_sw128(b0 + s * 2048, kRegion, 1024);
        } else {
          da = tc::smem_desc_sw128(a0 + (s / 4) * reg + (s % 4) * 32, 16, 1024);
          db = (mode == 1) ? tc::smem_desc_sw128(b0 + s * 2048, kRegion, 1024)
                           : tc::smem_desc_sw128(b0 + (s / 4) * reg + (s % 4) * 32, 16, 1024);
        }
        tc::mma_bf16(tbase, da, db, idesc, s > 0);
      }
      tc::mma_commit(&done);
    } else {
      mbar_arrive(&done);  // nothing issued: release the readers (the status word records the timeout)
    }
  }
  const bool ok = mbar_wait_bounded(&done, 0, status);
  tc::fence_after_sync();
  if (ok) {
    const int row = 32 * warp + lane;
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      tc::tmem_ld16(tc::tmem_at(tbase, 32 * warp, c0), v);
      tc::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) d[row * N + c0 + i] = v[i];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::tmem_relinquish();
    tc::tmem_dealloc(tbase, 128);
  }
}

}  // namespace
}  // namespace emab

using namespace emab;

extern "C" EMA_API int tc_selftest_gemm(int mode, const void* a, const void* b, float* d, uint32_t* status,
                                        void* stream) {
  if (mode < 0 || mode > 4 || !a || !b || !d || !status) {
    set_last_error("tc_selftest_gemm: bad arguments");
    return EMA_ERR_INVALID_ARGUMENT;
  }
  CUtensorMap ma{}, mb{};
  const uint64_t dims128[2] = {128, 128};
  const uint64_t st256[1] = {256};
  const uint32_t box[2] = {64, 128};
  int r = encode_map(&ma, a, dims128, st256, box);
  if (r) return r;
  if (mode == 4) {
    const uint64_t d64[2] = {128, 64};
    const uint32_t box64[2] = {64, 64};
    r = encode_map(&ma, a, d64, st256, box64);
    if (r) return r;
    r = encode_map(&mb, b, d64, st256, box64);
  } else if (mode == 1) {
    const uint64_t dims64[2] = {64, 128};
    const uint64_t st128[1] = {128};
    r = encode_map(&mb, b, dims64, st128, box);
  } else {
    r = encode_map(&mb, b, dims128, st256, box);
  }
  if (r) return r;
  const int smem = 4 * 128 * 128 + 1024;
  if (cudaFuncSetAttribute(tc_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    set_last_error("cudaFuncSetAttribute failed");
    return EMA_ERR_CUDA;
  }
  tc_selftest_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      ma, mb, mode, static_cast<const __nv_bfloat16*>(a), d, status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return EMA_ERR_CUDA;
  }
  return EMA_OK;
}

extern "C" EMA_API const char* tc_selftest_last_error(void) { return g_error.c_str(); }
