// Host-side dispatch from runtime (dtype, block headdim, chunk size, mode) to
// the compiled EMA scan kernel instantiations.  One definition per element
// type lives in ema_scan_{bf16,f16,f32}.cu so the instantiations compile in
// parallel.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <utility>

#include "ema_scan_kernels.cuh"

namespace emab {

struct FwdLaunch {
  const CUtensorMap* map_x;
  FwdParams params;
  int block_p, chunk, mode;
  bool seq;
  long long tiles;
  int num_sms;
  cudaStream_t stream;
};

struct BwdLaunch {
  const CUtensorMap* map_x;
  const CUtensorMap* map_dy;
  const CUtensorMap* map_dx;  // dx stored in boxes of bwd_segment_tokens(BP) tokens
  BwdParams params;
  int block_p, chunk, mode;
  long long tiles;
  int num_sms;
  cudaStream_t stream;
};

// Return values: 0 launched, -1 no instantiation for this combination,
// -2 the combination needs more shared memory than a CTA may have,
// otherwise a cudaError_t from the launch.
int fwd_dispatch_f32(const FwdLaunch& l);
int fwd_dispatch_bf16(const FwdLaunch& l);
int fwd_dispatch_f16(const FwdLaunch& l);
int bwd_dispatch_f32(const BwdLaunch& l);
int bwd_dispatch_bf16(const BwdLaunch& l);
int bwd_dispatch_f16(const BwdLaunch& l);

// Tensor-core backward (ema_bwd_tc.cu): bf16, headdim 64, 128-token chunks,
// dx requested.  Returns 1 when the case is not covered (run the CUDA-core
// kernel instead), 0 when launched, -3 when a tensor map could not be
// encoded (message set), otherwise a cudaError_t.
int bwd_tc_launch(const BwdLaunch& l, int dtype, const void* x, const int64_t xs[3], const void* dy,
                  const int64_t dys[3], void* dx, const int64_t dxs[3]);
// Tensor-core forward (ema_fwd_tc.cu): dt form, bf16, headdim 64, 128-token
// chunks, y requested, no seq_idx / mid-chunk states.  Same return values.
int fwd_tc_launch(const FwdLaunch& l, int dtype, const void* x, const int64_t xs[3], void* y,
                  const int64_t ys[3]);
// Whether the tensor-core backward / forward are used where they apply
// (ema_set_tensor_core_path bits 0 / 1; default off).
bool tensor_core_path_enabled();
bool fwd_tensor_core_path_enabled();

constexpr int kMaxDynSmem = 232448;  // 227 KB per CTA on sm_100

// Set the dynamic shared-memory opt-in of `fn` once per device.
int ensure_smem_attr(const void* fn, int bytes, unsigned long long* device_mask);

// Launch with programmatic stream serialisation: the kernel's CTAs may be
// scheduled while the previous kernel on the stream is still finishing, and
// run their prologue up to grid_dep_wait() (ema_common.cuh) meanwhile -- the
// launch latency and the prologue overlap the previous kernel's tail.
template <typename... Params, typename... Args>
inline cudaError_t launch_programmatic(void (*fn)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                       Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, std::forward<Args>(args)...);
}
// Tiled tensor map of `rank` dims (dims[0] innermost), byte strides of dims
// 1..rank-1, box extents; 128-byte swizzle or none.  EMA_OK or an error code
// with the message set.
int encode_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* ptr, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);

}  // namespace emab
