/*
 * ema_selftest_b200.h -- test-only library libema_selftest_b200.so.
 *
 * Not part of the product or of the reference interface: these check, on the
 * GPU, the tcgen05 operand conventions (128-byte-swizzled shared-memory tiles,
 * K-major and MN-major descriptors, tensor-memory accumulators) that the SSD
 * kernels are built on.  Used by the GPU test suite only.
 */
#ifndef EMA_SELFTEST_B200_H_
#define EMA_SELFTEST_B200_H_

#include "ema_ssd_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One 128-row bf16 GEMM with fp32 accumulation on the tensor cores (device
 * pointers, row-major, contiguous; `status` one zeroed device word):
 *   mode 0: d (128x128) = a (128x128) * b (128x128)^T
 *   mode 1: d (128x64)  = a (128x128) * b (128x64)
 *   mode 2: d (128x128) = a (128x128)^T * b (128x128)
 *   mode 3: as mode 0, with `a` staged into shared memory by the threads. */
EMA_API int tc_selftest_gemm(int mode, const void* a, const void* b, float* d, uint32_t* status, void* stream);
/* Detail of the last error returned on the calling thread. */
EMA_API const char* tc_selftest_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* EMA_SELFTEST_B200_H_ */
