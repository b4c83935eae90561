// EMA forward for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc at all: an FFI caller
// (cgo, JNI, a C plugin) that has no device allocator of its own, a serving
// runtime that forbids allocation once its memory plan is fixed, or code that
// must not disturb another framework's caching allocator.  ema_fwd_launch needs
// a caller-provided workspace for the look-back between chunk tiles; this
// entry point instead uses a fixed scratch array that is compiled into the
// library (file-scope static device memory), so the caller only passes its
// inputs and outputs.
//
// The array lives on every GPU that loads the library until the process exits.
// Its device address is looked up once per device (cudaGetSymbolAddress with
// that device current) on the first call there; that first call also clears
// the array, so it must come before any stream capture.  The kernels keep the
// scratch consistent between calls themselves (generation-tagged flags,
// counters reset by the last CTA), so later calls clear nothing.  All calls on
// a device share the one array: two calls that overlap on the GPU (different
// streams without ordering) race and give wrong results.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "ema_common.cuh"
#include "ema_ssd_b200.h"

namespace emab {
void set_last_error(const char* msg);  // ema_scan_host.cu: text returned by ema_last_error()
}

namespace {

static __device__ __align__(256) unsigned char g_ema_fwd_scratch[EMA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

int fail_msg(int code, const char* msg) {
  emab::set_last_error(msg);
  return code;
}

}  // namespace

extern "C" EMA_API int ema_fwd_launch_noalloc(const EmaFwdArgs* args, void* stream) {
  if (args == nullptr) return fail_msg(EMA_ERR_INVALID_ARGUMENT, "ema_fwd_launch_noalloc: args is NULL");
  const size_t need =
      ema_scan_workspace_size(args->batch, args->seqlen, args->nheads, args->headdim, args->chunk_size);
  char msg[256];
  if (need > EMA_NOALLOC_SCRATCH_BYTES) {
    snprintf(msg, sizeof(msg),
             "ema_fwd_launch_noalloc: this shape needs %zu bytes of scratch; the static array holds %u "
             "(use ema_fwd_launch with a caller-provided workspace)",
             need, static_cast<unsigned>(EMA_NOALLOC_SCRATCH_BYTES));
    return fail_msg(EMA_ERR_WORKSPACE, msg);
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail_msg(EMA_ERR_CUDA, "ema_fwd_launch_noalloc: no usable current device");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_ema_fwd_scratch);
      if (e != cudaSuccess || p == nullptr) {
        snprintf(msg, sizeof(msg), "ema_fwd_launch_noalloc: cudaGetSymbolAddress failed: %s",
                 cudaGetErrorString(e));
        return fail_msg(EMA_ERR_CUDA, msg);
      }
      // the look-back protocol starts from an all-zero scratch
      e = cudaMemsetAsync(p, 0, EMA_NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) {
        snprintf(msg, sizeof(msg), "ema_fwd_launch_noalloc: clearing the scratch failed: %s",
                 cudaGetErrorString(e));
        return fail_msg(EMA_ERR_CUDA, msg);
      }
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }
  EmaFwdArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = EMA_NOALLOC_SCRATCH_BYTES;
  return ema_fwd_launch(&a, stream);
}

// The kernels report a give-up of a bounded wait (a look-back or load that
// did not complete within its time limit) and a ticket count that shows two
// launches shared the scratch at once in the scratch's header status word.
// Callers of ema_fwd_launch read that word through their own workspace
// pointer (ema_workspace_status); callers of the entry point above never see
// the static array's address, so this reads (and optionally clears) the word
// for them.  Before the first ema_fwd_launch_noalloc on the current device
// there is nothing to report: *status is 0.
extern "C" EMA_API int ema_noalloc_status(uint32_t* status, int32_t clear, void* stream) {
  if (status == nullptr) return fail_msg(EMA_ERR_INVALID_ARGUMENT, "ema_noalloc_status: status is NULL");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail_msg(EMA_ERR_CUDA, "ema_noalloc_status: no usable current device");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    scratch = g_scratch_ptr[dev];
  }
  *status = 0u;
  if (scratch == nullptr) return EMA_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t* word = static_cast<uint32_t*>(scratch) + emab::kHdrStatus;
  char msg[256];
  cudaError_t e = cudaMemcpyAsync(status, word, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(word, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "ema_noalloc_status: %s", cudaGetErrorString(e));
    return fail_msg(EMA_ERR_CUDA, msg);
  }
  return EMA_OK;
}
