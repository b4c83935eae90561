// Instantiation helpers for one element type; included by ema_scan_<type>.cu
// with EMA_ELEM (the C++ element type) and EMA_SUFFIX (the dispatcher name
// suffix) defined.
#pragma once

#include "ema_scan_dispatch.h"

namespace emab {
namespace inst {

// Persistent grid: every SM runs C::CTAS CTAs, never more CTAs than tiles.
inline unsigned persistent_grid(long long tiles, int num_sms, int ctas_per_sm) {
  const long long g = static_cast<long long>(num_sms) * ctas_per_sm;
  return static_cast<unsigned>(tiles < g ? tiles : g);
}

template <typename T, int BP, int Q, int MODE, bool SEQ>
int launch_fwd(const FwdLaunch& l) {
  using C = FwdCfg<T, BP, Q>;
  if constexpr (!C::R::OK || C::kBytes > kMaxDynSmem) {
    return -2;
  } else {
    static unsigned long long mask = 0;
    auto fn = ema_fwd_kernel<T, BP, Q, MODE, SEQ>;
    int e = ensure_smem_attr(reinterpret_cast<const void*>(fn), C::kBytes, &mask);
    if (e) return e;
    const cudaError_t le = launch_programmatic(fn, dim3(persistent_grid(l.tiles, l.num_sms, C::CTAS)), dim3(C::NT),
                                               C::kBytes, l.stream, *l.map_x, l.params);
    return static_cast<int>(le != cudaSuccess ? le : cudaGetLastError());
  }
}

template <typename T, int BP, int Q, int MODE>
int launch_bwd(const BwdLaunch& l) {
  using C = BwdCfg<T, BP, Q>;
  if constexpr (!C::R::OK || C::kBytes > kMaxDynSmem) {
    return -2;
  } else {
    static unsigned long long mask = 0;
    auto fn = ema_bwd_kernel<T, BP, Q, MODE>;
    int e = ensure_smem_attr(reinterpret_cast<const void*>(fn), C::kBytes, &mask);
    if (e) return e;
    const cudaError_t le = launch_programmatic(fn, dim3(persistent_grid(l.tiles, l.num_sms, C::CTAS)), dim3(C::NT),
                                               C::kBytes, l.stream, *l.map_x, *l.map_dy, *l.map_dx, l.params);
    return static_cast<int>(le != cudaSuccess ? le : cudaGetLastError());
  }
}

template <typename T, int BP, int MODE, bool SEQ>
int fwd_q(const FwdLaunch& l) {
  switch (l.chunk) {
    case 64: return launch_fwd<T, BP, 64, MODE, SEQ>(l);
    case 128: return launch_fwd<T, BP, 128, MODE, SEQ>(l);
    case 256: return launch_fwd<T, BP, 256, MODE, SEQ>(l);
    default: return -1;
  }
}

template <typename T, int MODE, bool SEQ>
int fwd_bp(const FwdLaunch& l) {
  switch (l.block_p) {
    case 64: return fwd_q<T, 64, MODE, SEQ>(l);
    case 128: return fwd_q<T, 128, MODE, SEQ>(l);
    default: return -1;
  }
}

template <typename T>
int fwd_all(const FwdLaunch& l) {
  if (l.mode == kFwdLog2) return l.seq ? fwd_bp<T, kFwdLog2, true>(l) : fwd_bp<T, kFwdLog2, false>(l);
  if (l.mode == kFwdDt && !l.seq) return fwd_bp<T, kFwdDt, false>(l);
  return -1;
}

template <typename T, int BP, int MODE>
int bwd_q(const BwdLaunch& l) {
  switch (l.chunk) {
    case 64: return launch_bwd<T, BP, 64, MODE>(l);
    case 128: return launch_bwd<T, BP, 128, MODE>(l);
    case 256: return launch_bwd<T, BP, 256, MODE>(l);
    default: return -1;
  }
}

template <typename T, int MODE>
int bwd_bp(const BwdLaunch& l) {
  switch (l.block_p) {
    case 64: return bwd_q<T, 64, MODE>(l);
    case 128: return bwd_q<T, 128, MODE>(l);
    default: return -1;
  }
}

template <typename T>
int bwd_all(const BwdLaunch& l) {
  if (l.mode == kBwdCumsum) return bwd_bp<T, kBwdCumsum>(l);
  if (l.mode == kBwdDt) return bwd_bp<T, kBwdDt>(l);
  return -1;
}

}  // namespace inst
}  // namespace emab
