// EMA scan kernel instantiations for element type __nv_bfloat16.
#include "ema_scan_inst.cuh"

namespace emab {
int fwd_dispatch_bf16(const FwdLaunch& l) { return inst::fwd_all<__nv_bfloat16>(l); }
int bwd_dispatch_bf16(const BwdLaunch& l) { return inst::bwd_all<__nv_bfloat16>(l); }
}  // namespace emab
