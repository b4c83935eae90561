// EMA scan kernel instantiations for element type __half.
#include "ema_scan_inst.cuh"

namespace emab {
int fwd_dispatch_f16(const FwdLaunch& l) { return inst::fwd_all<__half>(l); }
int bwd_dispatch_f16(const BwdLaunch& l) { return inst::bwd_all<__half>(l); }
}  // namespace emab
