// EMA scan kernel instantiations for element type float.
#include "ema_scan_inst.cuh"

namespace emab {
int fwd_dispatch_f32(const FwdLaunch& l) { return inst::fwd_all<float>(l); }
int bwd_dispatch_f32(const BwdLaunch& l) { return inst::bwd_all<float>(l); }
}  // namespace emab
