// rans_push_fast_v0.cu -- instantiations of the fast push kernel for coder variant 0.
#include "rans_push_fast.cuh"

namespace tans {
TANS_DEFINE_PUSH_FAST(0)
}  // namespace tans
