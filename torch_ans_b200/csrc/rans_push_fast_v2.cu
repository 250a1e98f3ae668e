// rans_push_fast_v2.cu -- instantiations of the fast push kernel for coder variant 2.
#include "rans_push_fast.cuh"

namespace tans {
TANS_DEFINE_PUSH_FAST(2)
}  // namespace tans
