// rans_push_fast_v1.cu -- instantiations of the fast push kernel for coder variant 1.
#include "rans_push_fast.cuh"

namespace tans {
TANS_DEFINE_PUSH_FAST(1)
}  // namespace tans
