// rans_pop_fast_v1.cu -- instantiations of the fast pop kernel for coder variant 1 (one
// translation unit per variant so they compile in parallel).
#include "rans_pop_fast.cuh"

namespace tans {
TANS_DEFINE_POP_FAST(1)
}  // namespace tans
