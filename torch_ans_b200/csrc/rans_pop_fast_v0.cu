// rans_pop_fast_v0.cu -- instantiations of the fast pop kernel for coder variant 0 (one
// translation unit per variant so they compile in parallel).
#include "rans_pop_fast.cuh"

namespace tans {
TANS_DEFINE_POP_FAST(0)
}  // namespace tans
