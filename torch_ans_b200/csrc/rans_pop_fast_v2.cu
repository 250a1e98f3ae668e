// rans_pop_fast_v2.cu -- instantiations of the fast pop kernel for coder variant 2 (one
// translation unit per variant so they compile in parallel).
#include "rans_pop_fast.cuh"

namespace tans {
TANS_DEFINE_POP_FAST(2)
}  // namespace tans
