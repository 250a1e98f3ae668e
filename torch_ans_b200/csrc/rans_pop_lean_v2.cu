// rans_pop_lean_v2.cu -- instantiations of the lean pop kernel for coder variant 2.
#include "rans_pop_lean.cuh"

namespace tans {
TANS_DEFINE_POP_LEAN(2)
}  // namespace tans
