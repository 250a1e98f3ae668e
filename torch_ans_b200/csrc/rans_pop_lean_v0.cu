// rans_pop_lean_v0.cu -- instantiations of the lean pop kernel for coder variant 0.
#include "rans_pop_lean.cuh"

namespace tans {
TANS_DEFINE_POP_LEAN(0)
}  // namespace tans
