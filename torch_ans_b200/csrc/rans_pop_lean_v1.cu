// rans_pop_lean_v1.cu -- instantiations of the lean pop kernel for coder variant 1.
#include "rans_pop_lean.cuh"

namespace tans {
TANS_DEFINE_POP_LEAN(1)
}  // namespace tans
