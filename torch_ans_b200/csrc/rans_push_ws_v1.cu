// rans_push_ws_v1.cu -- instantiations of the warp-specialised push kernel for coder variant 1.
#include "rans_push_ws.cuh"

namespace tans {
TANS_DEFINE_PUSH_WS(1)
}  // namespace tans
