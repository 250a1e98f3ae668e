// rans_push_ws_v0.cu -- instantiations of the warp-specialised push kernel for coder variant 0.
#include "rans_push_ws.cuh"

namespace tans {
TANS_DEFINE_PUSH_WS(0)
}  // namespace tans
