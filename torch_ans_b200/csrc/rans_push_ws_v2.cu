// rans_push_ws_v2.cu -- instantiations of the warp-specialised push kernel for coder variant 2.
#include "rans_push_ws.cuh"

namespace tans {
TANS_DEFINE_PUSH_WS(2)
}  // namespace tans
