// launch.cuh -- how coding kernels map independent streams onto the B200.
//
// Each rANS stream is one serial dependency chain, so a coding kernel runs one thread per stream
// and its speed is set by the latency of one step, not by bandwidth (unless there are very many
// streams).  Uncoalesced per-lane accesses cost more L1/LSU cycles the more lanes of a warp are
// active, so streams are spread as evenly as possible over all SMs first (about B / num_SMs per
// SM), over up to 4 warps per SM next (one per scheduler), and only then over more lanes.
#pragma once

#include <cstdint>
#include <cstdlib>

namespace tans {

struct LaunchShape {
  int blocks;   // grid size
  int threads;  // threads per block (warps * 32)
  int lanes;    // active lanes (streams) per warp
};

constexpr int kMaxWarpsPerBlock = 8;

// count one kernel launch of this library (read back by tans_launch_count)
void note_launch();

inline int env_int(const char* name, int dflt) {
  const char* s = std::getenv(name);
  if (!s || !*s) return dflt;
  return std::atoi(s);
}

inline LaunchShape pick_launch(int64_t streams, int num_sms) {
  LaunchShape L{1, 32, 1};
  if (streams <= 0) return L;
  if (num_sms <= 0) num_sms = 148;
  const int64_t per_sm = (streams + num_sms - 1) / num_sms;
  int64_t warps = per_sm < 4 ? per_sm : 4;
  int64_t lanes = (per_sm + warps - 1) / warps;
  if (lanes > 32) {
    lanes = 32;
    warps = (per_sm + 31) / 32;
    if (warps > kMaxWarpsPerBlock) warps = kMaxWarpsPerBlock;
  }
  const int lanes_env = env_int("TORCH_ANS_B200_LANES", 0);
  const int warps_env = env_int("TORCH_ANS_B200_WARPS", 0);
  if (lanes_env > 0 && lanes_env <= 32) lanes = lanes_env;
  if (warps_env > 0 && warps_env <= kMaxWarpsPerBlock) warps = warps_env;
  const int64_t per_block = warps * lanes;
  L.blocks = (int)((streams + per_block - 1) / per_block);
  L.threads = (int)(warps * 32);
  L.lanes = (int)lanes;
  return L;
}

// stream index handled by this thread, or -1
__device__ __forceinline__ int64_t my_stream(int lanes, int64_t streams) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane >= lanes) return -1;
  const int64_t b = ((int64_t)blockIdx.x * (blockDim.x >> 5) + warp) * lanes + lane;
  return b < streams ? b : -1;
}

}  // namespace tans
