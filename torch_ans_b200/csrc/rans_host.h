// rans_host.h -- host-side helpers shared by the CUDA translation units of libtorch_ans_b200.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/torch_ans_b200.h"

namespace tans {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t n) { return (n + kAlign - 1) / kAlign * kAlign; }

// number of SMs of the current device (cached per device)
int sm_count();

// bits of state minus one minus word bits: the largest usable frequency precision per variant
// (rans_utils.hpp:181: freq_precision <= RANS_STATE_USED_BITS - RANS_STREAM_BITS)
inline int max_precision(int variant) { return variant == TANS_RANS64 ? 31 : (variant == TANS_RANS32 ? 23 : 15); }
inline int state_bytes(int variant) { return variant == TANS_RANS64 ? 8 : 4; }
inline int word_bytes(int variant) { return variant == TANS_RANS64 ? 4 : (variant == TANS_RANS32 ? 1 : 2); }

// argument checks shared by push and pop; returns TANS_OK or TANS_E_INVALID_ARGUMENT
int check_coding_args(int variant, int interleave, const int32_t* stream, int64_t batch, int64_t width,
                      const int32_t* indexes, int64_t nsym, const int32_t* cdfs, int64_t ntables,
                      int64_t cdf_width, const int32_t* sizes, int fp, int bypass, int bp);

size_t push_workspace_bytes(int variant, int64_t ntables, int64_t enc_stride);
int64_t push_entry_stride(int64_t cdf_width, int fp);
size_t pop_workspace_bytes(int variant, int lookup, int64_t ntables, int64_t cdf_width, int fp);

int push_impl(int variant, int use_alias, int interleave, int32_t* stream, int64_t batch, int64_t width,
              const int32_t* symbols, const int32_t* indexes, int64_t nsym, const int32_t* cdfs, int64_t ntables,
              int64_t cdf_width, const int32_t* sizes, const int32_t* offsets, int fp, int bypass, int bp,
              void* workspace, size_t ws_bytes, uint32_t* status, cudaStream_t s, bool allow_alloc);

int pop_impl(int variant, int lookup, int interleave, int32_t* stream, int64_t batch, int64_t width, int32_t* out,
             const int32_t* indexes, int64_t nsym, const int32_t* cdfs, int64_t ntables, int64_t cdf_width,
             const int32_t* sizes, const int32_t* offsets, int fp, int bypass, int bp, void* workspace,
             size_t ws_bytes, uint32_t* status, cudaStream_t s, bool allow_alloc);

}  // namespace tans
