// rans_noalloc.cu -- tans_push_noalloc: the encode entry point for callers that cannot allocate
// device memory.
//
// Some hosts of this library may not call cudaMalloc at all: code running inside a memory
// budget owned by someone else (an inference server or framework whose caching allocator owns
// all device memory, a plugin that may only use the buffers its host hands it), or code that
// must not allocate after start-up (latency-critical serving loops, where an allocation can
// synchronise the device).  tans_push needs scratch for its per-call encode tables and either
// takes it from the caller or allocates it; this variant takes it from a fixed array that lives
// in the library's own device image instead, so it allocates nothing.
//
// The scratch is one file-scope __device__ array of kNoAllocScratchBytes (8 MiB).  Every GPU
// that loads the library holds this array until the process exits.  Its device address is
// looked up with cudaGetSymbolAddress once per device, the first time this entry point runs on
// that device (the host-side name of a __device__ variable is only a stand-in, never a device
// pointer).  That first call therefore does the set-up and should come before any stream
// capture.  All calls share the array and it keeps whatever the previous call left in it:
// nothing needs clearing, because the push prep kernels write every scratch byte the push kernel
// later reads.  Calls whose GPU work overlaps (on different streams, or from several threads
// without ordering) race on the array and must be serialised by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/torch_ans_b200.h"
#include "rans_host.h"

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};

// device address of the scratch array on the current device (set-up on first use)
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TANS_E_CUDA;
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return TANS_E_CUDA;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return TANS_OK;
}

}  // namespace

extern "C" int tans_push_noalloc(int variant, int use_alias, int num_interleaves, int32_t* stream, int64_t batch,
                                 int64_t stream_width, const int32_t* symbols, const int32_t* indexes,
                                 int64_t num_symbols, const int32_t* cdfs, int64_t num_tables, int64_t cdf_width,
                                 const int32_t* cdf_sizes, const int32_t* offsets, int freq_precision,
                                 int bypass_coding, int bypass_precision, uint32_t* dev_status, void* cuda_stream) {
  // the arguments are checked first, so a call gets the same error code as from tans_push
  const int arc = tans::check_coding_args(variant, num_interleaves, stream, batch, stream_width, indexes, num_symbols,
                                          cdfs, num_tables, cdf_width, cdf_sizes, freq_precision, bypass_coding,
                                          bypass_precision);
  if (arc != TANS_OK) return arc;
  const size_t need = tans::push_workspace_bytes(variant, num_tables, tans::push_entry_stride(cdf_width, freq_precision));
  if (need > kNoAllocScratchBytes) return TANS_E_TOO_LARGE;
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != TANS_OK) return rc;
  return tans::push_impl(variant, use_alias, num_interleaves, stream, batch, stream_width, symbols, indexes,
                         num_symbols, cdfs, num_tables, cdf_width, cdf_sizes, offsets, freq_precision, bypass_coding,
                         bypass_precision, scratch, kNoAllocScratchBytes, dev_status,
                         reinterpret_cast<cudaStream_t>(cuda_stream), /*allow_alloc=*/false);
}
