// rans_aux.cu -- argument checks, stream initialisation, length reduction, bitstream
// assembly/parsing and cdf repair kernels of libtorch_ans_b200.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "../../include/torch_ans_b200.h"
#include "rans_device.cuh"
#include "rans_host.h"

namespace tans {

static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  std::lock_guard<std::mutex> g(mu);
  if (dev < 64) cache[dev] = n;
  return n;
}

int check_coding_args(int variant, int interleave, const int32_t* stream, int64_t batch, int64_t width,
                      const int32_t* indexes, int64_t nsym, const int32_t* cdfs, int64_t ntables,
                      int64_t cdf_width, const int32_t* sizes, int fp, int bypass, int bp) {
  if (variant < 0 || variant > 2) return TANS_E_INVALID_ARGUMENT;
  if (interleave != 1 && interleave != 4) return TANS_E_INVALID_ARGUMENT;
  if (batch < 0 || nsym < 0 || ntables < 0 || cdf_width < 0) return TANS_E_INVALID_ARGUMENT;
  if (fp < 1 || fp > max_precision(variant)) return TANS_E_INVALID_ARGUMENT;
  if (bypass && (bp < 1 || bp > max_precision(variant))) return TANS_E_INVALID_ARGUMENT;
  if (batch == 0) return TANS_OK;
  if (!stream) return TANS_E_INVALID_ARGUMENT;
  // the row must hold the length word and the state slots
  if (width < 1 + (int64_t)interleave * state_bytes(variant) / 4) return TANS_E_INVALID_ARGUMENT;
  if (nsym > 0 && (!indexes || !cdfs || !sizes || ntables < 1 || cdf_width < 2)) return TANS_E_INVALID_ARGUMENT;
  return TANS_OK;
}

// ---------------------------------------------------------------- stream helpers
__global__ void max_length_kernel(const int32_t* stream, int64_t batch, int64_t width, int32_t* out) {
  __shared__ int32_t red[32];
  int32_t m = INT32_MIN;
  for (int64_t b = threadIdx.x; b < batch; b += blockDim.x) m = max(m, stream[b * width]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : INT32_MIN;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) *out = batch > 0 ? m : 0;
  }
}

template <int V>
__global__ void init_stream_kernel(int32_t* stream, int64_t batch, int64_t width, int interleave) {
  const int64_t total = batch * width;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t col = e % width;
    int32_t v = 0;
    if (col == 0) v = interleave * VT<V>::SBYTES;
    else if (col <= (int64_t)interleave * VT<V>::SBYTES / 4) {
      // state slots hold the lower bound (rans_cpu.cpp:32-36)
      if constexpr (V == 0) v = ((col - 1) & 1) == 0 ? (int32_t)(uint32_t)VT<0>::LB : 0;
      else v = (int32_t)(uint32_t)VT<V>::LB;
    }
    stream[e] = v;
  }
}

// one block per row: write [prefix][payload[0:len]] at record_offsets[b]
__global__ void gather_payloads_kernel(const int32_t* stream, int64_t batch, int64_t width,
                                       const int64_t* offsets, int prefix_bytes, int64_t prefix_rows, uint8_t* out) {
  for (int64_t b = blockIdx.x; b < batch; b += gridDim.x) {
    const int32_t* row = stream + b * width;
    // the same clamp to the row's payload capacity as the host uses for the offsets
    const int64_t len = min(max((int64_t)row[0], (int64_t)0), (width - 1) * 4);
    const int pre = b < prefix_rows ? prefix_bytes : 0;
    uint8_t* dst = out + offsets[b];
    if (threadIdx.x < pre) dst[threadIdx.x] = (uint8_t)(((unsigned long long)len) >> (8 * threadIdx.x));
    const uint8_t* src = reinterpret_cast<const uint8_t*>(row + 1);
    dst += pre;
    for (int64_t i = threadIdx.x; i < len; i += blockDim.x) dst[i] = src[i];
  }
}

__global__ void scatter_payloads_kernel(const uint8_t* in, const int64_t* offsets, const int32_t* lengths,
                                        int32_t* stream, int64_t batch, int64_t width) {
  for (int64_t b = blockIdx.x; b < batch; b += gridDim.x) {
    int32_t* row = stream + b * width;
    const int64_t len = lengths[b];
    uint8_t* dst = reinterpret_cast<uint8_t*>(row + 1);
    const uint8_t* src = in + offsets[b];
    const int64_t cap = (width - 1) * 4;
    for (int64_t i = threadIdx.x; i < cap; i += blockDim.x) dst[i] = i < len ? src[i] : 0;
    if (threadIdx.x == 0) row[0] = (int32_t)len;
  }
}

// per-row zero-frequency repair (rans_cpu.cpp:351-379): one thread per row, same scan order
__global__ void cdf_fix_kernel(int32_t* cdfs, int64_t rows, int64_t n, uint32_t* status) {
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < rows; b += (int64_t)gridDim.x * blockDim.x) {
    int32_t* row = cdfs + b * (n + 1);
    for (int64_t i = 0; i < n; ++i) {
      if (row[i] != row[i + 1]) continue;
      int32_t best = INT32_MAX;
      int64_t steal = -1;
      for (int64_t j = 0; j < n; ++j) {
        const int32_t f = row[j + 1] - row[j];
        if (f > 1 && f < best) {
          best = f;
          steal = j;
        }
      }
      if (steal < 0) {
        if (status) atomicOr(status, DEV_BAD_FREQ);
        break;
      }
      if (steal < i) {
        for (int64_t j = steal + 1; j <= i; ++j) row[j] -= 1;
      } else {
        for (int64_t j = i + 1; j <= steal; ++j) row[j] += 1;
      }
    }
  }
}

}  // namespace tans

extern "C" int tans_version(void) { return (0 << 16) | (1 << 8) | 0; }

extern "C" const char* tans_status_string(int code) {
  switch (code) {
    case TANS_OK: return "ok";
    case TANS_E_INVALID_ARGUMENT: return "invalid argument";
    case TANS_E_CUDA: return "CUDA error";
    case TANS_E_WORKSPACE: return "workspace missing or too small";
    case TANS_E_TOO_LARGE: return "problem larger than the entry point supports";
    default: return "unknown status";
  }
}

extern "C" int tans_stream_max_length(const int32_t* stream, int64_t batch, int64_t stream_width, int32_t* out_max,
                                      void* cuda_stream) {
  if (batch < 0 || !out_max || (batch > 0 && (!stream || stream_width < 1))) return TANS_E_INVALID_ARGUMENT;
  tans::max_length_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(cuda_stream)>>>(stream, batch, stream_width,
                                                                                       out_max);
  tans::note_launch();
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}

extern "C" int tans_init_stream(int variant, int num_interleaves, int32_t* stream, int64_t batch,
                                int64_t stream_width, void* cuda_stream) {
  if (variant < 0 || variant > 2 || num_interleaves < 1 || batch < 0) return TANS_E_INVALID_ARGUMENT;
  if (batch == 0) return TANS_OK;
  if (!stream || stream_width < 1 + (int64_t)num_interleaves * tans::state_bytes(variant) / 4)
    return TANS_E_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(cuda_stream);
  const int64_t total = batch * stream_width;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 8 * (int64_t)tans::sm_count());
  if (variant == TANS_RANS64) tans::init_stream_kernel<0><<<blocks, 256, 0, s>>>(stream, batch, stream_width, num_interleaves);
  else if (variant == TANS_RANS32) tans::init_stream_kernel<1><<<blocks, 256, 0, s>>>(stream, batch, stream_width, num_interleaves);
  else tans::init_stream_kernel<2><<<blocks, 256, 0, s>>>(stream, batch, stream_width, num_interleaves);
  tans::note_launch();
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}

extern "C" int tans_gather_payloads(const int32_t* stream, int64_t batch, int64_t stream_width,
                                    const int64_t* record_offsets, int prefix_bytes, int64_t prefix_rows, uint8_t* out,
                                    void* cuda_stream) {
  if (batch < 0 || !(prefix_bytes == 0 || prefix_bytes == 1 || prefix_bytes == 2 || prefix_bytes == 4 ||
                     prefix_bytes == 8))
    return TANS_E_INVALID_ARGUMENT;
  if (batch == 0) return TANS_OK;
  if (!stream || !record_offsets || !out) return TANS_E_INVALID_ARGUMENT;
  const int blocks = (int)std::min<int64_t>(batch, 65535);
  tans::gather_payloads_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(cuda_stream)>>>(
      stream, batch, stream_width, record_offsets, prefix_bytes, prefix_rows, out);
  tans::note_launch();
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}

extern "C" int tans_scatter_payloads(const uint8_t* in, const int64_t* payload_offsets, const int32_t* lengths,
                                     int32_t* stream, int64_t batch, int64_t stream_width, void* cuda_stream) {
  if (batch < 0) return TANS_E_INVALID_ARGUMENT;
  if (batch == 0) return TANS_OK;
  if (!in || !payload_offsets || !lengths || !stream || stream_width < 1) return TANS_E_INVALID_ARGUMENT;
  const int blocks = (int)std::min<int64_t>(batch, 65535);
  tans::scatter_payloads_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(cuda_stream)>>>(
      in, payload_offsets, lengths, stream, batch, stream_width);
  tans::note_launch();
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}

extern "C" int tans_cdf_fix_zero_freqs(int32_t* cdfs, int64_t rows, int64_t n, uint32_t* dev_status,
                                       void* cuda_stream) {
  if (rows < 0 || n < 0) return TANS_E_INVALID_ARGUMENT;
  if (rows == 0) return TANS_OK;
  if (!cdfs) return TANS_E_INVALID_ARGUMENT;
  const int blocks = (int)std::min<int64_t>((rows + 127) / 128, 4 * (int64_t)tans::sm_count());
  tans::cdf_fix_kernel<<<blocks, 128, 0, reinterpret_cast<cudaStream_t>(cuda_stream)>>>(cdfs, rows, n, dev_status);
  tans::note_launch();
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}

extern "C" uint64_t tans_launch_count(void) { return (uint64_t)tans::g_launches.load(std::memory_order_relaxed); }
