// rans_probe.cu -- latency probes behind the kernel design (tans_probe, no counterpart in the
// reference).
//
// A rANS stream is one serial chain, so what bounds every coding kernel is the latency of one
// dependent step.  These probes measure, with clock64 on the device, the cycles of one step of:
//   * dependent loads around a random cycle in shared memory, in an L2-resident global buffer
//     (one thread), and in the same buffer with 56 chasing lanes on every SM (14 warps x 4 lanes,
//     the headline pop's occupancy);
//   * the arithmetic chain of a pop step and of a push step, rans32 (8-bit words) and rans64
//     (32-bit words), 16-bit frequency precision, one thread, with the table entry in shared
//     memory and the stream words produced in registers: nothing but the step's own dependent
//     instructions, i.e. the floor under a one-stream-per-SM kernel.
// The host side allocates its buffers, runs one probe synchronously and frees them; it is a
// diagnostic (the benchmark's --probe mode), not a coding path.
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "../../include/torch_ans_b200.h"
#include "launch.cuh"
#include "rans_host.h"

namespace tans {
namespace {

__device__ __forceinline__ uint64_t xorshift64(uint64_t s) {
  s ^= s << 13;
  s ^= s >> 7;
  s ^= s << 17;
  return s;
}

// ---------------------------------------------------------------- dependent-load chases
// next[i] holds the index of the element after i on one random cycle through the buffer
__global__ void chase_smem_kernel(const uint32_t* next, int n, int64_t steps, unsigned long long* out) {
  extern __shared__ uint32_t sm[];
  for (int i = threadIdx.x; i < n; i += blockDim.x) sm[i] = next[i];
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint32_t j = 0;
  for (int w = 0; w < 64; ++w) j = sm[j];
  const long long t0 = clock64();
  for (int64_t s = 0; s < steps; ++s) j = sm[j];
  const long long t1 = clock64();
  out[0] = (unsigned long long)(t1 - t0);
  out[1] = j;  // keeps the chain live
}

// one dependent load per step; `per_lane` cycles each start at a different element.  The
// entries are 8 bytes (the bucket table's entry size) and the index sits in their low word.
__global__ void chase_global_kernel(const unsigned long long* next, int64_t n, int64_t steps, int lanes,
                                    unsigned long long* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane >= lanes) return;
  const int64_t g = ((int64_t)blockIdx.x * (blockDim.x >> 5) + warp) * lanes + lane;
  uint64_t j = (uint64_t)((g * 2654435761ull) % (uint64_t)n);
  for (int w = 0; w < 16; ++w) j = __ldcg(next + j) & 0xFFFFFFFFull;
  const long long t0 = clock64();
  for (int64_t s = 0; s < steps; ++s) j = __ldcg(next + j) & 0xFFFFFFFFull;
  const long long t1 = clock64();
  out[2 * g] = (unsigned long long)(t1 - t0);
  out[2 * g + 1] = j;
}

// ---------------------------------------------------------------- step chains (one thread)
// Table: 4,096 symbols of frequency 16 over 2^16 (symbol s covers cum [16 s, 16 s + 16)); the
// pop's entry for cum is entry[cum >> 4] = freq | start << 16, the push's entry for a symbol
// is {reciprocal, shift, start}.  Every step decodes / encodes a real symbol of that table, so
// the state stays in range and each step renormalises like a coding step at ~12 bits per symbol.
__global__ void pop32_step_kernel(int64_t steps, uint64_t seed, unsigned long long* out) {
  __shared__ uint32_t ent[4096];
  for (int i = threadIdx.x; i < 4096; i += blockDim.x) ent[i] = 16u | ((uint32_t)(16 * i) << 16);
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint32_t x = (1u << 23) | (uint32_t)(seed & 0x7FFFFFu);
  uint64_t rnd = seed | 1u;
  uint32_t acc = 0;
  const long long t0 = clock64();
  for (int64_t s = 0; s < steps; ++s) {
    rnd = xorshift64(rnd);  // stream bytes: independent of the state
    const uint32_t cum = x & 0xFFFFu;
    const uint32_t e = ent[cum >> 4];
    const uint32_t f = e & 0xFFFFu, start = e >> 16;
    acc += cum >> 4;  // the decoded symbol
    x = f * (x >> 16) + (cum - start);
    // renormalisation without a branch: the bytes needed to reach [2^23, 2^31)
    const uint32_t n = x < (1u << 23) ? (uint32_t)(__clz(x) - 1) >> 3 : 0u;
    x = n ? (x << (8 * n)) | (uint32_t)(rnd >> (64 - 8 * n)) : x;
  }
  const long long t1 = clock64();
  out[0] = (unsigned long long)(t1 - t0);
  out[1] = x + acc;
}

__global__ void push32_step_kernel(int64_t steps, uint64_t seed, unsigned long long* out) {
  // per symbol, as the push's encode entries: reciprocal of the frequency, frequency, start
  __shared__ uint32_t rec[4096], frq[4096], st[4096];
  for (int i = threadIdx.x; i < 4096; i += blockDim.x) {
    rec[i] = 1u << 28;  // 2^32 / 16: mulhi(x, rec) = x / 16
    frq[i] = 16u;
    st[i] = (uint32_t)(16 * i);
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint32_t x = 1u << 23;
  uint64_t rnd = seed | 1u;
  uint32_t emitted = 0;
  const long long t0 = clock64();
  for (int64_t s = 0; s < steps; ++s) {
    rnd = xorshift64(rnd);
    const uint32_t sym = (uint32_t)rnd & 4095u;  // symbol: independent of the state
    const uint32_t m = rec[sym], f = frq[sym], start = st[sym];
    // renormalisation: emit bytes while x >= ((2^23 >> 16) << 8) * f (at most 2 here)
    const uint32_t xmax = ((1u << 23) >> 16 << 8) * f;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const bool e = x >= xmax;
      emitted += e ? (x & 0xFFu) : 0u;
      x = e ? x >> 8 : x;
    }
    const uint32_t q = __umulhi(x, m);
    x = x + start + q * ((1u << 16) - f);
  }
  const long long t1 = clock64();
  out[0] = (unsigned long long)(t1 - t0);
  out[1] = x + emitted;
}

__global__ void pop64_step_kernel(int64_t steps, uint64_t seed, unsigned long long* out) {
  __shared__ uint32_t ent[4096];
  for (int i = threadIdx.x; i < 4096; i += blockDim.x) ent[i] = 16u | ((uint32_t)(16 * i) << 16);
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint64_t x = (1ull << 31) | (seed & 0x7FFFFFFFFFFFull);
  uint64_t rnd = seed | 1u;
  uint32_t acc = 0;
  const long long t0 = clock64();
  for (int64_t s = 0; s < steps; ++s) {
    rnd = xorshift64(rnd);
    const uint32_t cum = (uint32_t)x & 0xFFFFu;
    const uint32_t e = ent[cum >> 4];
    const uint32_t f = e & 0xFFFFu, start = e >> 16;
    acc += cum >> 4;
    x = (x >> 16) * f + (cum - start);
    x = x < (1ull << 31) ? (x << 32) | (uint32_t)rnd : x;  // one 32-bit word at most
  }
  const long long t1 = clock64();
  out[0] = (unsigned long long)(t1 - t0);
  out[1] = x + acc;
}

__global__ void push64_step_kernel(int64_t steps, uint64_t seed, unsigned long long* out) {
  __shared__ unsigned long long rec[2048];  // (2,048 symbols: the static shared-memory limit)
  __shared__ uint32_t frq[2048], st[2048];
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) {
    rec[i] = 1ull << 60;  // 2^64 / 16: mulhi(x, rec) = x / 16
    frq[i] = 16u;
    st[i] = (uint32_t)(16 * i);
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  uint64_t x = 1ull << 31;
  uint64_t rnd = seed | 1u;
  uint64_t emitted = 0;
  const long long t0 = clock64();
  for (int64_t s = 0; s < steps; ++s) {
    rnd = xorshift64(rnd);
    const uint32_t sym = (uint32_t)rnd & 2047u;
    const unsigned long long m = rec[sym];
    const uint64_t f = frq[sym], start = st[sym];
    const uint64_t xmax = ((1ull << 31) >> 16 << 32) * f;
    const bool e = x >= xmax;
    emitted += e ? (uint32_t)x : 0u;
    x = e ? x >> 32 : x;
    const uint64_t q = __umul64hi(x, m);
    x = x + start + q * ((1ull << 16) - f);
  }
  const long long t1 = clock64();
  out[0] = (unsigned long long)(t1 - t0);
  out[1] = x + emitted;
}

// a random cyclic permutation of [0, n): next[order[i]] = order[i + 1]
std::vector<uint32_t> random_cycle(int64_t n, uint64_t seed) {
  std::vector<uint32_t> order((size_t)n);
  for (int64_t i = 0; i < n; ++i) order[(size_t)i] = (uint32_t)i;
  uint64_t r = seed | 1u;
  for (int64_t i = n - 1; i > 0; --i) {
    r ^= r << 13;
    r ^= r >> 7;
    r ^= r << 17;
    std::swap(order[(size_t)i], order[(size_t)(r % (uint64_t)(i + 1))]);
  }
  std::vector<uint32_t> next((size_t)n);
  for (int64_t i = 0; i < n; ++i) next[order[(size_t)i]] = order[(size_t)((i + 1) % n)];
  return next;
}

}  // namespace
}  // namespace tans

extern "C" int tans_probe(int kind, int64_t steps, double* cycles_per_step) {
  using namespace tans;
  if (!cycles_per_step || steps < 1 || steps > ((int64_t)1 << 30)) return TANS_E_INVALID_ARGUMENT;
  if (kind < TANS_PROBE_SMEM_CHASE || kind > TANS_PROBE_PUSH64_STEP) return TANS_E_INVALID_ARGUMENT;
  unsigned long long* d_out = nullptr;
  const int sms = sm_count();
  const int64_t out_words = 2 * (int64_t)sms * 56 + 2;
  if (cudaMalloc(&d_out, (size_t)out_words * 8) != cudaSuccess) return TANS_E_CUDA;
  int rc = TANS_OK;
  std::vector<unsigned long long> h(2);
  int64_t chains = 1;
  void* d_buf = nullptr;
  switch (kind) {
    case TANS_PROBE_SMEM_CHASE: {
      const int n = 12288;  // 48 KB
      const std::vector<uint32_t> nx = random_cycle(n, 7);
      if (cudaMalloc(&d_buf, nx.size() * 4) != cudaSuccess) { rc = TANS_E_CUDA; break; }
      cudaMemcpy(d_buf, nx.data(), nx.size() * 4, cudaMemcpyHostToDevice);
      chase_smem_kernel<<<1, 256, n * 4>>>(static_cast<const uint32_t*>(d_buf), n, steps, d_out);
      break;
    }
    case TANS_PROBE_L2_CHASE:
    case TANS_PROBE_L2_CHASE_BUSY: {
      const int64_t n = (8 << 20) / 8;  // 8 MB of 8-byte entries: the headline's bucket table size
      const std::vector<uint32_t> nx = random_cycle(n, 11);
      std::vector<unsigned long long> nx64(nx.begin(), nx.end());
      if (cudaMalloc(&d_buf, (size_t)n * 8) != cudaSuccess) { rc = TANS_E_CUDA; break; }
      cudaMemcpy(d_buf, nx64.data(), (size_t)n * 8, cudaMemcpyHostToDevice);
      const unsigned long long* nb = static_cast<const unsigned long long*>(d_buf);
      // one pass over the buffer first so that it is resident in L2
      chase_global_kernel<<<sms, 14 * 32>>>(nb, n, n / (sms * 56) + 1, 4, d_out);
      if (kind == TANS_PROBE_L2_CHASE) {
        chase_global_kernel<<<1, 32>>>(nb, n, steps, 1, d_out);
      } else {
        chase_global_kernel<<<sms, 14 * 32>>>(nb, n, steps, 4, d_out);
        chains = (int64_t)sms * 56;
      }
      break;
    }
    case TANS_PROBE_POP32_STEP: pop32_step_kernel<<<1, 256>>>(steps, 12345, d_out); break;
    case TANS_PROBE_PUSH32_STEP: push32_step_kernel<<<1, 256>>>(steps, 12345, d_out); break;
    case TANS_PROBE_POP64_STEP: pop64_step_kernel<<<1, 256>>>(steps, 12345, d_out); break;
    case TANS_PROBE_PUSH64_STEP: push64_step_kernel<<<1, 256>>>(steps, 12345, d_out); break;
    default: rc = TANS_E_INVALID_ARGUMENT;
  }
  if (rc == TANS_OK) {
    note_launch();
    h.resize((size_t)(2 * chains));
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(h.data(), d_out, h.size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) {
      rc = TANS_E_CUDA;
    } else {
      double sum = 0.0;
      for (int64_t c = 0; c < chains; ++c) sum += (double)h[(size_t)(2 * c)];
      *cycles_per_step = sum / (double)chains / (double)steps;
    }
  }
  if (d_buf) cudaFree(d_buf);
  cudaFree(d_out);
  return rc;
}
