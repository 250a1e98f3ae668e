// rans_push_common.cuh -- encode (push) building blocks shared by the push kernels: parameters,
// the word cursor, escape-value push (rans_utils.hpp:106-164), per-symbol preparation and the
// reference-exact symbol step (rans_utils.hpp:168-323).
#pragma once

#include <cuda_runtime.h>

#include "launch.cuh"
#include "rans_device.cuh"

namespace tans {

struct PushParams {
  int32_t* stream;
  int64_t batch, width;
  const int32_t* sym;
  const int32_t* idx;
  int64_t nsym;
  const uint4* enc;
  int64_t enc_stride;
  const TableInfo* tinfo;
  int64_t ntables;
  const int32_t* cdfs;
  int64_t cdf_width;
  int fp, bp;
  uint32_t* status;
  int lanes;
  int vec;
  int tin_smem;  // per-table info staged in shared memory
  unsigned wait_limit;  // tries of each bounded hand-over wait (warp-specialised kernel)
  int ws_tcopies;       // warp-specialised kernel: copies of the per-table {size, offset} records (1 or 16)
};

// ---------------------------------------------------------------- step pieces
template <int V> struct PushCursor {
  uint8_t* payload;  // row + 1
  int64_t p;         // index of the last written word
  int64_t cap;       // words that fit in the row
  uint32_t err;

  __device__ __forceinline__ void emit(typename VT<V>::State& x) {
    using W = typename VT<V>::Word;
    p += 1;
    if (p >= 0 && p < cap) reinterpret_cast<W*>(payload)[p] = (W)x;
    else err |= DEV_OVERFLOW;
    x >>= VT<V>::WB;
  }
};

// RANS_APPEND_BITS, rans_utils.hpp:63-68
template <int V>
__device__ __forceinline__ void append_bits(typename VT<V>::State& x, PushCursor<V>& c, int32_t value, int nbits) {
  using S = typename VT<V>::State;
  const unsigned long long bound = (VT<V>::LB >> nbits) << VT<V>::WB;
#pragma unroll
  for (int t = 0; t < VT<V>::MAX_RENORM; ++t)
    if ((unsigned long long)x >= bound) c.emit(x);
  x = (S)((x << nbits) | to_state<S>(value));
}

__device__ __forceinline__ int32_t shr_defined(int32_t a, int n) { return n >= 32 ? (a < 0 ? -1 : 0) : (a >> n); }

// rans_push_raw_value_step, rans_utils.hpp:106-164 (escape value, rare path)
template <int V>
__device__ __noinline__ void push_escape(typename VT<V>::State& x, PushCursor<V>& c, int32_t raw, int bp) {
  const int32_t maxb = (int32_t)((1u << bp) - 1u);
  int32_t nb = 0;
  while (nb <= 32 && shr_defined(raw, nb * bp) != 0) ++nb;
  const int32_t ncodes = nb / maxb;
  const int32_t rest = nb - ncodes * maxb;
  for (int32_t j = nb - 1; j >= 0; --j) append_bits<V>(x, c, shr_defined(raw, j * bp) & maxb, bp);
  append_bits<V>(x, c, rest, bp);
  for (int32_t j = 0; j < ncodes; ++j) append_bits<V>(x, c, maxb, bp);
}

enum : uint32_t { PREP_SKIP = 1u, PREP_ESC = 2u };

struct PushPrep {
  uint4 e;           // encode entry (in flight while the previous chunk runs)
  int64_t rbase;     // alias: index of the remap row start (k * cdf_width + cdf_size)
  int32_t rcap;      // alias: remap entries available in the row
  int32_t raw;       // escape value
  uint32_t flags;
};

template <int V, bool ALIAS, bool BYPASS>
__device__ __forceinline__ PushPrep push_prepare(const PushParams& P, int32_t s, int32_t k, bool in_row,
                                                 uint32_t& err) {
  PushPrep r;
  r.flags = PREP_SKIP;
  r.raw = 0;
  r.rbase = 0;
  r.rcap = 0;
  r.e = make_uint4(0, 0, 0, 0);
  if (!in_row) return r;
  if (k < 0 || (int64_t)k >= P.ntables) {
    err |= DEV_BAD_INDEX;
    return r;
  }
  const TableInfo t = load_tinfo(P.tinfo, k);
  int32_t v = (int32_t)((uint32_t)s - (uint32_t)t.offset);
  const int32_t maxv = t.size - 2;
  uint32_t flags = 0;
  if constexpr (BYPASS) {
    if (v < 0) {
      r.raw = -2 * v - 1;
      v = maxv;
    } else if (v >= maxv) {
      r.raw = 2 * (v - maxv);
      v = maxv;
    }
    if (v == maxv) flags |= PREP_ESC;
  }
  if (v < 0 || v >= t.size - 1 || (int64_t)v >= P.enc_stride) {
    err |= DEV_BAD_VALUE;
    return r;
  }
  r.e = __ldg(P.enc + (int64_t)k * P.enc_stride + v);
  if constexpr (ALIAS) {
    r.rbase = (int64_t)k * P.cdf_width + t.size;
    const int64_t cap = P.cdf_width - t.size;
    r.rcap = cap <= 0 ? 0 : (cap > 0x7fffffff ? 0x7fffffff : (int32_t)cap);
  }
  r.flags = flags;
  return r;
}

// one symbol: escape (if any), renormalise, x = C(s, x)  (rans_utils.hpp:209-321)
template <int V, bool ALIAS, bool BYPASS>
__device__ __forceinline__ void push_chain(const PushParams& P, typename VT<V>::State& x, PushCursor<V>& c,
                                           const PushPrep& r) {
  using S = typename VT<V>::State;
  if (r.flags & PREP_SKIP) return;
  if constexpr (BYPASS) {
    if (r.flags & PREP_ESC) push_escape<V>(x, c, r.raw, P.bp);
  }
  const bool packed = P.fp <= 23;
  const uint32_t freq = entry_freq(r.e, packed);
  if (freq == 0u) {
    c.err |= DEV_BAD_FREQ;
    return;
  }
  const unsigned long long bound = (unsigned long long)freq << (VT<V>::USED - P.fp);
#pragma unroll
  for (int t = 0; t < VT<V>::MAX_RENORM; ++t)
    if ((unsigned long long)x >= bound) c.emit(x);
  const S q = quotient_exact<V>(x, r.e, packed, freq);
  const S start = to_state<S>((int32_t)r.e.w);
  if constexpr (ALIAS) {
    const S ri = (S)(x - q * (S)freq + start);
    if ((unsigned long long)ri >= (unsigned long long)r.rcap) {
      c.err |= DEV_BAD_VALUE;
      return;
    }
    const int32_t rv = __ldg(P.cdfs + r.rbase + (int64_t)ri);
    x = (S)((q << P.fp) + to_state<S>(rv));
  } else {
    const S cmpl = (S)((S)1 << P.fp) - (S)freq;
    x = (S)(x + start + q * cmpl);
  }
}

}  // namespace tans
