// rans_pop.cuh -- decode (pop) building blocks shared by the pop kernels: parameters, the
// word cursor, the escape-value pop, the symbol lookup of the reference (bisection / inverse cdf
// / alias, rans_utils.hpp:401-449) and the state update (rans_utils.hpp:473-531).
#pragma once

#include <cuda_runtime.h>

#include "launch.cuh"
#include "rans_device.cuh"

namespace tans {

struct PopParams {
  int32_t* stream;
  int64_t batch, width;
  int32_t* out;
  const int32_t* idx;
  int64_t nsym;
  const int32_t* cdfs;
  int64_t ntables, cdf_width;
  const TableInfo* tinfo;
  int fp, bp;
  uint32_t* status;
  int lanes;
  int vec;
  const uint32_t* fD;  // fused decode table D[k][cum] (nullptr: direct lookups)
  const uint16_t* fS;  // symbol table S[k][cum] (fused and split layouts)
  const uint32_t* fST; // split layout: per-symbol {freq - 1, start} ST[k][s]
  int64_t st_stride;   // split layout: entries per table in ST
  const unsigned long long* fBK;  // bucket layout: one entry per 16 cum values
  const unsigned long long* fSEC; // bucket layout: per-cum blocks of marker buckets (type 2)
  int64_t sec_cap;                // blocks the secondary table holds
  const unsigned long long* fL1;  // bucket layout: level-1 table staged in shared memory (or null)
  int64_t l1_bytes;               // its bytes (a multiple of 16; 0: no level-1 table)
  int l1_bits;                    // log2 of the cum values one level-1 entry covers
  int spt;             // streams per thread (fast kernel)
  int fused_smem;      // fused table staged in shared memory
  int tin_smem;        // per-table info staged in shared memory
  int vec_out;         // out is 16-byte aligned
  int iring;           // bucket kernel: indexes through a per-stream shared-memory ring fed by bulk copies
  int64_t iring_off;   // its byte offset in the block's dynamic shared memory
};

template <int V> struct PopCursor {
  const uint8_t* payload;  // row + 1
  int64_t p;               // index of the next word to read
  int64_t first;           // first word index after the state slots
  int64_t cap;             // words in the row (reads at or above are refused)
  uint32_t err;

  __device__ __forceinline__ void refill(typename VT<V>::State& x) {
    using S = typename VT<V>::State;
    using W = typename VT<V>::Word;
#pragma unroll
    for (int t = 0; t < VT<V>::MAX_RENORM; ++t) {
      if ((unsigned long long)x < VT<V>::LB) {
        S w = 0;
        if (p >= first && p < cap) w = (S)__ldg(reinterpret_cast<const W*>(payload) + p);
        else err |= DEV_UNDERFLOW;
        x = (S)((x << VT<V>::WB) | w);
        p -= 1;
      }
    }
  }
};

// rans_pop_raw_value_step, rans_utils.hpp:327-375 (escape value, rare path)
template <int V>
__device__ __noinline__ int32_t pop_escape(typename VT<V>::State& x, PopCursor<V>& c, int bp) {
  using S = typename VT<V>::State;
  const int32_t maxb = (int32_t)((1u << bp) - 1u);
  int32_t val = (int32_t)(x & (S)maxb);
  x >>= bp;
  c.refill(x);
  int32_t n = val;
  while (val == maxb && n <= 32) {
    val = (int32_t)(x & (S)maxb);
    x >>= bp;
    c.refill(x);
    n += val;
  }
  if (n > 32) {
    c.err |= DEV_BAD_ESCAPE;
    n = 0;
  }
  uint32_t raw = 0;
  for (int32_t j = 0; j < n; ++j) {
    val = (int32_t)(x & (S)maxb);
    x >>= bp;
    c.refill(x);
    if (j * bp < 32) raw |= (uint32_t)val << (j * bp);
  }
  return (int32_t)raw;
}

enum : int { LK_SEARCH = 0, LK_INVCDF = 1, LK_ALIAS = 2 };

// bucket kernel's index ring: two halves of kRingChunks chunks (4 indexes each) per stream, plus
// two 8-byte mbarriers per stream.  A stream's ring starts kRingStride bytes after the previous
// one: 16 bytes more than the ring, so the lanes of a warp reading the same chunk slot hit
// different shared-memory banks.
constexpr int kRingChunks = 16;
constexpr int64_t kRingStride = 2 * kRingChunks * 16 + 16;
constexpr int64_t kRingBytesPerStream = kRingStride + 16;
// tries of a ring wait before it gives up (TANS_DEV_STALLED): far beyond any real copy
constexpr unsigned kRingWaitLimit = 1u << 20;

// a table word: read-only global memory (GLOBAL) or a row staged in shared memory
template <bool GLOBAL> __device__ __forceinline__ int32_t ldrow(const int32_t* p) {
  if constexpr (GLOBAL) return __ldg(p);
  else return *p;
}

// Symbol lookup of rans_utils.hpp:401-449 for one cum value of table row `row`: sets s and the
// offset cum - start (alias: cum - alias_start) and the symbol's frequency.  Returns false where
// the reference would index outside the row (then nothing is read out of bounds).
template <int V, int LK, bool GLOBAL = true>
__device__ __forceinline__ bool lookup_symbol(const int32_t* row, const TableInfo& t, int32_t cum, int64_t cdf_width,
                                              int fp, int64_t& s, int32_t& cum_off, int32_t& freq) {
  using S = typename VT<V>::State;
  const int32_t size = t.size;
  if (size < 2 || (int64_t)size > cdf_width) return false;
  cum_off = cum;
  if constexpr (LK == LK_ALIAS) {
    if (t.cut <= 0) return false;
    const int32_t id = t.cut_log2 >= 0 ? (cum >> t.cut_log2) : (cum / t.cut);
    const int64_t at = (int64_t)size + 4 * (int64_t)id;
    if (at + 3 >= cdf_width) return false;
    const int32_t cut_cdf = ldrow<GLOBAL>(row + at);
    const int32_t other = ldrow<GLOBAL>(row + at + 1);
    const int32_t self_off = ldrow<GLOBAL>(row + at + 2);
    const int32_t other_off = ldrow<GLOBAL>(row + at + 3);
    const bool hi = cum >= cut_cdf;
    s = hi ? other : id;
    cum_off -= hi ? other_off : self_off;
  } else if constexpr (LK == LK_INVCDF) {
    if ((int64_t)size + cum >= cdf_width) return false;
    s = ldrow<GLOBAL>(row + size + cum);
  } else {
    // probe (cdf_size * cum) >> fp, then bisection on [0, cdf_size - 1] (rans_utils.hpp:427-448)
    S ix = to_state<S>((int32_t)((uint32_t)size * (uint32_t)cum) >> fp);
    uint32_t low = 0, high = (uint32_t)(size - 1);
    while (high > low) {
      if ((unsigned long long)ix >= (unsigned long long)size) return false;
      if (cum >= ldrow<GLOBAL>(row + ix)) low = (uint32_t)ix + 1u;
      else high = (uint32_t)ix;
      ix = (S)((low + high) / 2u);
    }
    s = (int64_t)(unsigned long long)(S)(ix - 1);
  }
  if (s < 0 || s >= (int64_t)size - 1) return false;
  const int32_t lo_c = ldrow<GLOBAL>(row + s), hi_c = ldrow<GLOBAL>(row + s + 1);
  if constexpr (LK != LK_ALIAS) cum_off -= lo_c;
  freq = (int32_t)((uint32_t)hi_c - (uint32_t)lo_c);
  return true;
}

// the rest of a pop step once the lookup is done: x = D(x), refill, escape (rans_utils.hpp:473-531)
template <int V, bool BYPASS>
__device__ __forceinline__ int32_t pop_finish(const PopParams& P, typename VT<V>::State& x, PopCursor<V>& c,
                                              int32_t s, int32_t cum_off, int32_t freq, int32_t maxv) {
  using S = typename VT<V>::State;
  x = (S)((x >> P.fp) * to_state<S>(freq) + to_state<S>(cum_off));
  c.refill(x);
  int32_t value = s;
  if constexpr (BYPASS) {
    if (value == maxv) {
      const int32_t raw = pop_escape<V>(x, c, P.bp);
      value = raw >> 1;
      value = (raw & 1) ? (-value - 1) : (value + maxv);
    }
  }
  return value;
}

// one symbol straight from the caller's tables.  `ok` is cleared when the step was skipped.
template <int V, int LK, bool BYPASS>
__device__ __forceinline__ int32_t pop_chain(const PopParams& P, typename VT<V>::State& x, PopCursor<V>& c,
                                             int32_t k, const TableInfo& t, bool& ok) {
  using S = typename VT<V>::State;
  ok = false;
  const int32_t* row = P.cdfs + (int64_t)k * P.cdf_width;
  const int32_t cum = (int32_t)(uint32_t)(x & (S)((1ull << P.fp) - 1ull));
  int64_t s;
  int32_t cum_off, freq;
  if (!lookup_symbol<V, LK>(row, t, cum, P.cdf_width, P.fp, s, cum_off, freq)) {
    c.err |= DEV_BAD_VALUE;
    return 0;
  }
  ok = true;
  return pop_finish<V, BYPASS>(P, x, c, (int32_t)s, cum_off, freq, t.size - 2);
}


__device__ __forceinline__ TableInfo tinfo_or_zero(const PopParams& P, int32_t k, bool in_row) {
  if (in_row && k >= 0 && (int64_t)k < P.ntables) return load_tinfo(P.tinfo, k);
  TableInfo t;
  t.size = 0;
  t.offset = 0;
  t.cut = 0;
  t.cut_log2 = -1;
  return t;
}

}  // namespace tans
