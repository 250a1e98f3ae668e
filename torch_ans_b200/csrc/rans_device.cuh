// rans_device.cuh -- device-side building blocks of the B200 rANS engine.
//
// Coder variants (state bits / word bits) follow the three instantiations the reference binds
// (torch_ans/rans.hpp:297-322).  Arithmetic semantics follow torch_ans/rans_utils.hpp:32-71 and
// :168-532: the state is an unsigned 64- or 32-bit integer, the lower bound of the normalisation
// interval is L = 2^(state_bits - 1 - word_bits), a push emits words while
// x >= ((L >> fp) << word_bits) * freq (a single `if` when state_bits-1-word_bits < word_bits), a
// pop refills while x < L, and int32 table values enter the state arithmetic through C's
// int32 -> unsigned conversion (sign extension to 64 bits, then reduction mod 2^state_bits).
//
// The division x / freq of the push is done with an exact multiply-high by a precomputed
// reciprocal (Granlund & Montgomery, "Division by invariant integers using multiplication",
// PLDI 1994, Thm 4.2): for a divisor 2 <= d <= 2^31 with l = ceil(log2 d) and
// m = ceil(2^(N+l) / d) < 2^W, floor(n / d) = mulhi_W(n, m) >> (l - 1) for every n < 2^N, where
// (N, W) = (63, 64) for the 64-bit state and (31, 32) for the 32-bit states.  Proof: m*d =
// 2^(N+l) + e with 0 <= e < d <= 2^l, so n*m / 2^(N+l) = n/d + n*e/(d*2^(N+l)) and the second
// term is < 1/d; since n/d = floor(n/d) + j/d with j <= d-1 the floor is unchanged.  The push
// only divides a renormalised state, which is < freq * 2^(state_bits-1-fp) <= 2^N (or a
// word-shifted state < 2^(state_bits-word_bits)), so the precondition n < 2^N always holds.
// d = 1 is handled by a select (q = n).
#pragma once

#include <cstdint>

namespace tans {

enum : uint32_t {
  DEV_BAD_INDEX = 1u,
  DEV_BAD_VALUE = 2u,
  DEV_OVERFLOW = 4u,
  DEV_UNDERFLOW = 8u,
  DEV_BAD_FREQ = 16u,
  DEV_BAD_ESCAPE = 32u,
};

template <int V> struct Variant;
template <> struct Variant<0> {  // rans64
  using State = unsigned long long;
  using Word = uint32_t;
  static constexpr int SB = 64, WB = 32;
};
template <> struct Variant<1> {  // rans32 (byte words)
  using State = uint32_t;
  using Word = uint8_t;
  static constexpr int SB = 32, WB = 8;
};
template <> struct Variant<2> {  // rans32_16
  using State = uint32_t;
  using Word = uint16_t;
  static constexpr int SB = 32, WB = 16;
};

template <int V> struct VT : Variant<V> {
  using typename Variant<V>::State;
  using typename Variant<V>::Word;
  static constexpr int SB = Variant<V>::SB, WB = Variant<V>::WB;
  static constexpr int USED = SB - 1;
  static constexpr int WBYTES = WB / 8;
  static constexpr int SBYTES = SB / 8;
  static constexpr unsigned long long LB = 1ull << (USED - WB);
  // rans_utils.hpp:45-61: `while` renorm only when USED - WB >= WB (rans32); else a single `if`
  static constexpr bool LOOP = (USED - WB) >= WB;
  // most words one renormalisation can emit / consume (rans32: state < 2^32, bound >= 2^8)
  static constexpr int MAX_RENORM = LOOP ? (SB - 8 + WB - 1) / WB : 1;
};

// int32 -> state type as C converts it in the reference (sign-extend, then reduce)
template <typename S> __device__ __forceinline__ S to_state(int32_t a) {
  return (S)(long long)a;
}

// One encode-table entry: everything the push needs about (table k, symbol v), 16 bytes.
//   x: low 32 bits of the reciprocal, y: high 32 bits (64-bit state only),
//   z: frequency (0 marks an unusable entry: freq <= 0), w: start = cdf[v] (int32 bits)
__device__ __forceinline__ unsigned shift_for(uint32_t d) {  // l - 1, l = ceil(log2 d); 0 for d < 2
  return d > 1u ? 31u - (unsigned)__clz((int)(d - 1u)) : 0u;
}

__device__ __forceinline__ unsigned long long recip64(uint32_t d) {
  // m = ceil(2^(63+l) / d) computed as two 64-bit divisions (2^(63+l) = 2^(31+l) * 2^32)
  const unsigned l = 32u - (unsigned)__clz((int)(d - 1u));
  const unsigned long long A = 1ull << (31 + l);
  const unsigned long long qa = A / d, ra = A % d;
  const unsigned long long hi = ra << 32;
  const unsigned long long qb = hi / d, rb = hi % d;
  return (qa << 32) + qb + (rb != 0 ? 1ull : 0ull);
}

__device__ __forceinline__ uint32_t recip32(uint32_t d) {
  const unsigned l = 32u - (unsigned)__clz((int)(d - 1u));
  const unsigned long long A = 1ull << (31 + l);
  return (uint32_t)((A + d - 1) / d);
}

template <int V>
__device__ __forceinline__ typename VT<V>::State quotient(typename VT<V>::State x, uint4 e) {
  if constexpr (V == 0) {
    const unsigned long long m = ((unsigned long long)e.y << 32) | e.x;
    const unsigned long long q = __umul64hi(x, m) >> shift_for(e.z);
    return e.z == 1u ? x : q;
  } else {
    const uint32_t q = __umulhi(x, e.x) >> shift_for(e.z);
    return e.z == 1u ? x : q;
  }
}

// Per-table information, 16 bytes: cdf_size, offset, alias cut width, log2(cut) or -1.
struct __align__(16) TableInfo {
  int32_t size;
  int32_t offset;
  int32_t cut;
  int32_t cut_log2;
};

__device__ __forceinline__ TableInfo load_tinfo(const TableInfo* t, int64_t k) {
  const int4 v = __ldg(reinterpret_cast<const int4*>(t) + k);
  TableInfo r;
  r.size = v.x;
  r.offset = v.y;
  r.cut = v.z;
  r.cut_log2 = v.w;
  return r;
}

// Stream row helpers.  The payload starts at row + 1 (4-byte aligned).
template <int V>
__device__ __forceinline__ typename VT<V>::State load_state(const int32_t* row, int k) {
  using S = typename VT<V>::State;
  if constexpr (V == 0) {
    const uint32_t lo = (uint32_t)row[1 + 2 * k], hi = (uint32_t)row[2 + 2 * k];
    return ((S)hi << 32) | lo;
  } else {
    return (S)(uint32_t)row[1 + k];
  }
}

template <int V>
__device__ __forceinline__ void store_state(int32_t* row, int k, typename VT<V>::State x) {
  if constexpr (V == 0) {
    row[1 + 2 * k] = (int32_t)(uint32_t)x;
    row[2 + 2 * k] = (int32_t)(uint32_t)(x >> 32);
  } else {
    row[1 + k] = (int32_t)x;
  }
}

__device__ __forceinline__ void report(uint32_t* status, uint32_t err) {
  if (err && status) atomicOr(status, err);
}

// ---------------------------------------------------------------- async copies and L2 policy
// LDGSTS (cp.async) copies global -> shared without passing through registers, so a load issued
// several chunks ahead of its use never stalls the issuing thread.  src_bytes < cp-size
// zero-fills the rest (src_bytes = 0 reads nothing).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async16_hint(void* smem, const void* gmem, unsigned long long policy) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "l"(policy)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// L2 eviction policies: tables that every step reads stay (evict_last); data read or written
// once goes first (evict_first), so streaming rows do not push the tables out of L2.
__device__ __forceinline__ unsigned long long policy_evict_last() {
  unsigned long long p;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
__device__ __forceinline__ unsigned long long policy_evict_first() {
  unsigned long long p;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
// (not volatile: these read data that no thread writes during the kernel, so the compiler may
// hoist and interleave them like ordinary loads -- the independent chains of a thread then keep
// several table loads in flight at once)
__device__ __forceinline__ uint32_t ld_hint_u32(const uint32_t* p, unsigned long long policy) {
  uint32_t v;
  asm("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;\n" : "=r"(v) : "l"(p), "l"(policy));
  return v;
}
__device__ __forceinline__ uint32_t ld_hint_u16(const uint16_t* p, unsigned long long policy) {
  unsigned short v;
  asm("ld.global.nc.L2::cache_hint.u16 %0, [%1], %2;\n" : "=h"(v) : "l"(p), "l"(policy));
  return v;
}
__device__ __forceinline__ unsigned long long ld_hint_u64(const unsigned long long* p, unsigned long long policy) {
  unsigned long long v;
  asm("ld.global.nc.L2::cache_hint.u64 %0, [%1], %2;\n" : "=l"(v) : "l"(p), "l"(policy));
  return v;
}
__device__ __forceinline__ void st_hint_v4(int4* p, int4 v, unsigned long long policy) {
  asm volatile("st.global.L2::cache_hint.v4.s32 [%0], {%1, %2, %3, %4}, %5;\n" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w), "l"(policy)
               : "memory");
}

}  // namespace tans
