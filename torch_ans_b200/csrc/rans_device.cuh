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
// PLDI 1994, Thm 4.2): for a divisor 1 <= d <= 2^31 with l = ceil(log2 d) and
// m = ceil(2^(N+l) / d) <= 2^W, floor(n / d) = floor(n * m / 2^(N+l)) for every n < 2^N, where
// (N, W) = (63, 64) for the 64-bit state and (31, 32) for the 32-bit states.  Proof: m*d =
// 2^(N+l) + e with 0 <= e < d <= 2^l, so n*m / 2^(N+l) = n/d + n*e/(d*2^(N+l)) and the second
// term is < 1/d; since n/d = floor(n/d) + j/d with j <= d-1 the floor is unchanged.  m fits in
// W bits (m < 2^W for d >= 3, m = 2^N for d = 1 and 2), and floor(n*m / 2^(N+l)) =
// mulhi_W(2n, m) >> l, so one form covers every divisor.  The fast push steps divide only a
// renormalised state of a step with freq <= 2^fp, which is < freq * 2^(state_bits-1-fp) <= 2^N,
// so the precondition n < 2^N holds there; the exact step code uses quotient_exact below.
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
  DEV_STALLED = 64u,  // a bounded wait between the warps of a block ran out; the rows are not valid
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
//   x, y: the reciprocal m = ceil(2^(N+l) / freq) (y = high word, 64-bit state only), with
//         l = ceil(log2 freq) and N = 63 (64-bit state) or 31 (32-bit states);
//   z:    freq, and when fp <= 23 also l in bits 24..28 (freq < 2^24 then);
//   w:    start = cdf[v] (int32 bits).
// z = 0 marks an unusable entry (freq <= 0).  Quotient: floor(x / freq) = mulhi(2x, m) >> l for
// every freq >= 1 and x < 2^N (the GM bound above, with 2x absorbing the one-bit shift; for
// freq = 1, l = 0 and m = 2^N give floor(2x * 2^N / 2^(N+1)) = x), so there is no special case.
// The fast steps of the push kernels take only entries with 1 <= freq <= 2^fp: there the
// renormalised state is below bound = freq << (N - fp) <= 2^N.  Any other step runs push_chain,
// which divides with quotient_exact.
__device__ __forceinline__ unsigned ceil_log2(uint32_t d) {  // 0 for d <= 1
  return d > 1u ? 32u - (unsigned)__clz((int)(d - 1u)) : 0u;
}

__device__ __forceinline__ unsigned long long recip64(uint32_t d) {
  // m = ceil(2^(63+l) / d) as two 64-bit divisions (2^(63+l) = 2^(31+l) * 2^32); d = 1 -> 2^63
  const unsigned l = ceil_log2(d);
  const unsigned long long A = 1ull << (31 + l);
  const unsigned long long qa = A / d, ra = A % d;
  const unsigned long long hi = ra << 32;
  const unsigned long long qb = hi / d, rb = hi % d;
  return (qa << 32) + qb + (rb != 0 ? 1ull : 0ull);
}

__device__ __forceinline__ uint32_t recip32(uint32_t d) {  // ceil(2^(31+l) / d); d = 1 -> 2^31
  const unsigned l = ceil_log2(d);
  const unsigned long long A = 1ull << (31 + l);
  return (uint32_t)((A + d - 1) / d);
}

// freq and l of an entry (l packed when the caller's fp <= 23)
__device__ __forceinline__ uint32_t entry_freq(uint4 e, bool packed) { return packed ? (e.z & 0xFFFFFFu) : e.z; }
__device__ __forceinline__ unsigned entry_shift(uint4 e, bool packed) { return packed ? (e.z >> 24) : ceil_log2(e.z); }

template <int V>
__device__ __forceinline__ typename VT<V>::State quotient(typename VT<V>::State x, uint4 e, bool packed) {
  const unsigned l = entry_shift(e, packed);
  if constexpr (V == 0) {
    const unsigned long long m = ((unsigned long long)e.y << 32) | e.x;
    return __umul64hi(x << 1, m) >> l;
  } else {
    return __umulhi(x << 1, e.x) >> l;
  }
}

// floor(x / freq) for every state x (quotient() needs x < 2^N).  A state of 2^N or more reaches
// the division only after a step whose frequency exceeds 2^fp (bound = freq << (N - fp) > 2^N):
// no quantised cdf has one, but the reference divides exactly there too.  With l >= 1,
// mulhi(x, m) >> (l - 1) = floor(x * m / 2^(N+l)) is floor(x / freq) or one more (m * freq =
// 2^(N+l) + e with e < freq, so the excess x * e / (freq * 2^(N+l)) is below 2^(1-l) <= 1): one
// downward correction.  l = 0 is freq = 1.
template <int V>
__device__ __forceinline__ typename VT<V>::State quotient_exact(typename VT<V>::State x, uint4 e, bool packed,
                                                                uint32_t freq) {
  using S = typename VT<V>::State;
  const unsigned l = entry_shift(e, packed);
  if (l == 0u) return x;
  S q;
  if constexpr (V == 0) {
    const unsigned long long m = ((unsigned long long)e.y << 32) | e.x;
    q = __umul64hi(x, m) >> (l - 1u);
    if (__umul64hi(q, (unsigned long long)freq) != 0ull || q * (unsigned long long)freq > x) --q;
  } else {
    q = __umulhi(x, e.x) >> (l - 1u);
    if ((unsigned long long)q * freq > (unsigned long long)x) --q;
  }
  return q;
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
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem) : "memory");
}
// *p = v when c holds, as one predicated store (no branch around it); p addresses global memory
template <typename W> __device__ __forceinline__ void st_global_if(W* p, uint32_t v, bool c);
template <> __device__ __forceinline__ void st_global_if<uint8_t>(uint8_t* p, uint32_t v, bool c) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.u8 [%0], %1;\n}\n" ::"l"(p), "r"(v),
               "r"((int)c)
               : "memory");
}
template <> __device__ __forceinline__ void st_global_if<uint16_t>(uint16_t* p, uint32_t v, bool c) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.u16 [%0], %1;\n}\n" ::"l"(p), "r"(v),
               "r"((int)c)
               : "memory");
}
template <> __device__ __forceinline__ void st_global_if<uint32_t>(uint32_t* p, uint32_t v, bool c) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.u32 [%0], %1;\n}\n" ::"l"(p), "r"(v),
               "r"((int)c)
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

// ---------------------------------------------------------------- shared-memory barriers
// mbarrier objects (8 bytes of shared memory each) hand ring slots between the warps of a block.
// A phase completes when its expected arrivals are in; waiters name the phase by its parity.
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(unsigned long long* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
// arrive with release semantics: this thread's earlier shared-memory writes (and reads) are
// ordered before the phase completes
__device__ __forceinline__ void mbar_arrive(unsigned long long* b) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(b)) : "memory");
}
// arrive once every cp.async this thread issued so far has landed (counts as one of the
// expected arrivals)
__device__ __forceinline__ void mbar_arrive_cp_async(unsigned long long* b) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0u;
}
// Warp-uniform bounded wait (call with the whole warp converged).  Gives up after `limit` tries
// (each try_wait may suspend the warp for a short while) or as soon as another warp of the block
// has given up (*abort != 0); returns whether the phase completed.
__device__ __forceinline__ bool warp_wait(unsigned long long* b, unsigned parity, volatile int* abort,
                                          unsigned limit) {
  for (unsigned it = 0; it < limit; ++it) {
    const bool done = mbar_try_wait(b, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    if (__any_sync(0xffffffffu, *abort != 0)) return false;
  }
  return false;
}

// ---------------------------------------------------------------- TMA bulk copies (1D)
// fence that makes a freshly initialised mbarrier visible to the asynchronous (TMA) proxy
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
// one arrival that also announces `bytes` of TMA transactions the phase must wait for
__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
// global -> shared bulk copy by the copy engine (both addresses 16-byte aligned, size a multiple of
// 16); its bytes count against the mbarrier's transaction count.  The copy lands in this CTA only.
__device__ __forceinline__ void bulk_copy_g2s(void* smem, const void* gmem, unsigned bytes, unsigned long long* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(smem)),
               "l"(gmem), "r"(bytes), "r"(smem_u32(b))
               : "memory");
}

// orders this thread's earlier generic-proxy accesses of shared memory before its later
// async-proxy (bulk copy) accesses: needed before a bulk copy overwrites data the thread read
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
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
