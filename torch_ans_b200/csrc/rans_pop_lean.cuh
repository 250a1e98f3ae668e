// rans_pop_lean.cuh -- single-state pops with the shortest serial step, one thread per stream
// (rows 16-byte aligned, length % 4 == 0).
//
// A pop is one serial chain per stream (rans_utils.hpp:379-532 per symbol); with one thread per
// stream, its speed is the latency of one step.  Two kernels:
//   pop_lean_kernel   the split and fused layouts: cum -> table load(s) -> (symbol, start, freq)
//                     -> x = freq * (x >> fp) + cum - start -> refill with the word prefetched
//                     into a register; table indexes arrive four chunks ahead, offsets and escape
//                     slots come from shared memory, four symbols leave as one 16-byte store;
//   pop_bucket_kernel the bucket layout (and its level-1 table in shared memory), described above
//                     the kernel.
// Steps the straight-line code cannot do exactly (an index outside the table list, a table entry
// marked as not describable, an escape, a row whose length points outside it) take the
// reference-exact step out of line on their own lane; a word outside the row reads as 0 and sets
// TANS_DEV_UNDERFLOW, as the exact step does.
//
// Table layouts are those of the fast kernel (built per call by replaying the reference lookup).
#pragma once

#include "rans_pop_fast.cuh"

namespace tans {

// state of one stream that the rare exact step reads and writes (passed by value both ways, so the
// kernel never takes the address of its state and keeps it in registers); the kernel parameters
// are __grid_constant__, so the out-of-line steps read them through a reference into the
// parameter space instead of a copy on the stack
template <int V> struct LeanState {
  typename VT<V>::State x, nextw;
  long long p;
  uint32_t err;
  int32_t v;  // decoded symbol (output of the exact step)
};

// the reference-exact step of one symbol, out of line (rare path); refreshes the prefetched word
template <int V, int LK, bool BYPASS, int TM>
__device__ __noinline__ LeanState<V> popl_exact(const PopParams& P, LeanState<V> st, const int32_t* row, int32_t k,
                                                const TableInfo* tsm, const uint32_t* tD, const uint16_t* tS) {
  FastCursor<V> cur;
  cur.c.payload = reinterpret_cast<const uint8_t*>(row + 1);
  cur.c.p = st.p;
  cur.c.first = VT<V>::SBYTES / VT<V>::WBYTES;
  cur.c.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
  cur.c.err = st.err;
  cur.nextw = st.nextw;
  typename VT<V>::State x = st.x;
  st.v = popf_exact<V, LK, BYPASS, TM>(P, x, cur, k, tsm, tD, tS, policy_evict_last());
  cur.prime();
  st.x = x;
  st.nextw = cur.nextw;
  st.p = cur.c.p;
  st.err = cur.c.err;
  return st;
}

__device__ __forceinline__ int4 ld_idx4(const int32_t* p, unsigned long long policy) {
  int4 v;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.s32 {%0, %1, %2, %3}, [%4], %5;\n"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(policy));
  return v;
}

template <int V, int LK, bool BYPASS, int TM>
__global__ void __launch_bounds__(512) pop_lean_kernel(const __grid_constant__ PopParams P) {
  using S = typename VT<V>::State;
  using W = typename VT<V>::Word;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  const int warps = T >> 5, warp = tid >> 5, lane = tid & 31;
  TableInfo* tsm = reinterpret_cast<TableInfo*>(smem_raw);
  int2* tsm2 = reinterpret_cast<int2*>(tsm + P.ntables);  // {offset, escape slot} per table
  unsigned char* tab = popf_align16(tsm2 + P.ntables);
  const int64_t M = (int64_t)1 << P.fp;
  const int64_t m = P.ntables << P.fp;
  uint32_t* tD = reinterpret_cast<uint32_t*>(tab);  // fused: D; split: ST
  uint16_t* tS = reinterpret_cast<uint16_t*>(
      tab + (((TM == TM_FUSED_SMEM ? m * 4 : (TM == TM_SPLIT_SMEM ? P.ntables * P.st_stride * 4 : 0)) + 15) &
             ~(int64_t)15));
  __shared__ unsigned long long stage_bar;
  __shared__ int stage_tma;
  popf_stage_begin<TM>(P, tD, tS, m, &stage_bar, &stage_tma);  // the copy engine runs while the records fill
  for (int64_t k = tid; k < P.ntables; k += T) {
    const TableInfo ti = P.tinfo[k];
    tsm[k] = ti;
    tsm2[k] = make_int2(ti.offset, BYPASS ? ti.size - 2 : -1);
  }
  const bool staged = __syncthreads_and(popf_stage_end<TM>(&stage_bar, &stage_tma) ? 1 : 0) != 0;
  if (!staged) {
    popf_stage_drain<TM>(&stage_bar, &stage_tma, P.status);
    return;
  }
  if (lane >= P.lanes) return;
  const int64_t b = ((int64_t)blockIdx.x * warps + warp) * P.lanes + lane;
  if (b >= P.batch) return;

  int32_t* row = P.stream + b * P.width;
  FastCursor<V> cur;
  cur.c.payload = reinterpret_cast<const uint8_t*>(row + 1);
  cur.c.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
  cur.c.first = VT<V>::SBYTES / VT<V>::WBYTES;
  cur.c.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
  cur.c.err = 0;
  S x = load_state<V>(row, 0);
  cur.prime();
  const W* pw = reinterpret_cast<const W*>(cur.c.payload);
  // a row whose length points past its end, or past what 32-bit cursors hold, is decoded exactly
  const bool row_bad = cur.c.p >= cur.c.cap || cur.c.p > 0x7ffffff0;
  const int first = (int)cur.c.first;
  const int capw = (int)min(cur.c.cap, (int64_t)0x7fffffff);
  int p = (int)min(max(cur.c.p, (int64_t)-0x7fffffff), (int64_t)0x7fffffff);
  S nextw = cur.nextw;
  uint32_t err = 0;

  const unsigned long long pol_keep = policy_evict_last(), pol_stream = policy_evict_first();
  const uint32_t cmask = (uint32_t)(M - 1);
  const uint32_t kmax = (uint32_t)(P.ntables - 1);
  const int64_t N = P.nsym;
  const int nch = (int)(N >> 2);
  const int32_t* irow = P.idx + b * N;
  // table indexes four chunks (16 steps) ahead of their use: several microseconds even when few
  // streams share an SM and steps are short
  int4 kn0 = nch > 0 ? ld_idx4(irow, pol_stream) : make_int4(0, 0, 0, 0);
  int4 kn1 = nch > 1 ? ld_idx4(irow + 4, pol_stream) : make_int4(0, 0, 0, 0);
  int4 kn2 = nch > 2 ? ld_idx4(irow + 8, pol_stream) : make_int4(0, 0, 0, 0);
  int4 kn3 = nch > 3 ? ld_idx4(irow + 12, pol_stream) : make_int4(0, 0, 0, 0);

#pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    const int4 k4 = kn0;
    kn0 = kn1;
    kn1 = kn2;
    kn2 = kn3;
    if (c + 4 < nch) kn3 = ld_idx4(irow + 4 * (int64_t)(c + 4), pol_stream);
    const int32_t kv[4] = {k4.x, k4.y, k4.z, k4.w};
    int32_t ov[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int32_t k = kv[q];
      const uint32_t kc = min((uint32_t)k, kmax);
      const int2 om = tsm2[kc];
      const uint32_t cum = (uint32_t)x & cmask;
      uint32_t sv, fm1, off;
      bool slow = row_bad || (uint32_t)k > kmax;
      if constexpr (TM == TM_FUSED_SMEM || TM == TM_FUSED_GLOBAL) {
        const size_t e = ((size_t)kc << P.fp) | cum;
        uint32_t d;
        if constexpr (TM == TM_FUSED_SMEM) {
          d = tD[e];
          sv = tS[e];
        } else {
          d = ld_hint_u32(P.fD + e, pol_keep);
          sv = ld_hint_u16(P.fS + e, pol_keep);
        }
        slow |= sv == 0xFFFFu;
        fm1 = d & 0xFFFFu;
        off = d >> 16;
      } else {  // split layouts: S[k][cum], then ST[k][s] = (freq - 1) | start << 16
        const size_t e = ((size_t)kc << P.fp) | cum;
        uint32_t st;
        if constexpr (TM == TM_SPLIT_SMEM) {
          sv = tS[e];
          st = tD[(size_t)kc * P.st_stride + min(sv, (uint32_t)(P.st_stride - 1))];
        } else {
          sv = ld_hint_u16(P.fS + e, pol_keep);
          st = ld_hint_u32(P.fST + (size_t)kc * P.st_stride + min(sv, (uint32_t)(P.st_stride - 1)), pol_keep);
        }
        slow |= sv == 0xFFFFu;
        fm1 = st & 0xFFFFu;
        off = cum - (st >> 16);
      }
      if constexpr (BYPASS) slow |= (int32_t)sv == om.y;
      if (slow) {
        LeanState<V> st{x, nextw, (long long)p, err, 0};
        st = popl_exact<V, LK, BYPASS, TM>(P, st, row, k, tsm, tD, tS);
        x = st.x;
        nextw = st.nextw;
        p = (int)min(max(st.p, -0x7fffffffll), 0x7fffffffll);
        err = st.err;
        ov[q] = st.v;
        continue;
      }
      x = (S)((x >> P.fp) * (S)(fm1 + 1u) + (S)off);
      // refill (rans_utils.hpp RANS_POP_STATE_RENORM): the first word is already in a register; a
      // word outside the row's data reads as 0 and flags underflow, as in the exact step
      {
        const bool r = (unsigned long long)x < VT<V>::LB;
        const int pc = p;
        if (r && (pc < first || pc >= capw)) err |= DEV_UNDERFLOW;
        x = r ? (S)((x << VT<V>::WB) | nextw) : x;
        p = pc - (r ? 1 : 0);
        if (r) nextw = (p >= first && p < capw) ? (S)__ldg(pw + p) : (S)0;
      }
      if constexpr (VT<V>::LOOP) {
#pragma unroll
        for (int t = 1; t < VT<V>::MAX_RENORM; ++t) {
          if ((unsigned long long)x < VT<V>::LB) {
            if (p < first || p >= capw) err |= DEV_UNDERFLOW;
            x = (S)((x << VT<V>::WB) | nextw);
            p -= 1;
            nextw = (p >= first && p < capw) ? (S)__ldg(pw + p) : (S)0;
          }
        }
      }
      ov[q] = (int32_t)(sv + (uint32_t)om.x);
    }
    int32_t* o = P.out + b * N + 4 * (int64_t)c;
    st_hint_v4(reinterpret_cast<int4*>(o), make_int4(ov[0], ov[1], ov[2], ov[3]), pol_stream);
  }
  store_state<V>(row, 0, x);
  row[0] = (int32_t)((int64_t)(p + 1) * VT<V>::WBYTES);
  report(P.status, err);
}

// The rare step of the bucket pop, out of line with the state passed by value: marker entries of
// type 1 (unit-frequency run: symbol = cum + d, freq 1, offset 0) and type 2 (one load from the
// secondary table's per-cum block) decode here with the same update and refill as the straight
// step; everything else (type-0 markers, bad indexes, escapes) takes the exact step.
template <int V, int LK, bool BYPASS>
__device__ __noinline__ LeanState<V> popb_rare(const PopParams& P, LeanState<V> st, const int32_t* row, int32_t k,
                                               unsigned long long e, const TableInfo* tsm) {
  using S = typename VT<V>::State;
  const uint32_t kind = (uint32_t)(e >> 16) & 3u;
  if ((e & 0xFFFFull) == 0xFFFFull && (kind == 1u || kind == 2u) && (uint32_t)k < (uint64_t)P.ntables) {
    const uint32_t cum = (uint32_t)st.x & ((1u << P.fp) - 1u);
    uint32_t f, off;
    int32_t sv;
    if (kind == 1u) {
      f = 1u;
      off = 0u;
      sv = (int32_t)(cum + (uint32_t)(e >> 32));
    } else {
      const unsigned long long d =
          ld_hint_u64(P.fSEC + ((e >> 18) << kBucketBits) + (cum & ((1u << kBucketBits) - 1u)), policy_evict_last());
      sv = (int32_t)(d & 0xFFFFull);
      off = (uint32_t)(d >> 16) & 0xFFFFu;
      f = (uint32_t)(d >> 32);
    }
    const TableInfo ti = tsm[k];
    if (!BYPASS || sv != ti.size - 2) {
      FastCursor<V> cur;
      cur.c.payload = reinterpret_cast<const uint8_t*>(row + 1);
      cur.c.p = st.p;
      cur.c.first = VT<V>::SBYTES / VT<V>::WBYTES;
      cur.c.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
      cur.c.err = st.err;
      cur.nextw = st.nextw;
      S x = st.x;
      x = (S)((x >> P.fp) * (S)f + (S)off);
      cur.refill(x);
      if constexpr (VT<V>::LOOP) cur.prime();
      st.x = x;
      st.nextw = cur.nextw;
      st.p = cur.c.p;
      st.err = cur.c.err;
      st.v = (int32_t)((uint32_t)sv + (uint32_t)ti.offset);
      return st;
    }
  }
  return popl_exact<V, LK, BYPASS, TM_BUCKET_GLOBAL>(P, st, row, k, tsm, nullptr, nullptr);
}

// Bucket entry at address `a`; volatile, so the compiler keeps it where it is written (ahead of
// the rare-step branch) instead of moving it into the branch's fall-through path
__device__ __forceinline__ unsigned long long ld_entry(uintptr_t a, unsigned long long policy) {
  unsigned long long v;
  asm volatile("ld.global.nc.L2::cache_hint.u64 %0, [%1], %2;\n" : "=l"(v) : "l"(a), "l"(policy));
  return v;
}
// the same from a 32-bit shared-memory address (the level-1 table)
__device__ __forceinline__ unsigned long long ld_entry_shared(uint32_t a) {
  unsigned long long v;
  asm volatile("ld.shared.u64 %0, [%1];\n" : "=l"(v) : "r"(a));
  return v;
}
// the fused layout's two entries of index i (D: (freq - 1) | offset << 16, S: the symbol) from
// shared memory, as D | S << 32
__device__ __forceinline__ unsigned long long ld_fused_shared(uint32_t dbase, uint32_t sbase, uint32_t i) {
  uint32_t d, s;
  asm volatile("ld.shared.u32 %0, [%2];\n ld.shared.u16 %1, [%3];\n"
               : "=r"(d), "=r"(s)
               : "r"(dbase + 4u * i), "r"(sbase + 2u * i));
  return (unsigned long long)d | ((unsigned long long)s << 32);
}

// Stream word at p when `pred`, else `w` (a predicated load, zero-extended: no branch on the
// serial step)
__device__ __forceinline__ uint32_t ld_word_if(const uint32_t* p, bool pred, uint32_t w) {
  asm("{\n .reg .pred q;\n setp.ne.u32 q, %2, 0;\n @q ld.global.nc.u32 %0, [%1];\n}\n"
      : "+r"(w)
      : "l"(p), "r"((uint32_t)pred));
  return w;
}
__device__ __forceinline__ uint32_t ld_word_if(const uint16_t* p, bool pred, uint32_t w) {
  asm("{\n .reg .pred q;\n setp.ne.u32 q, %2, 0;\n @q ld.global.nc.u16 %0, [%1];\n}\n"
      : "+r"(w)
      : "l"(p), "r"((uint32_t)pred));
  return w;
}
__device__ __forceinline__ uint32_t ld_word_if(const uint8_t* p, bool pred, uint32_t w) {
  asm("{\n .reg .pred q;\n setp.ne.u32 q, %2, 0;\n @q ld.global.nc.u8 %0, [%1];\n}\n"
      : "+r"(w)
      : "l"(p), "r"((uint32_t)pred));
  return w;
}

// Pop over the bucket layout (TM_BUCKET_GLOBAL): one dependent L2 load per step, or with L1 one
// dependent shared-memory load (the level-1 table: the same entry format over 256 cum values,
// copied into each block; its markers read the 16-cum entry from L2 in the rare branch, then the
// rare step if that is a marker too).  L1 is chosen for at most two streams per SM, where every
// stream has its own warp and a level-1 miss delays only its own lane.
//
// Entry of 16 cum values (built per call, every cum checked against the reference lookup):
//   lo = s0 | (c1 - 1) << 16,  hi = f0 | f1 << 16
// (s0 the symbol of the bucket's first cum, f0 its freq, c1 the start of s0 + 1, f1 its freq;
// s0 = 0xFFFF marks a bucket the entry cannot describe, which the out-of-line rare step decodes:
// unit-frequency runs with no load, other buckets from a per-cum block in one more load, the
// remaining cases by the exact step).  The serial chain of a step is
//   entry load -> up = (cum << 16) > lo, one compare on the loaded word -> freq = up ? f1 : f0,
//   offset = cum - c1 + (up ? 0 : f0) -> x = freq * (x >> fp) + offset -> refill test ->
//   next entry address -> next entry load (issued before the step's rare-step branch, so the
//   branch resolves in the load's shadow; the rare step reissues it),
// where the next address is a select between the two candidates computed beside the refill test
// (refill: the low word becomes the prefetched stream word; else the low word of the product),
// each a row address OR-ed with (low word >> 1) & mask: rows are aligned to their size, so the OR
// is the add.  A row of markers after the last table stands for table indexes outside the table
// list, so the marker test is the step's only check.  Off the chain: symbol output and table
// offsets (read once per chunk, only when some table has a non-zero offset or escapes are coded),
// index loads two chunks ahead, the predicated prefetch of the next stream word,
// and the underflow test, made once at the end of the stream (a refill read below the first data
// word happened exactly when the cursor fell below first - 1).
// table modes of pop_bucket_kernel
enum : int { BM_L2 = 0, BM_L1 = 1, BM_FUSED = 2 };

template <int V, int LK, bool BYPASS, int MODE, bool IRING>
__global__ void __maxnreg__(96) pop_bucket_kernel(const __grid_constant__ PopParams P) {
  using S = typename VT<V>::State;
  using W = typename VT<V>::Word;
  constexpr bool L1 = MODE == BM_L1;
  constexpr bool FUSED = MODE == BM_FUSED;
  constexpr int TM = FUSED ? TM_FUSED_SMEM : TM_BUCKET_GLOBAL;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  const int warps = T >> 5, warp = tid >> 5, lane = tid & 31;
  // per-table records: TableInfo, then {offset, escape slot} with one more entry for the marker
  // row (the shared region holds 32 bytes per table, these use 24 + 8)
  TableInfo* tsm = reinterpret_cast<TableInfo*>(smem_raw);
  int2* tsm2 = reinterpret_cast<int2*>(tsm + P.ntables);
  // level-1 table (L1): one entry per 2^P.l1_bits cum values, copied in by the whole block; or
  // (FUSED) the fused D and S tables of every table, staged by bulk copies
  unsigned char* l1s = popf_align16(smem_raw + P.ntables * 32);
  const int64_t m = P.ntables << P.fp;
  uint32_t* tD = reinterpret_cast<uint32_t*>(l1s);
  uint16_t* tS = reinterpret_cast<uint16_t*>(l1s + ((m * 4 + 15) & ~(int64_t)15));
  __shared__ unsigned long long stage_bar;
  __shared__ int stage_tma;
  if constexpr (FUSED) popf_stage_begin<TM_FUSED_SMEM>(P, tD, tS, m, &stage_bar, &stage_tma);
  if constexpr (L1) {
    const uint4* src = reinterpret_cast<const uint4*>(P.fL1);
    uint4* dst = reinterpret_cast<uint4*>(l1s);
    const int64_t n16 = P.l1_bytes >> 4;
#pragma unroll 4
    for (int64_t i = tid; i < n16; i += T) dst[i] = __ldg(src + i);
  }
  int any_off = 0;
  for (int64_t k = tid; k < P.ntables; k += T) {
    const TableInfo ti = P.tinfo[k];
    tsm[k] = ti;
    tsm2[k] = make_int2(ti.offset, BYPASS ? ti.size - 2 : -1);
    any_off |= ti.offset != 0 ? 1 : 0;
  }
  if (tid == 0) tsm2[P.ntables] = make_int2(0, -1);
  bool staged = true;
  if constexpr (FUSED) staged = __syncthreads_and(popf_stage_end<TM_FUSED_SMEM>(&stage_bar, &stage_tma) ? 1 : 0) != 0;
  const bool use_off = __syncthreads_or(any_off) != 0;
  if (!staged) {
    popf_stage_drain<TM_FUSED_SMEM>(&stage_bar, &stage_tma, P.status);
    return;
  }
  if (lane >= P.lanes) return;
  const int64_t b = ((int64_t)blockIdx.x * warps + warp) * P.lanes + lane;
  if (b >= P.batch) return;

  int32_t* row = P.stream + b * P.width;
  FastCursor<V> cur;
  cur.c.payload = reinterpret_cast<const uint8_t*>(row + 1);
  cur.c.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
  cur.c.first = VT<V>::SBYTES / VT<V>::WBYTES;
  cur.c.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
  cur.c.err = 0;
  S x = load_state<V>(row, 0);
  cur.prime();
  const W* pw = reinterpret_cast<const W*>(cur.c.payload);
  // a row whose length points past its end, or past what 32-bit cursors hold, is decoded exactly
  const bool row_bad = cur.c.p >= cur.c.cap || cur.c.p > 0x7ffffff0;
  const int first = (int)cur.c.first;
  int p = (int)min(max(cur.c.p, (int64_t)-0x7fffffff), (int64_t)0x7fffffff);
  const int p_init = p;
  uint32_t nextw = (uint32_t)cur.nextw;  // every word type fits 32 bits
  uint32_t err = 0;

  const unsigned long long pol_keep = policy_evict_last(), pol_stream = policy_evict_first();
  const uint32_t cmask = (1u << P.fp) - 1u;
  const uint32_t bmask = (cmask >> 1) & ~7u;  // byte offset of cum's entry in its row, from (cum >> 1)
  const uint32_t kmark = (uint32_t)P.ntables;
  const uint32_t rowbytes = 1u << (P.fp - 1);
  const uintptr_t bk0 = reinterpret_cast<uintptr_t>(P.fBK);
  // entry addresses: the bucket table's row of table k, or with L1 the level-1 row in shared
  // memory (a 32-bit shared address), plus the entry's byte offset taken from the state's low word
  const uint32_t l1base = smem_u32(l1s);
  const uint32_t l1rowbytes = 8u << (P.fp - P.l1_bits);
  const uint32_t l1mask = (cmask >> P.l1_bits) << 3;
  const uint32_t l1shift = (uint32_t)P.l1_bits - 3u;
  // FUSED: entry index (k << fp) | cum into the shared D and S tables; a table index outside the
  // list reads table 0 and is flagged separately (the fused tables have no marker row)
  const uint32_t fdbase = smem_u32(tD), fsbase = smem_u32(tS);
  const uint32_t klast = (uint32_t)(P.ntables - 1);
  auto row_of = [&](int32_t k) -> uintptr_t {
    if constexpr (L1) return (uintptr_t)(l1base + min((uint32_t)k, kmark) * l1rowbytes);
    else if constexpr (FUSED) return (uintptr_t)(((uint32_t)k <= klast ? (uint32_t)k : 0u) << P.fp);
    else return bk0 + (uintptr_t)min((uint32_t)k, kmark) * rowbytes;
  };
  auto addr_of = [&](uintptr_t rowp, uint32_t lowword) -> uintptr_t {
    if constexpr (L1) return rowp + ((lowword >> l1shift) & l1mask);
    else if constexpr (FUSED) return rowp + (lowword & cmask);
    else return rowp | ((lowword >> 1) & bmask);
  };
  auto load_at = [&](uintptr_t at) -> unsigned long long {
    if constexpr (L1) return ld_entry_shared((uint32_t)at);
    else if constexpr (FUSED) return ld_fused_shared(fdbase, fsbase, (uint32_t)at);
    else return ld_entry(at, pol_keep);
  };
  const int64_t N = P.nsym;
  const int nch = (int)(N >> 2);
  const int32_t* irow = P.idx + b * N;
  int32_t* orow = P.out + b * N;

  if (row_bad) {
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      int32_t ov[4];
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        LeanState<V> st{x, (S)nextw, (long long)p, err, 0};
        st = popl_exact<V, LK, BYPASS, TM>(P, st, row, irow[4 * (int64_t)c + q], tsm, tD, tS);
        x = st.x;
        nextw = (uint32_t)st.nextw;
        p = (int)min(max(st.p, -0x7fffffffll), 0x7fffffffll);
        err = st.err;
        ov[q] = st.v;
      }
      st_hint_v4(reinterpret_cast<int4*>(orow + 4 * (int64_t)c), make_int4(ov[0], ov[1], ov[2], ov[3]), pol_stream);
    }
  } else {
    // indexes two chunks (eight steps) ahead: kn0 holds chunk c + 1, kn1 chunk c + 2 (the copy
    // kn0 = kn1 reads a load issued a whole chunk earlier).
    // IRING: the indexes come from shared memory instead.  This lane keeps its stream's indexes in
    // a two-half ring of kRingChunks-chunk tiles; a half is filled by one 1D bulk copy (copy
    // engine, completing on the half's mbarrier) issued a whole half ahead of its first read.
    // Measured on this path: an index load through the load pipeline delays the table-entry loads
    // behind it by ~40 cycles per step; the ring's reads are shared-memory loads.
    int4* ring = nullptr;
    unsigned long long* ibar = nullptr;
    uint32_t wpar = 0;  // bit h: parity of the next phase of half h
    uint32_t pend = 0;  // bit h: a copy into half h is in flight
    auto ring_issue = [&](int h, int start) {
      const int n = min(kRingChunks, nch - start);
      if (n > 0) {
        mbar_arrive_expect_tx(ibar + h, (unsigned)n * 16u);
        bulk_copy_g2s(ring + h * kRingChunks, irow + 4 * (int64_t)start, (unsigned)n * 16u, ibar + h);
        pend |= 1u << h;
      }
    };
    auto ring_wait = [&](int h) -> bool {
      const unsigned par = (wpar >> h) & 1u;
      for (unsigned it = 0; it < kRingWaitLimit; ++it)
        if (mbar_try_wait(ibar + h, par)) {
          wpar ^= 1u << h;
          pend &= ~(1u << h);
          return true;
        }
      err |= DEV_STALLED;
      return false;
    };
    bool dead = false;  // a ring wait ran out: the stream stops
    if constexpr (IRING) {
      const int sl = warp * P.lanes + lane, nsl = warps * P.lanes;
      ring = reinterpret_cast<int4*>(smem_raw + P.iring_off + (size_t)sl * kRingStride);
      ibar = reinterpret_cast<unsigned long long*>(smem_raw + P.iring_off + (size_t)nsl * kRingStride) + 2 * sl;
      mbar_init(ibar, 1u);
      mbar_init(ibar + 1, 1u);
      mbar_init_fence();
      ring_issue(0, 0);
      ring_issue(1, kRingChunks);
      if (pend & 1u) dead = !ring_wait(0);  // nothing was issued for an empty row
    }
    int4 kn0 = make_int4(0, 0, 0, 0), kn1 = make_int4(0, 0, 0, 0);
    if constexpr (IRING) {
      kn0 = ring[0];
      kn1 = ring[1];
    } else {
      if (nch > 0) kn0 = ld_idx4(irow, pol_stream);
      if (nch > 1) kn1 = ld_idx4(irow + 4, pol_stream);
    }
    uintptr_t a = addr_of(row_of(kn0.x), (uint32_t)x);
    // the entry of the next step: each step issues the next step's load before its own rare-step
    // branch, so the branch resolves while the load is in flight (the rare step reissues it)
    unsigned long long en = load_at(a);
    // With the ring the chunks run in halves of kRingChunks, each in two parts: the first
    // kRingChunks - 2 chunks read indexes of this half only (two chunks ahead); then this half has
    // been read in full, so its slots are refilled with the half after next (needed a whole half
    // later), and the next half -- copied a whole half ago -- is waited for before the last two
    // chunks read into it.  Without the ring there is one part over all chunks.
    const int span = IRING ? kRingChunks : nch;
#pragma unroll 1
    for (int c0 = 0; c0 < nch && !dead; c0 += span) {
#pragma unroll 1
    for (int part = 0; part < (IRING ? 2 : 1) && !dead; ++part) {
      const int ca = part == 0 ? c0 : c0 + kRingChunks - 2;
      const int cb = IRING ? min(nch, part == 0 ? c0 + kRingChunks - 2 : c0 + kRingChunks) : nch;
#pragma unroll 1
    for (int c = ca; c < cb; ++c) {
      {
        const int4 k4 = kn0;
        kn0 = kn1;
        const int32_t knext = kn0.x;  // first index of chunk c + 1
        if constexpr (IRING) {
          kn1 = ring[(c + 2) & (2 * kRingChunks - 1)];  // past the row's end: a stale entry, unused
        } else {
          if (c + 2 < nch) kn1 = ld_idx4(irow + 4 * (int64_t)(c + 2), pol_stream);
        }
        const int32_t kv[5] = {k4.x, k4.y, k4.z, k4.w, knext};
        // table offsets (and escape slots) of the chunk's four steps, read only when some table
        // has an offset or escapes are coded (a block-uniform branch, once per chunk)
        int32_t ofs[4] = {0, 0, 0, 0}, esc[4] = {-1, -1, -1, -1};
        if (BYPASS || use_off) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int2 om = tsm2[min((uint32_t)kv[q], kmark)];
            ofs[q] = om.x;
            esc[q] = om.y;
          }
        }
        int32_t ov[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int32_t k = kv[q];
          const uintptr_t rown = row_of(kv[q + 1]);
          const S x0 = x;
          const uint32_t w0 = nextw;
          const int p0 = p;
          const unsigned long long e = en;
          const uint32_t cum = (uint32_t)x & cmask;
          const S xs = x >> P.fp;
          const uint32_t lo = (uint32_t)e, hi = (uint32_t)(e >> 32);
          uint32_t f, off, sv;
          bool slow;
          if constexpr (FUSED) {
            f = (lo & 0xFFFFu) + 1u;
            off = lo >> 16;
            sv = hi;
            slow = hi == 0xFFFFu || (uint32_t)k > klast;
          } else {
            const bool up = (cum << 16) > lo;  // cum >= c1
            const uint32_t f0 = hi & 0xFFFFu;
            f = up ? (hi >> 16) : f0;
            off = (cum - 1u - (lo >> 16)) + (up ? 0u : f0);
            const uint32_t s0 = lo & 0xFFFFu;
            sv = s0 + (up ? 1u : 0u);
            slow = s0 == 0xFFFFu;
          }
          if constexpr (BYPASS) slow |= (int32_t)sv == esc[q];
          x = (S)(xs * (S)f + (S)off);
          if constexpr (!VT<V>::LOOP) {
            // single refill (rans64, rans32_16): the low word after a refill is the prefetched word
            const bool r = (unsigned long long)x < VT<V>::LB;
            const uintptr_t an = addr_of(rown, (uint32_t)x);
            const uintptr_t ar = addr_of(rown, nextw);
            x = r ? (S)((x << VT<V>::WB) | (S)nextw) : x;
            a = r ? ar : an;
            p -= r ? 1 : 0;
            // (on a slow step this prefetch is wasted but harmless: the index check still holds and
            // the rare branch restarts from the saved cursor and word)
            nextw = ld_word_if(pw + p, r && p >= first, r ? 0u : nextw);
          } else {
            // rans32 (byte words): up to MAX_RENORM refills, the first from the prefetched word
#pragma unroll
            for (int t = 0; t < VT<V>::MAX_RENORM; ++t) {
              const bool r = (unsigned long long)x < VT<V>::LB;
              x = r ? (S)((x << VT<V>::WB) | (S)nextw) : x;
              p -= r ? 1 : 0;
              nextw = ld_word_if(pw + p, r && p >= first, r ? 0u : nextw);
            }
            a = addr_of(rown, (uint32_t)x);
          }
          ov[q] = (int32_t)sv;  // the table offset is added per chunk (rare steps return it added)
          en = load_at(a);  // every address is a row plus a masked offset: inside the table
          if (slow) {
            bool done = false;
            unsigned long long er = e;  // the entry the rare step decodes
            const uint32_t c0 = (uint32_t)x0 & cmask;
            // finish the step from the saved state with x already decoded (before renormalisation)
            auto finish = [&](S xx, uint32_t svv) {
              uint32_t ww = w0;
              int pp = p0;
#pragma unroll
              for (int t = 0; t < VT<V>::MAX_RENORM; ++t) {
                const bool r = (unsigned long long)xx < VT<V>::LB;
                xx = r ? (S)((xx << VT<V>::WB) | (S)ww) : xx;
                pp -= r ? 1 : 0;
                ww = ld_word_if(pw + pp, r && pp >= first, r ? 0u : ww);
              }
              x = xx;
              nextw = ww;
              p = pp;
              ov[q] = (int32_t)svv;
              done = true;
            };
            if constexpr (L1) {
              // the level-1 entry could not decode this cum: the 16-cum entry from the bucket table
              const uintptr_t rk = bk0 + (uintptr_t)min((uint32_t)k, kmark) * rowbytes;
              er = ld_hint_u64(reinterpret_cast<const unsigned long long*>(rk | ((((uint32_t)x0) >> 1) & bmask)),
                               pol_keep);
              const uint32_t lo2 = (uint32_t)er, hi2 = (uint32_t)(er >> 32);
              const bool up2 = (c0 << 16) > lo2;
              const uint32_t g0 = hi2 & 0xFFFFu;
              const uint32_t f2 = up2 ? (hi2 >> 16) : g0;
              const uint32_t off2 = (c0 - 1u - (lo2 >> 16)) + (up2 ? 0u : g0);
              const uint32_t s2 = lo2 & 0xFFFFu;
              const uint32_t sv2 = s2 + (up2 ? 1u : 0u);
              bool slow2 = s2 == 0xFFFFu;
              if constexpr (BYPASS) slow2 |= (int32_t)sv2 == esc[q];
              if (!slow2) finish((S)((x0 >> P.fp) * (S)f2 + (S)off2), sv2);
            }
            if constexpr (!FUSED) {
              // the typed markers, decoded here without the call: a run of unit-frequency symbols
              // (type 1: symbol cum + d, freq 1, offset 0) or a block of per-cum entries in the
              // secondary table (type 2: s | offset << 16 | freq << 32, one load)
              if (!done && (er & 0x3FFFFull) == 0x1FFFFull) {
                const uint32_t svu = c0 + (uint32_t)(er >> 32);
                if (!BYPASS || (int32_t)svu != esc[q]) finish((S)(x0 >> P.fp), svu);
              } else if (!done && (er & 0x3FFFFull) == 0x2FFFFull) {
                const unsigned long long d2 =
                    ld_hint_u64(P.fSEC + ((er >> 18) << kBucketBits) + (c0 & ((1u << kBucketBits) - 1u)), pol_keep);
                const uint32_t svs = (uint32_t)(d2 & 0xFFFFull);
                if (!BYPASS || (int32_t)svs != esc[q])
                  finish((S)((x0 >> P.fp) * (S)(uint32_t)(d2 >> 32) + (S)((uint32_t)(d2 >> 16) & 0xFFFFu)), svs);
              }
            }
            if (!done) {
              LeanState<V> st{x0, (S)w0, (long long)p0, err, 0};
              if constexpr (FUSED) st = popl_exact<V, LK, BYPASS, TM_FUSED_SMEM>(P, st, row, k, tsm, tD, tS);
              else st = popb_rare<V, LK, BYPASS>(P, st, row, k, er, tsm);
              x = st.x;
              nextw = (uint32_t)st.nextw;
              p = (int)min(max(st.p, -0x7fffffffll), 0x7fffffffll);
              err = st.err;
              ov[q] = (int32_t)((uint32_t)st.v - (uint32_t)ofs[q]);
            }
            a = addr_of(rown, (uint32_t)x);
            en = load_at(a);
          }
        }
        if (use_off) {
#pragma unroll
          for (int q = 0; q < 4; ++q) ov[q] = (int32_t)((uint32_t)ov[q] + (uint32_t)ofs[q]);
        }
        st_hint_v4(reinterpret_cast<int4*>(orow + 4 * (int64_t)c), make_int4(ov[0], ov[1], ov[2], ov[3]), pol_stream);
      }
    }
      if (IRING && part == 0) {
        const int h = (c0 / kRingChunks) & 1;
        if (c0 + 2 * kRingChunks < nch) {
          fence_proxy_async_shared();  // this half's reads come before the copy over it
          ring_issue(h, c0 + 2 * kRingChunks);
        }
        if (c0 + kRingChunks < nch && !ring_wait(h ^ 1)) dead = true;
      }
    }
    }
    // after a wait that ran out, let the copies still in flight land (bounded) before leaving
    if constexpr (IRING) {
      for (int h = 0; h < 2; ++h)
        if (pend & (1u << h)) ring_wait(h);
    }
    if (p < p_init && p + 1 < first) err |= DEV_UNDERFLOW;
  }
  store_state<V>(row, 0, x);
  row[0] = (int32_t)(((int64_t)p + 1) * VT<V>::WBYTES);
  report(P.status, err);
}

template <int V>
bool launch_pop_lean(const PopParams& P, int lookup, bool bypass, int tm, int blocks, int threads, size_t smem,
                     cudaStream_t s);

template <int V, int LK, bool BY, int MODE, bool IR>
void popb_go2(const PopParams& P, int blocks, int threads, size_t smem, cudaStream_t s) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(pop_bucket_kernel<V, LK, BY, MODE, IR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  pop_bucket_kernel<V, LK, BY, MODE, IR><<<blocks, threads, smem, s>>>(P);
  note_launch();
}
template <int V, int LK, bool BY, int MODE>
void popb_go1(const PopParams& P, int blocks, int threads, size_t smem, cudaStream_t s) {
  if (P.iring) popb_go2<V, LK, BY, MODE, true>(P, blocks, threads, smem, s);
  else popb_go2<V, LK, BY, MODE, false>(P, blocks, threads, smem, s);
}
template <int V, int LK, bool BY>
void popb_go(const PopParams& P, int blocks, int threads, size_t smem, cudaStream_t s) {
  if (P.fL1 && P.l1_bytes > 0) popb_go1<V, LK, BY, BM_L1>(P, blocks, threads, smem, s);
  else popb_go1<V, LK, BY, BM_L2>(P, blocks, threads, smem, s);
}

template <int V, int LK, bool BY, int TM>
void popl_go(const PopParams& P, int blocks, int threads, size_t smem, cudaStream_t s) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(pop_lean_kernel<V, LK, BY, TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  pop_lean_kernel<V, LK, BY, TM><<<blocks, threads, smem, s>>>(P);
  note_launch();
}

template <int V, bool BY>
bool popl_tm(const PopParams& P, int lookup, int tm, int blocks, int threads, size_t smem, cudaStream_t s) {
  if (lookup == 2) {  // alias: only the fused layout (its offsets depend on cum, not on s)
    if (tm == TM_FUSED_SMEM) popb_go1<V, 2, BY, BM_FUSED>(P, blocks, threads, smem, s);
    else if (tm == TM_FUSED_GLOBAL) popl_go<V, 2, BY, TM_FUSED_GLOBAL>(P, blocks, threads, smem, s);
    else return false;
    return true;
  }
  if (lookup == 1) {
    if (tm == TM_BUCKET_GLOBAL) popb_go<V, 1, BY>(P, blocks, threads, smem, s);
    else if (tm == TM_FUSED_SMEM) popb_go1<V, 1, BY, BM_FUSED>(P, blocks, threads, smem, s);
    else if (tm == TM_SPLIT_SMEM) popl_go<V, 1, BY, TM_SPLIT_SMEM>(P, blocks, threads, smem, s);
    else if (tm == TM_SPLIT_GLOBAL) popl_go<V, 1, BY, TM_SPLIT_GLOBAL>(P, blocks, threads, smem, s);
    else return false;
    return true;
  }
  if (tm == TM_BUCKET_GLOBAL) popb_go<V, 0, BY>(P, blocks, threads, smem, s);
  else if (tm == TM_FUSED_SMEM) popb_go1<V, 0, BY, BM_FUSED>(P, blocks, threads, smem, s);
  else if (tm == TM_SPLIT_SMEM) popl_go<V, 0, BY, TM_SPLIT_SMEM>(P, blocks, threads, smem, s);
  else if (tm == TM_SPLIT_GLOBAL) popl_go<V, 0, BY, TM_SPLIT_GLOBAL>(P, blocks, threads, smem, s);
  else return false;
  return true;
}

#define TANS_DEFINE_POP_LEAN(VV)                                                                               \
  template <>                                                                                                  \
  bool launch_pop_lean<VV>(const PopParams& P, int lookup, bool bypass, int tm, int blocks, int threads,       \
                           size_t smem, cudaStream_t s) {                                                      \
    return bypass ? popl_tm<VV, true>(P, lookup, tm, blocks, threads, smem, s)                                 \
                  : popl_tm<VV, false>(P, lookup, tm, blocks, threads, smem, s);                               \
  }

}  // namespace tans
