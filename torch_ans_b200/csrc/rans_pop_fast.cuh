// rans_pop_fast.cuh -- the fast single-state pop kernel (rows 16-byte aligned, length % 4 == 0).
//
// Each thread decodes SPT streams at once: the SPT serial chains are independent, so while one
// waits on its table load the others issue (instruction-level parallelism inside a warp, which
// matters because a latency-bound launch has only a few warps per SM).  Per symbol a chain does
// one table access (or two for the split layout) and a multiply-add; table indexes arrive by
// cp.async in a shared-memory ring POPF_L chunks ahead; the next stream word is prefetched into a
// register so a refill never waits on memory; decoded symbols leave as 16-byte stores.
//
// Table layouts (TM), all built per call from the caller's tables by replaying the reference's
// own lookup, so every layout returns exactly what rans_pop_step would:
//   TM_FUSED_SMEM / TM_FUSED_GLOBAL: D[k][cum] = (freq - 1) | (cum - start) << 16, S[k][cum] = s
//   TM_SPLIT_SMEM / TM_SPLIT_GLOBAL: S[k][cum] = s, ST[k][s] = (freq - 1) | start << 16
//   TM_BUCKET_GLOBAL: one 8-byte entry per 16 cum values holding the bucket's first symbol, its
//     freq, the start and freq of the next symbol (so at most one boundary inside the bucket):
//     one load resolves (s, start, freq); buckets the entry cannot describe (verified per cum at
//     build time) carry a marker and use the split tables, which are built alongside
// S = 0xFFFF marks the entries the packed layouts cannot hold; those steps take the direct lookup.
#pragma once

#include "rans_pop.cuh"

namespace tans {

enum : int { TM_FUSED_SMEM = 0, TM_FUSED_GLOBAL = 1, TM_SPLIT_SMEM = 2, TM_SPLIT_GLOBAL = 3, TM_BUCKET_GLOBAL = 4 };
constexpr int kBucketBits = 4;  // bucket layout: 16 cum values per bucket
constexpr int kL1Bits = 8;      // level-1 table in shared memory: 256 cum values per entry
constexpr int kL1AutoBits = 8;  // coarsest level-1 entry (cum values, log2) chosen without being asked
constexpr int POPF_RS = 8;  // index ring slots (chunks of 4)
constexpr int POPF_L = 6;   // chunks between an index load and its use

// bytes of shared memory the tables of a layout occupy (each region 16-byte aligned and padded to
// a multiple of 16 bytes for the bulk copies)
inline int64_t popf_table_smem(int tm, int64_t ntables, int fp, int64_t cdf_width, int64_t st_stride) {
  (void)cdf_width;
  const int64_t m = ntables << fp;
  const int64_t info = ntables * 32;  // TableInfo + a per-table record of the kernels, padded
  auto r16 = [](int64_t b) { return (b + 15) & ~(int64_t)15; };
  switch (tm) {
    case TM_FUSED_SMEM: return info + r16(m * 4) + r16(m * 2) + 16;
    case TM_SPLIT_SMEM: return info + r16(ntables * st_stride * 4) + r16(m * 2) + 16;
    default: return info;
  }
}

// 16-byte aligned start of the table region after the per-table records
__device__ __forceinline__ unsigned char* popf_align16(void* p) {
  return reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 15) & ~(uintptr_t)15);
}

// Stage the shared-memory table layouts (fused D + S, or split ST + S) with 1D TMA bulk copies:
// thread 0 announces the bytes on an mbarrier and issues the copies (popf_stage_begin), the copy
// engine moves the tables while the block fills its per-table records, then every thread waits
// for the phase with a bounded loop (popf_stage_end).  The regions are the workspace arrays
// (256-byte aligned, padded) and 16-byte aligned shared regions, sizes rounded up to 16 bytes;
// anything misaligned falls back to a thread copy.
template <int TM>
__device__ __forceinline__ void popf_stage_begin(const PopParams& P, uint32_t* tD, uint16_t* tS, int64_t m,
                                                 unsigned long long* bar, int* use_tma) {
  if constexpr (TM == TM_FUSED_SMEM || TM == TM_SPLIT_SMEM) {
    const int T = blockDim.x, tid = threadIdx.x;
    const void* srcA = TM == TM_FUSED_SMEM ? (const void*)P.fD : (const void*)P.fST;
    const int64_t nA = TM == TM_FUSED_SMEM ? m : P.ntables * P.st_stride;  // 4-byte words of D / ST
    const unsigned bytesA = (unsigned)((nA * 4 + 15) & ~(int64_t)15);
    const unsigned bytesS = (unsigned)((m * 2 + 15) & ~(int64_t)15);
    if (tid == 0) {
      const bool ok = ((reinterpret_cast<uintptr_t>(srcA) | reinterpret_cast<uintptr_t>(P.fS)) & 15u) == 0 &&
                      ((smem_u32(tD) | smem_u32(tS)) & 15u) == 0 && bytesA + bytesS < (1u << 20);
      *use_tma = ok ? 1 : 0;
      if (ok) {
        mbar_init(bar, 1);
        mbar_init_fence();
        constexpr unsigned kChunk = 32768;
        mbar_arrive_expect_tx(bar, bytesA + bytesS);
        for (unsigned o = 0; o < bytesA; o += kChunk)
          bulk_copy_g2s(reinterpret_cast<unsigned char*>(tD) + o, reinterpret_cast<const unsigned char*>(srcA) + o,
                        min(kChunk, bytesA - o), bar);
        for (unsigned o = 0; o < bytesS; o += kChunk)
          bulk_copy_g2s(reinterpret_cast<unsigned char*>(tS) + o, reinterpret_cast<const unsigned char*>(P.fS) + o,
                        min(kChunk, bytesS - o), bar);
      }
    }
    __syncthreads();
    if (!*use_tma) {
      for (int64_t i = tid; i < nA; i += T) tD[i] = reinterpret_cast<const uint32_t*>(srcA)[i];
      for (int64_t i = tid; i < m; i += T) tS[i] = P.fS[i];
    }
  }
}

// wait for the staged tables; false when the wait ran out.  Callers combine the result over the
// block (__syncthreads_and) and, when any thread gave up, call popf_stage_drain before leaving.
template <int TM>
__device__ __forceinline__ bool popf_stage_end(unsigned long long* bar, const int* use_tma) {
  if constexpr (TM == TM_FUSED_SMEM || TM == TM_SPLIT_SMEM) {
    if (!*use_tma) return true;
    for (unsigned it = 0; it < (1u << 20); ++it)
      if (mbar_try_wait(bar, 0)) return true;
    return false;
  } else {
    return true;
  }
}

// After a wait that ran out: wait once more, again bounded, for the bulk copies to land, so that no
// copy is still writing the block's shared memory when its threads leave; then report the stall.
template <int TM>
__device__ __forceinline__ void popf_stage_drain(unsigned long long* bar, const int* use_tma, uint32_t* status) {
  popf_stage_end<TM>(bar, use_tma);
  __syncthreads();
  if (threadIdx.x == 0) report(status, DEV_STALLED);
}

template <int V> struct FastCursor {
  using S = typename VT<V>::State;
  using W = typename VT<V>::Word;
  PopCursor<V> c;
  S nextw;  // word at index c.p (0 outside the row's data words)

  __device__ __forceinline__ void prime() {
    nextw = (c.p >= c.first && c.p < c.cap) ? (S)__ldg(reinterpret_cast<const W*>(c.payload) + c.p) : (S)0;
  }
  // RANS_POP_STATE_RENORM with the word already in a register (single-refill variants)
  __device__ __forceinline__ void refill(S& x) {
    if constexpr (VT<V>::LOOP) {
      c.refill(x);
    } else {
      if ((unsigned long long)x < VT<V>::LB) {
        if (c.p < c.first || c.p >= c.cap) c.err |= DEV_UNDERFLOW;
        x = (S)((x << VT<V>::WB) | nextw);
        c.p -= 1;
        prime();
      }
    }
  }
};

// Exact handling of one symbol of one stream (every case the reference has: bad index, packed
// table miss, escapes, underflow).  Used to replay a chunk the optimistic pass flagged.
template <int V, int LK, bool BYPASS, int TM>
__device__ __forceinline__ int32_t popf_exact(const PopParams& P, typename VT<V>::State& x, FastCursor<V>& cur,
                                              int32_t k, const TableInfo* tsm, const uint32_t* tD, const uint16_t* tS,
                                              unsigned long long pol_keep) {
  using S = typename VT<V>::State;
  if ((uint32_t)k >= (uint64_t)P.ntables) {
    cur.c.err |= DEV_BAD_INDEX;
    return 0;
  }
  const TableInfo ti = P.tin_smem ? tsm[k] : load_tinfo(P.tinfo, k);
  const uint32_t cum = (uint32_t)x & (uint32_t)(((int64_t)1 << P.fp) - 1);
  const int64_t e = ((int64_t)k << P.fp) | cum;
  bool fast = false;
  int32_t sv = 0, off = 0, freq = 0;
  if constexpr (TM == TM_FUSED_SMEM || TM == TM_FUSED_GLOBAL) {
    uint32_t d, s16;
    if constexpr (TM == TM_FUSED_SMEM) {
      d = tD[e];
      s16 = tS[e];
    } else {
      d = ld_hint_u32(P.fD + e, pol_keep);
      s16 = ld_hint_u16(P.fS + e, pol_keep);
    }
    fast = s16 != 0xFFFFu;
    sv = (int32_t)s16;
    freq = (int32_t)(d & 0xFFFFu) + 1;
    off = (int32_t)(d >> 16);
  } else {
    uint32_t s16, st = 0;
    if constexpr (TM == TM_SPLIT_SMEM) {
      s16 = tS[e];
      fast = s16 != 0xFFFFu;
      if (fast) st = tD[(int64_t)k * P.st_stride + s16];
    } else {
      s16 = ld_hint_u16(P.fS + e, pol_keep);
      fast = s16 != 0xFFFFu;
      if (fast) st = ld_hint_u32(P.fST + (int64_t)k * P.st_stride + s16, pol_keep);
    }
    sv = (int32_t)s16;
    freq = (int32_t)(st & 0xFFFFu) + 1;
    off = (int32_t)cum - (int32_t)(st >> 16);
  }
  int32_t v;
  bool ok = true;
  if (fast) {
    x = (S)((x >> P.fp) * to_state<S>(freq) + to_state<S>(off));
    cur.c.refill(x);
    v = sv;
    if constexpr (BYPASS) {
      if (v == ti.size - 2) {
        const int32_t raw = pop_escape<V>(x, cur.c, P.bp);
        v = raw >> 1;
        v = (raw & 1) ? (-v - 1) : (v + ti.size - 2);
      }
    }
  } else {
    v = pop_chain<V, LK, BYPASS>(P, x, cur.c, k, ti, ok);
  }
  return ok ? (int32_t)((uint32_t)v + (uint32_t)ti.offset) : 0;
}

template <int V, int LK, bool BYPASS, int TM, int SPT>
__global__ void __launch_bounds__(512) pop_fast_kernel(const PopParams P) {
  using S = typename VT<V>::State;
  using W = typename VT<V>::Word;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  const int warps = T >> 5, warp = tid >> 5, lane = tid & 31;
  const int nact = warps * P.lanes;
  const int at = warp * P.lanes + lane;
  int4* ring = reinterpret_cast<int4*>(smem_raw);
  TableInfo* tsm = reinterpret_cast<TableInfo*>(ring + POPF_RS * nact * SPT);
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
    tsm2[k] = make_int2(ti.offset, ti.size - 2);
  }
  const bool staged = __syncthreads_and(popf_stage_end<TM>(&stage_bar, &stage_tma) ? 1 : 0) != 0;
  if (!staged) {
    popf_stage_drain<TM>(&stage_bar, &stage_tma, P.status);
    return;
  }
  if (lane >= P.lanes) return;

  // streams of this thread; slots past the batch shadow the thread's first stream (same reads,
  // nothing written), so the arithmetic below stays free of per-stream branches
  const int64_t tg = ((int64_t)blockIdx.x * warps + warp) * P.lanes + lane;
  if (tg * SPT >= P.batch) return;
  int64_t b[SPT];
  bool live[SPT];
  FastCursor<V> cur[SPT];
  S x[SPT];
  const W* pw[SPT];
  int32_t pcap[SPT];
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    live[j] = tg * SPT + j < P.batch;
    b[j] = live[j] ? tg * SPT + j : tg * SPT;
    const int32_t* row = P.stream + b[j] * P.width;
    cur[j].c.payload = reinterpret_cast<const uint8_t*>(row + 1);
    cur[j].c.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
    cur[j].c.first = VT<V>::SBYTES / VT<V>::WBYTES;
    cur[j].c.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
    cur[j].c.err = 0;
    x[j] = load_state<V>(row, 0);
    cur[j].prime();
    pw[j] = reinterpret_cast<const W*>(cur[j].c.payload);
    pcap[j] = (int32_t)min(cur[j].c.cap - 1, (int64_t)0x7fffffff);
  }
  bool always_exact = false;  // a row whose length points past its end is replayed exactly
#pragma unroll
  for (int j = 0; j < SPT; ++j) always_exact |= cur[j].c.p >= cur[j].c.cap || cur[j].c.p > 0x7ffffff0;
  const unsigned long long pol_keep = policy_evict_last(), pol_stream = policy_evict_first();
  const uint32_t cmask = (uint32_t)(M - 1);
  const uint32_t kmax = (uint32_t)(P.ntables - 1);
  const int64_t N = P.nsym;
  const int nch = (int)(N >> 2);
  const int first = VT<V>::SBYTES / VT<V>::WBYTES;

  for (int t = 0; t < nch + POPF_L; ++t) {
    if (t < nch) {
      int4* slot = ring + ((int64_t)(t & (POPF_RS - 1)) * nact + at) * SPT;
#pragma unroll
      for (int j = 0; j < SPT; ++j) cp_async16_hint(slot + j, P.idx + b[j] * N + 4 * (int64_t)t, pol_stream);
    }
    cp_async_commit();
    cp_async_wait<POPF_L - 1>();
    const int cc = t - POPF_L;
    if (cc < 0) continue;
    const int4* slot = ring + ((int64_t)(cc & (POPF_RS - 1)) * nact + at) * SPT;
    int32_t kv[SPT][4], ov[SPT][4];
    S x0[SPT], w0[SPT];
    int32_t p0[SPT];
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
      const int4 k4 = slot[j];
      kv[j][0] = k4.x;
      kv[j][1] = k4.y;
      kv[j][2] = k4.z;
      kv[j][3] = k4.w;
      x0[j] = x[j];
      w0[j] = cur[j].nextw;
      p0[j] = (int32_t)cur[j].c.p;
    }
    // ---- optimistic pass: straight-line code over the chunk's 4 x SPT steps
    bool redo = always_exact;
    if constexpr (!VT<V>::LOOP) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        // phase 1: table loads of every stream (independent, all in flight together)
        uint32_t kc[SPT], cum[SPT], sv[SPT], d[SPT];
        unsigned long long bk[SPT];
        bool fb[SPT];
        int2 om[SPT];
#pragma unroll
        for (int j = 0; j < SPT; ++j) {
          const int32_t k = kv[j][q];
          kc[j] = min((uint32_t)k, kmax);
          redo |= (uint32_t)k > kmax;
          om[j] = tsm2[kc[j]];
          cum[j] = (uint32_t)x[j] & cmask;
          const int64_t e = ((int64_t)kc[j] << P.fp) | cum[j];
          if constexpr (TM == TM_FUSED_SMEM) {
            d[j] = tD[e];
            sv[j] = tS[e];
          } else if constexpr (TM == TM_FUSED_GLOBAL) {
            d[j] = ld_hint_u32(P.fD + e, pol_keep);
            sv[j] = ld_hint_u16(P.fS + e, pol_keep);
          } else if constexpr (TM == TM_SPLIT_SMEM) {
            sv[j] = tS[e];
          } else if constexpr (TM == TM_BUCKET_GLOBAL) {
            bk[j] = ld_hint_u64(P.fBK + (e >> kBucketBits), pol_keep);
          } else {
            sv[j] = ld_hint_u16(P.fS + e, pol_keep);
          }
        }
        if constexpr (TM == TM_BUCKET_GLOBAL) {
          // decode the bucket entries; marked buckets take the split tables (warp-uniform branch)
          bool fb_any = false;
#pragma unroll
          for (int j = 0; j < SPT; ++j) {
            // lo = s0 | (c1 - 1) << 16, hi = freq(s0) | freq(s0 + 1) << 16
            const uint32_t lo = (uint32_t)bk[j], hi = (uint32_t)(bk[j] >> 32);
            const uint32_t s0 = lo & 0xFFFFu, c1 = (lo >> 16) + 1u, f0 = hi & 0xFFFFu;
            fb[j] = s0 == 0xFFFFu;
            fb_any |= fb[j];
            const bool up = (cum[j] << 16) > lo;  // cum >= c1
            sv[j] = s0 + (up ? 1u : 0u);
            // d = (freq - 1) | start << 16 (start < 2^16 for every describable bucket)
            d[j] = up ? (((hi >> 16) - 1u) | (c1 << 16)) : ((f0 - 1u) | ((c1 - f0) << 16));
          }
          if (__any_sync(__activemask(), fb_any)) {
#pragma unroll
            for (int j = 0; j < SPT; ++j)
              if (fb[j]) sv[j] = ld_hint_u16(P.fS + ((((int64_t)kc[j]) << P.fp) | cum[j]), pol_keep);
#pragma unroll
            for (int j = 0; j < SPT; ++j)
              if (fb[j])
                d[j] = ld_hint_u32(P.fST + (int64_t)kc[j] * P.st_stride + min(sv[j], (uint32_t)(P.st_stride - 1)),
                                   pol_keep);
          }
        }
        // phase 2 (split layouts): the per-symbol {freq, start} loads
        if constexpr (TM == TM_SPLIT_SMEM || TM == TM_SPLIT_GLOBAL) {
#pragma unroll
          for (int j = 0; j < SPT; ++j) {
            const int64_t si = (int64_t)kc[j] * P.st_stride + min(sv[j], (uint32_t)(P.st_stride - 1));
            if constexpr (TM == TM_SPLIT_SMEM) d[j] = tD[si];
            else d[j] = ld_hint_u32(P.fST + si, pol_keep);
          }
        }
        // phase 3: state updates and refills
#pragma unroll
        for (int j = 0; j < SPT; ++j) {
          uint32_t freq, off;
          if constexpr (TM == TM_FUSED_SMEM || TM == TM_FUSED_GLOBAL) {
            freq = (d[j] & 0xFFFFu) + 1u;
            off = d[j] >> 16;
          } else {  // split and bucket layouts: d = (freq - 1) | start << 16
            freq = (d[j] & 0xFFFFu) + 1u;
            off = cum[j] - (d[j] >> 16);
          }
          redo |= sv[j] == 0xFFFFu;
          if constexpr (BYPASS) redo |= (int32_t)sv[j] == om[j].y;
          x[j] = (S)((x[j] >> P.fp) * (S)freq + (S)off);
          // single refill with the prefetched word; the next word is fetched at a clamped index
          const bool r = (unsigned long long)x[j] < VT<V>::LB;
          const int32_t pc = (int32_t)cur[j].c.p;
          redo |= r && (pc < first);
          x[j] = r ? (S)((x[j] << VT<V>::WB) | cur[j].nextw) : x[j];
          const int32_t pn = pc - (r ? 1 : 0);
          cur[j].c.p = pn;
          if (r) cur[j].nextw = (S)__ldg(pw[j] + min(max(pn, 0), pcap[j]));
          ov[j][q] = (int32_t)(sv[j] + (uint32_t)om[j].x);
        }
      }
    } else {
      redo = true;  // byte-word coder: several refills per step, always the exact path
    }
    if (redo) {
      // ---- exact replay of this chunk from the saved states
#pragma unroll
      for (int j = 0; j < SPT; ++j) {
        x[j] = x0[j];
        cur[j].nextw = w0[j];
        cur[j].c.p = p0[j];
      }
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int j = 0; j < SPT; ++j) {
          ov[j][q] = popf_exact<V, LK, BYPASS, TM>(P, x[j], cur[j], kv[j][q], tsm, tD, tS, pol_keep);
          cur[j].prime();
        }
      }
    }
#pragma unroll
    for (int j = 0; j < SPT; ++j)
      if (live[j])
        st_hint_v4(reinterpret_cast<int4*>(P.out + b[j] * N + 4 * (int64_t)cc),
                   make_int4(ov[j][0], ov[j][1], ov[j][2], ov[j][3]), pol_stream);
  }
  cp_async_wait<0>();
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    if (!live[j]) continue;
    int32_t* row = P.stream + b[j] * P.width;
    store_state<V>(row, 0, x[j]);
    row[0] = (int32_t)((cur[j].c.p + 1) * VT<V>::WBYTES);
    report(P.status, cur[j].c.err);
  }
}

// launch one (V) variant of the fast kernel; returns false when no layout applies
template <int V>
bool launch_pop_fast(const PopParams& P, int lookup, bool bypass, int tm, int spt, int blocks, int threads,
                     size_t smem, cudaStream_t s);

}  // namespace tans

namespace tans {

template <int V, int LK, bool BY, int TM, int SPT>
void popf_go(const PopParams& P, int blocks, int threads, size_t smem, cudaStream_t s) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(pop_fast_kernel<V, LK, BY, TM, SPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  pop_fast_kernel<V, LK, BY, TM, SPT><<<blocks, threads, smem, s>>>(P);
  note_launch();
}

template <int V, int LK, bool BY, int TM>
void popf_spt(const PopParams& P, int spt, int blocks, int threads, size_t smem, cudaStream_t s) {
  if (spt >= 4) popf_go<V, LK, BY, TM, 4>(P, blocks, threads, smem, s);
  else if (spt == 2) popf_go<V, LK, BY, TM, 2>(P, blocks, threads, smem, s);
  else popf_go<V, LK, BY, TM, 1>(P, blocks, threads, smem, s);
}

template <int V, bool BY>
bool popf_tm(const PopParams& P, int lookup, int tm, int spt, int blocks, int threads, size_t smem, cudaStream_t s) {
  if (lookup == 2) {  // alias: only the fused layout (its offsets depend on cum, not on s)
    if (tm == TM_FUSED_SMEM) popf_spt<V, 2, BY, TM_FUSED_SMEM>(P, spt, blocks, threads, smem, s);
    else if (tm == TM_FUSED_GLOBAL) popf_spt<V, 2, BY, TM_FUSED_GLOBAL>(P, spt, blocks, threads, smem, s);
    else return false;
    return true;
  }
  if (lookup == 1) {
    if (tm == TM_BUCKET_GLOBAL) popf_spt<V, 1, BY, TM_BUCKET_GLOBAL>(P, spt, blocks, threads, smem, s);
    else if (tm == TM_FUSED_SMEM) popf_spt<V, 1, BY, TM_FUSED_SMEM>(P, spt, blocks, threads, smem, s);
    else if (tm == TM_SPLIT_SMEM) popf_spt<V, 1, BY, TM_SPLIT_SMEM>(P, spt, blocks, threads, smem, s);
    else if (tm == TM_SPLIT_GLOBAL) popf_spt<V, 1, BY, TM_SPLIT_GLOBAL>(P, spt, blocks, threads, smem, s);
    else return false;
    return true;
  }
  if (tm == TM_BUCKET_GLOBAL) popf_spt<V, 0, BY, TM_BUCKET_GLOBAL>(P, spt, blocks, threads, smem, s);
  else if (tm == TM_FUSED_SMEM) popf_spt<V, 0, BY, TM_FUSED_SMEM>(P, spt, blocks, threads, smem, s);
  else if (tm == TM_SPLIT_SMEM) popf_spt<V, 0, BY, TM_SPLIT_SMEM>(P, spt, blocks, threads, smem, s);
  else if (tm == TM_SPLIT_GLOBAL) popf_spt<V, 0, BY, TM_SPLIT_GLOBAL>(P, spt, blocks, threads, smem, s);
  else return false;
  return true;
}

#define TANS_DEFINE_POP_FAST(VV)                                                                              \
  template <>                                                                                                 \
  bool launch_pop_fast<VV>(const PopParams& P, int lookup, bool bypass, int tm, int spt, int blocks, int threads, \
                           size_t smem, cudaStream_t s) {                                                     \
    return bypass ? popf_tm<VV, true>(P, lookup, tm, spt, blocks, threads, smem, s)                           \
                  : popf_tm<VV, false>(P, lookup, tm, spt, blocks, threads, smem, s);                         \
  }

}  // namespace tans
