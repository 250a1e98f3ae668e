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
//   TM_CDF_SMEM: the cdf rows themselves in shared memory, bisection as in rans_utils.hpp:427-448
// S = 0xFFFF marks the entries the packed layouts cannot hold; those steps take the direct lookup.
#pragma once

#include "rans_pop.cuh"

namespace tans {

enum : int { TM_FUSED_SMEM = 0, TM_FUSED_GLOBAL = 1, TM_SPLIT_SMEM = 2, TM_SPLIT_GLOBAL = 3, TM_CDF_SMEM = 4 };
constexpr int POPF_RS = 8;  // index ring slots (chunks of 4)
constexpr int POPF_L = 6;   // chunks between an index load and its use

// bytes of shared memory the tables of a layout occupy
inline int64_t popf_table_smem(int tm, int64_t ntables, int fp, int64_t cdf_width, int64_t st_stride) {
  const int64_t m = ntables << fp;
  switch (tm) {
    case TM_FUSED_SMEM: return m * 4 + m * 2 + 16;
    case TM_SPLIT_SMEM: return ntables * st_stride * 4 + m * 2 + 16;
    case TM_CDF_SMEM: return ntables * cdf_width * 4;
    default: return 0;
  }
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

template <int V, int LK, bool BYPASS, int TM, int SPT>
__global__ void __launch_bounds__(128) pop_fast_kernel(const PopParams P) {
  using S = typename VT<V>::State;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  const int warps = T >> 5, warp = tid >> 5, lane = tid & 31;
  const int nact = warps * P.lanes;
  const int at = warp * P.lanes + lane;
  int4* ring = reinterpret_cast<int4*>(smem_raw);
  TableInfo* tsm = reinterpret_cast<TableInfo*>(ring + POPF_RS * nact * SPT);
  unsigned char* tab = reinterpret_cast<unsigned char*>(tsm + (P.tin_smem ? P.ntables : 0));
  const int64_t M = (int64_t)1 << P.fp;
  const int64_t m = P.ntables << P.fp;
  uint32_t* tD = reinterpret_cast<uint32_t*>(tab);  // fused: D; split: ST; cdf: rows
  uint16_t* tS = reinterpret_cast<uint16_t*>(
      tab + (TM == TM_FUSED_SMEM ? m * 4 : (TM == TM_SPLIT_SMEM ? P.ntables * P.st_stride * 4 : 0)));
  if (P.tin_smem)
    for (int64_t k = tid; k < P.ntables; k += T) tsm[k] = P.tinfo[k];
  if constexpr (TM == TM_FUSED_SMEM) {
    for (int64_t i = tid; i < m; i += T) tD[i] = P.fD[i];
    for (int64_t i = tid; i < m; i += T) tS[i] = P.fS[i];
  } else if constexpr (TM == TM_SPLIT_SMEM) {
    const int64_t n = P.ntables * P.st_stride;
    for (int64_t i = tid; i < n; i += T) tD[i] = P.fST[i];
    for (int64_t i = tid; i < m; i += T) tS[i] = P.fS[i];
  } else if constexpr (TM == TM_CDF_SMEM) {
    const int64_t n = P.ntables * P.cdf_width;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(P.cdfs);
    for (int64_t i = tid; i < n; i += T) tD[i] = src[i];
  }
  __syncthreads();
  if (lane >= P.lanes) return;

  const int64_t tg = ((int64_t)blockIdx.x * warps + warp) * P.lanes + lane;
  int64_t b[SPT];
  bool live[SPT];
  FastCursor<V> cur[SPT];
  S x[SPT];
  int32_t* rows[SPT];
#pragma unroll
  for (int j = 0; j < SPT; ++j) {
    b[j] = tg * SPT + j;
    live[j] = b[j] < P.batch;
    const int64_t bb = live[j] ? b[j] : 0;
    rows[j] = P.stream + bb * P.width;
    cur[j].c.payload = reinterpret_cast<const uint8_t*>(rows[j] + 1);
    cur[j].c.p = live[j] ? (int64_t)rows[j][0] / VT<V>::WBYTES - 1 : -1;
    cur[j].c.first = VT<V>::SBYTES / VT<V>::WBYTES;
    cur[j].c.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
    cur[j].c.err = 0;
    x[j] = load_state<V>(rows[j], 0);
    cur[j].prime();
  }
  if (!live[0]) return;
  const unsigned long long pol_keep = policy_evict_last(), pol_stream = policy_evict_first();
  const uint32_t cmask = (uint32_t)(M - 1);
  const int64_t N = P.nsym;
  const int nch = (int)(N >> 2);

  for (int t = 0; t < nch + POPF_L; ++t) {
    if (t < nch) {
      int4* slot = ring + ((int64_t)(t & (POPF_RS - 1)) * nact + at) * SPT;
#pragma unroll
      for (int j = 0; j < SPT; ++j)
        if (live[j]) cp_async16_hint(slot + j, P.idx + b[j] * N + 4 * (int64_t)t, pol_stream);
    }
    cp_async_commit();
    cp_async_wait<POPF_L - 1>();
    const int cc = t - POPF_L;
    if (cc < 0) continue;
    const int4* slot = ring + ((int64_t)(cc & (POPF_RS - 1)) * nact + at) * SPT;
    int32_t kv[SPT][4], ov[SPT][4];
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
      const int4 k4 = slot[j];
      kv[j][0] = k4.x;
      kv[j][1] = k4.y;
      kv[j][2] = k4.z;
      kv[j][3] = k4.w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int j = 0; j < SPT; ++j) {
        ov[j][q] = 0;
        if (!live[j]) continue;
        const int32_t k = kv[j][q];
        if ((uint32_t)k >= (uint64_t)P.ntables) {
          cur[j].c.err |= DEV_BAD_INDEX;
          continue;
        }
        const TableInfo ti = P.tin_smem ? tsm[k] : load_tinfo(P.tinfo, k);
        const uint32_t cum = (uint32_t)x[j] & cmask;
        bool fast = true;
        int32_t sv = 0, off = 0, freq = 0;
        if constexpr (TM == TM_FUSED_SMEM || TM == TM_FUSED_GLOBAL) {
          const int64_t e = ((int64_t)k << P.fp) | cum;
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
        } else if constexpr (TM == TM_SPLIT_SMEM || TM == TM_SPLIT_GLOBAL) {
          const int64_t e = ((int64_t)k << P.fp) | cum;
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
        } else {  // TM_CDF_SMEM: the reference's probe + bisection on the shared-memory row
          const int32_t size = ti.size;
          fast = size >= 2 && (int64_t)size <= P.cdf_width;
          if (fast) {
            const int32_t* row = reinterpret_cast<const int32_t*>(tD) + (int64_t)k * P.cdf_width;
            S ix = to_state<S>((int32_t)((uint32_t)size * cum) >> P.fp);
            uint32_t low = 0, high = (uint32_t)(size - 1);
            while (high > low) {
              if ((unsigned long long)ix >= (unsigned long long)size) {
                fast = false;
                break;
              }
              if ((int32_t)cum >= row[ix]) low = (uint32_t)ix + 1u;
              else high = (uint32_t)ix;
              ix = (S)((low + high) / 2u);
            }
            const int64_t s = (int64_t)(unsigned long long)(S)(ix - 1);
            if (fast && s >= 0 && s < (int64_t)size - 1) {
              sv = (int32_t)s;
              const int32_t lo_c = row[s], hi_c = row[s + 1];
              freq = (int32_t)((uint32_t)hi_c - (uint32_t)lo_c);
              off = (int32_t)cum - lo_c;
            } else {
              fast = false;
            }
          }
        }
        int32_t v;
        bool ok = true;
        if (fast) {
          x[j] = (S)((x[j] >> P.fp) * to_state<S>(freq) + to_state<S>(off));
          cur[j].refill(x[j]);
          v = sv;
          if constexpr (BYPASS) {
            if (v == ti.size - 2) {
              const int32_t raw = pop_escape<V>(x[j], cur[j].c, P.bp);
              v = raw >> 1;
              v = (raw & 1) ? (-v - 1) : (v + ti.size - 2);
              cur[j].prime();
            }
          }
        } else {
          v = pop_chain<V, LK, BYPASS>(P, x[j], cur[j].c, k, ti, ok);
          cur[j].prime();
        }
        ov[j][q] = ok ? (int32_t)((uint32_t)v + (uint32_t)ti.offset) : 0;
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
    store_state<V>(rows[j], 0, x[j]);
    rows[j][0] = (int32_t)((cur[j].c.p + 1) * VT<V>::WBYTES);
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
    if (tm == TM_FUSED_SMEM) popf_spt<V, 1, BY, TM_FUSED_SMEM>(P, spt, blocks, threads, smem, s);
    else if (tm == TM_SPLIT_SMEM) popf_spt<V, 1, BY, TM_SPLIT_SMEM>(P, spt, blocks, threads, smem, s);
    else if (tm == TM_SPLIT_GLOBAL) popf_spt<V, 1, BY, TM_SPLIT_GLOBAL>(P, spt, blocks, threads, smem, s);
    else return false;
    return true;
  }
  if (tm == TM_FUSED_SMEM) popf_spt<V, 0, BY, TM_FUSED_SMEM>(P, spt, blocks, threads, smem, s);
  else if (tm == TM_SPLIT_SMEM) popf_spt<V, 0, BY, TM_SPLIT_SMEM>(P, spt, blocks, threads, smem, s);
  else if (tm == TM_SPLIT_GLOBAL) popf_spt<V, 0, BY, TM_SPLIT_GLOBAL>(P, spt, blocks, threads, smem, s);
  else if (tm == TM_CDF_SMEM) popf_spt<V, 0, BY, TM_CDF_SMEM>(P, spt, blocks, threads, smem, s);
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
