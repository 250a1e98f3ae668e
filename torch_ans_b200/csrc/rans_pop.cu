// rans_pop.cu -- decode (pop) kernels and the tans_pop C entry point.
//
// Replaces the reference's rans_pop_indexed_cpu / rans_pop_indexed_cuda
// (torch_ans/rans_cpu.cpp:191-322, torch_ans/rans_cuda.cu:171-286): per stream, symbols are popped
// first-first with the step of torch_ans/rans_utils.hpp:379-532, writing the int32 symbols and
// leaving the row's length and state updated in place.
//
// B200 design: one thread per stream (launch.cuh); table indexes are read with 16-byte vector
// loads four chunks ahead of the chain and the per-table size/offset record one chunk ahead.  The
// symbol lookup itself (bisection, inverse cdf, alias) is on the serial chain by construction.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <string>

#include "../../include/torch_ans_b200.h"
#include "launch.cuh"
#include "rans_device.cuh"
#include "rans_host.h"
#include "rans_pop.cuh"
#include "rans_pop_fast.cuh"
#include "rans_pop_lean.cuh"

namespace tans {

__global__ void build_table_info_kernel(const int32_t* sizes, const int32_t* offsets, int64_t ntables, int fp,
                                        TableInfo* out);

// Fused decode table: for every (table k, cum < 2^fp) the lookup above replayed once per call,
// packed as D = (freq - 1) | (cum_off << 16) and S = s; S = 0xFFFF marks entries that do not pack
// (freq or offset outside 16 bits, s >= 0xFFFF, or a lookup the reference cannot do), for which
// the kernel runs the lookup itself.  Results are therefore identical to the direct lookup.
template <int V, int LK>
__global__ void build_fused_kernel(const int32_t* cdfs, int64_t ntables, int64_t cdf_width, const TableInfo* tinfo,
                                   int fp, uint32_t* D, uint16_t* Sx) {
  const int64_t M = (int64_t)1 << fp, total = ntables * M;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = e >> fp;
    const int32_t cum = (int32_t)(e & (M - 1));
    const TableInfo t = tinfo[k];
    int64_t s;
    int32_t cum_off, freq;
    uint32_t d = 0;
    uint16_t sv = 0xFFFFu;
    if (lookup_symbol<V, LK>(cdfs + k * cdf_width, t, cum, cdf_width, fp, s, cum_off, freq) && s < 0xFFFF &&
        freq >= 1 && freq <= 65536 && cum_off >= 0 && cum_off <= 65535) {
      d = (uint32_t)(freq - 1) | ((uint32_t)cum_off << 16);
      sv = (uint16_t)s;
    }
    D[e] = d;
    Sx[e] = sv;
  }
}

// Split decode tables (inverse-cdf and bisection lookups, whose offset is cum - cdf[s]):
// S[k][cum] = s from the reference's lookup, ST[k][s] = (freq - 1) | start << 16.  S = 0xFFFF where
// the lookup fails or s, freq or start do not pack; those steps take the direct lookup.
template <int V, int LK>
__global__ void build_split_s_kernel(const int32_t* cdfs, int64_t ntables, int64_t cdf_width, const TableInfo* tinfo,
                                     int fp, int64_t st_stride, uint16_t* Sx) {
  const int64_t M = (int64_t)1 << fp, total = ntables * M;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = e >> fp;
    const int32_t cum = (int32_t)(e & (M - 1));
    const TableInfo t = tinfo[k];
    int64_t s;
    int32_t cum_off, freq;
    uint16_t sv = 0xFFFFu;
    if (lookup_symbol<V, LK>(cdfs + k * cdf_width, t, cum, cdf_width, fp, s, cum_off, freq)) {
      const int64_t start = (int64_t)cum - cum_off;
      if (s < st_stride && s < 0xFFFF && freq >= 1 && freq <= 65536 && start >= 0 && start <= 65535) sv = (uint16_t)s;
    }
    Sx[e] = sv;
  }
}

// Bucket table: one 8-byte entry per 16 consecutive cum values of a table,
//   bits  0..15  s0, the symbol of the bucket's first cum (0xFFFF: the entry cannot describe the
//                bucket; those cum values are decoded through the split tables),
//   bits 16..31  c1 - 1, where c1 = start(s0) + freq(s0) is the start of s0 + 1 (it may lie past
//                the bucket),
//   bits 32..47  freq(s0),
//   bits 48..63  freq(s0 + 1) (0 when s0 covers the whole bucket).
// Decode: a cum below c1 is s0 (start c1 - freq(s0)), a cum at or past c1 is s0 + 1 (start c1), so
// at most one boundary lies inside a bucket; "cum >= c1" is the single compare
// (cum << 16) > (bits 0..31).  Every cum of the bucket is checked against the reference lookup when
// the entry is built.  A bucket with more symbols carries a marker (bits 0..15 = 0xFFFF) whose bits
// 16..17 say how the rare step decodes it:
//   0  the exact step (the split tables, or the direct lookup);
//   1  a run of unit-frequency symbols: symbol = cum + (int32)(bits 32..63), freq 1, offset 0;
//   2  a block of 16 per-cum entries s | (cum - start) << 16 | freq << 32 in the secondary table,
//      at block index bits 18..63 (blocks are handed out by an atomic counter up to the table's
//      capacity; the order differs between builds, the decoded values do not).
// One extra row (index ntables) holds only type-0 markers: the decoders route table indexes
// outside the table list to it.
template <int V, int LK>
__global__ void build_bucket_kernel(const int32_t* cdfs, int64_t ntables, int64_t cdf_width, const TableInfo* tinfo,
                                    int fp, unsigned long long* BK, unsigned long long* SEC, int64_t sec_cap,
                                    unsigned long long* sec_count) {
  constexpr int NB = 1 << kBucketBits;
  const int64_t nb = (int64_t)1 << (fp - kBucketBits), total = (ntables + 1) * nb;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = e / nb;
    if (k >= ntables) {
      BK[e] = 0xFFFFull;
      continue;
    }
    const int32_t lo = (int32_t)((e - k * nb) << kBucketBits);
    const TableInfo t = tinfo[k];
    const int32_t* row = cdfs + k * cdf_width;
    int64_t s[NB];
    int32_t off[NB], f[NB];
    bool all = true;
    for (int i = 0; i < NB; ++i) {
      all = all && lookup_symbol<V, LK>(row, t, lo + i, cdf_width, fp, s[i], off[i], f[i]);
      if (!all) break;
    }
    unsigned long long out = 0xFFFFull;
    if (all) {
      const int64_t s0 = s[0];
      const int32_t start0 = lo - off[0], f0 = f[0];
      const int32_t c1 = start0 + f0;
      bool good = s0 >= 0 && s0 < 0xFFFE && start0 >= 0 && start0 <= 0xFFFF && f0 >= 1 && f0 <= 0xFFFF;
      int32_t f1 = 1;
      bool seen1 = false;
      bool unit = true, packs = true;
      for (int i = 0; i < NB; ++i) {
        const int32_t cum = lo + i, st = cum - off[i];
        if (i > 0 && good) {
          if (cum < c1) {
            good = s[i] == s0 && st == start0 && f[i] == f0;
          } else {
            if (!seen1) {
              f1 = f[i];
              seen1 = true;
            }
            good = s[i] == s0 + 1 && st == c1 && f[i] == f1 && f1 >= 1 && f1 <= 0xFFFF;
          }
        }
        unit = unit && f[i] == 1 && off[i] == 0 && s[i] == s0 + i;
        packs = packs && s[i] >= 0 && s[i] < 0xFFFF && off[i] >= 0 && off[i] <= 0xFFFF && f[i] >= 1 && f[i] <= 0x10000;
      }
      if (good) {
        out = (unsigned long long)s0 | ((unsigned long long)(c1 - 1) << 16) | ((unsigned long long)f0 << 32) |
              ((unsigned long long)(seen1 ? f1 : 0) << 48);
      } else if (unit && s0 - lo >= INT32_MIN && s0 - lo <= INT32_MAX) {
        out = 0xFFFFull | (1ull << 16) | ((unsigned long long)(uint32_t)(int32_t)(s0 - lo) << 32);
      } else if (packs && sec_cap > 0) {
        const unsigned long long blk = atomicAdd(sec_count, 1ull);
        if (blk < (unsigned long long)sec_cap) {
          for (int i = 0; i < NB; ++i)
            SEC[blk * NB + i] = (unsigned long long)s[i] | ((unsigned long long)off[i] << 16) |
                                ((unsigned long long)f[i] << 32);
          out = 0xFFFFull | (2ull << 16) | (blk << 18);
        }
      }
    }
    BK[e] = out;
  }
}

// Level-1 table for few streams per SM: one entry per 2^l1b cum values (l1b >= kL1Bits), in the
// bucket format, derived from the (exact) 16-cum entries: a coarse bucket is describable when its
// fine entries all follow one two-symbol model -- a fine bucket before the boundary c1 repeats
// (s0, c1, f0), the one holding c1 adds f1, one past it starts at c1 with symbol s0 + 1 and
// freq f1 and holds no further boundary.  Anything else is a plain marker (the kernel then reads
// the fine entry).
__global__ void build_level1_kernel(const unsigned long long* BK, int64_t ntables, int fp, int l1b,
                                    unsigned long long* L1) {
  const int R = 1 << (l1b - kBucketBits);  // fine entries per coarse entry
  const int64_t nb1 = (int64_t)1 << (fp - l1b), total = (ntables + 1) * nb1;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = e / nb1;
    unsigned long long out = 0xFFFFull;
    if (k < ntables) {
      const int64_t cb = e - k * nb1;
      const unsigned long long* fe = BK + (k << (fp - kBucketBits)) + cb * R;
      const uint32_t base = (uint32_t)(cb << l1b);
      const unsigned long long e0 = fe[0];
      const uint32_t s0 = (uint32_t)(e0 & 0xFFFFu), c1 = (uint32_t)((e0 >> 16) & 0xFFFFu) + 1u,
                     f0 = (uint32_t)((e0 >> 32) & 0xFFFFu);
      uint32_t f1 = 0;
      bool seen1 = false, ok = s0 != 0xFFFFu;
      for (int j = 0; ok && j < R; ++j) {
        const unsigned long long ej = fe[j];
        const uint32_t sj = (uint32_t)(ej & 0xFFFFu), c1j = (uint32_t)((ej >> 16) & 0xFFFFu) + 1u,
                       f0j = (uint32_t)((ej >> 32) & 0xFFFFu), f1j = (uint32_t)(ej >> 48);
        const uint32_t lj = base + ((uint32_t)j << kBucketBits), hj = lj + (1u << kBucketBits) - 1u;
        if (sj == 0xFFFFu) {
          ok = false;
        } else if (hj < c1) {  // before the boundary
          ok = sj == s0 && c1j == c1 && f0j == f0;
        } else if (lj < c1) {  // holds the boundary
          ok = sj == s0 && c1j == c1 && f0j == f0 && f1j != 0u && (!seen1 || f1j == f1);
          f1 = f1j;
          seen1 = true;
        } else {  // past the boundary: symbol s0 + 1 from c1, no boundary of its own
          ok = sj == s0 + 1u && c1j - f0j == c1 && c1j > hj && (!seen1 || f0j == f1);
          f1 = f0j;
          seen1 = true;
        }
      }
      if (ok)
        out = (unsigned long long)s0 | ((unsigned long long)(c1 - 1u) << 16) | ((unsigned long long)f0 << 32) |
              ((unsigned long long)(seen1 ? f1 : 0u) << 48);
    }
    L1[e] = out;
  }
}

__global__ void build_split_st_kernel(const int32_t* cdfs, int64_t ntables, int64_t cdf_width, int64_t st_stride,
                                      uint32_t* ST) {
  const int64_t total = ntables * st_stride;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = e / st_stride, sidx = e - k * st_stride;
    uint32_t v = 0;
    if (sidx + 1 < cdf_width) {
      const int32_t start = cdfs[k * cdf_width + sidx];
      const int32_t freq = (int32_t)((uint32_t)cdfs[k * cdf_width + sidx + 1] - (uint32_t)start);
      v = ((uint32_t)(freq - 1) & 0xFFFFu) | ((uint32_t)start << 16);
    }
    ST[e] = v;
  }
}

template <int V, int LK, bool BYPASS>
__device__ __forceinline__ void pop_elem(const PopParams& P, typename VT<V>::State& x, PopCursor<V>& c, int64_t g,
                                         int64_t lo, int64_t hi, int32_t k, const TableInfo& t) {
  if (g < lo || g >= hi) return;
  if (k < 0 || (int64_t)k >= P.ntables) {
    c.err |= DEV_BAD_INDEX;
    P.out[g] = 0;
    return;
  }
  bool ok;
  const int32_t v = pop_chain<V, LK, BYPASS>(P, x, c, k, t, ok);
  P.out[g] = ok ? (int32_t)((uint32_t)v + (uint32_t)t.offset) : 0;
}

// ---------------------------------------------------------------- single-state kernel
// Table indexes are staged by cp.async into a per-thread shared-memory ring POP_L chunks ahead of
// the chain.  MODE 0 looks symbols up in the caller's tables; MODE 1 reads the fused decode
// table from global memory (L2 evict_last); MODE 2 reads it from shared memory.  Decoded
// symbols are written four at a time (16-byte stores, L2 evict_first) where the chunk allows.
constexpr int POP_RS = 8;
constexpr int POP_L = 6;
constexpr int64_t kPopTinfoSmemMax = 4096;

template <int V, int LK, bool BYPASS, int MODE>
__global__ void __launch_bounds__(256) pop_i1_kernel(const PopParams P) {
  using S = typename VT<V>::State;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  int4* ring = reinterpret_cast<int4*>(smem_raw);
  TableInfo* tsm = reinterpret_cast<TableInfo*>(ring + POP_RS * T);
  uint32_t* sD = reinterpret_cast<uint32_t*>(tsm + (P.tin_smem ? P.ntables : 0));
  const int64_t fused_n = MODE == 2 ? (P.ntables << P.fp) : 0;
  uint16_t* sS = reinterpret_cast<uint16_t*>(sD + fused_n);
  if (P.tin_smem)
    for (int64_t k = tid; k < P.ntables; k += T) tsm[k] = P.tinfo[k];
  if constexpr (MODE == 2) {
    const int4* gD = reinterpret_cast<const int4*>(P.fD);
    int4* dD = reinterpret_cast<int4*>(sD);
    for (int64_t i = tid; i < fused_n / 4; i += T) dD[i] = gD[i];
    for (int64_t i = (fused_n / 4) * 4 + tid; i < fused_n; i += T) sD[i] = P.fD[i];
    for (int64_t i = tid; i < fused_n; i += T) sS[i] = P.fS[i];
  }
  if (P.tin_smem || MODE == 2) __syncthreads();

  const int64_t b = my_stream(P.lanes, P.batch);
  if (b < 0) return;
  int32_t* row = P.stream + b * P.width;
  PopCursor<V> cur;
  cur.payload = reinterpret_cast<const uint8_t*>(row + 1);
  cur.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
  cur.first = VT<V>::SBYTES / VT<V>::WBYTES;
  cur.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
  cur.err = 0;
  S x = load_state<V>(row, 0);
  const unsigned long long pol_keep = policy_evict_last(), pol_stream = policy_evict_first();
  const int64_t lo = b * P.nsym, hi = lo + P.nsym, total = P.batch * P.nsym;
  const bool vec = P.vec != 0;
  const S mask = (S)((1ull << P.fp) - 1ull);

  if (P.nsym > 0) {
    const int64_t c_lo = lo >> 2, c_hi = (hi - 1) >> 2;
    for (int64_t t = 0; t <= (c_hi - c_lo) + POP_L; ++t) {
      const int64_t xr = c_lo + t;
      if (xr <= c_hi) {
        int4* dst = ring + (int)(xr & (POP_RS - 1)) * T + tid;
        const int64_t g = xr * 4;
        if (vec && g + 4 <= total) {
          cp_async16_hint(dst, P.idx + g, pol_stream);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (g + e < total) cp_async4(reinterpret_cast<int32_t*>(dst) + e, P.idx + g + e);
        }
      }
      cp_async_commit();
      cp_async_wait<POP_L - 1>();
      const int64_t xc = xr - POP_L;
      if (xc < c_lo) continue;
      const int4 k4 = ring[(int)(xc & (POP_RS - 1)) * T + tid];
      const int32_t ks[4] = {k4.x, k4.y, k4.z, k4.w};
      int32_t outv[4] = {0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t g = xc * 4 + j;
        if (g < lo || g >= hi) continue;
        const int32_t k = ks[j];
        if (k < 0 || (int64_t)k >= P.ntables) {
          cur.err |= DEV_BAD_INDEX;
          continue;
        }
        const TableInfo ti = P.tin_smem ? tsm[k] : load_tinfo(P.tinfo, k);
        bool ok = false;
        int32_t v = 0;
        if constexpr (MODE == 0) {
          v = pop_chain<V, LK, BYPASS>(P, x, cur, k, ti, ok);
        } else {
          const int64_t e = ((int64_t)k << P.fp) | (int64_t)(uint32_t)(x & mask);
          uint32_t d, sv;
          if constexpr (MODE == 2) {
            d = sD[e];
            sv = sS[e];
          } else {
            d = ld_hint_u32(P.fD + e, pol_keep);
            sv = ld_hint_u16(P.fS + e, pol_keep);
          }
          if (sv == 0xFFFFu) {
            v = pop_chain<V, LK, BYPASS>(P, x, cur, k, ti, ok);
          } else {
            v = pop_finish<V, BYPASS>(P, x, cur, (int32_t)sv, (int32_t)(d >> 16), (int32_t)(d & 0xFFFFu) + 1,
                                      ti.size - 2);
            ok = true;
          }
        }
        outv[j] = ok ? (int32_t)((uint32_t)v + (uint32_t)ti.offset) : 0;
      }
      const int64_t g0 = xc * 4;
      if (P.vec_out && g0 >= lo && g0 + 4 <= hi) {
        st_hint_v4(reinterpret_cast<int4*>(P.out + g0), make_int4(outv[0], outv[1], outv[2], outv[3]), pol_stream);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (g0 + j >= lo && g0 + j < hi) P.out[g0 + j] = outv[j];
      }
    }
    cp_async_wait<0>();
  }
  store_state<V>(row, 0, x);
  row[0] = (int32_t)((cur.p + 1) * VT<V>::WBYTES);
  report(P.status, cur.err);
}

// ---------------------------------------------------------------- four-state (i4) kernel
// rans_cpu.cpp:229-312: blocks [i, i+3] while i < N-3: four symbol pops (state j) without escape,
// then the escapes of the block (state j, j = 0..3); the last N % 4 symbols use state i % 4 with
// inline escapes.
template <int V, int LK, bool BYPASS>
__global__ void __launch_bounds__(256) pop_i4_kernel(const PopParams P) {
  using S = typename VT<V>::State;
  const int64_t b = my_stream(P.lanes, P.batch);
  if (b < 0) return;
  int32_t* row = P.stream + b * P.width;
  PopCursor<V> cur;
  cur.payload = reinterpret_cast<const uint8_t*>(row + 1);
  cur.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
  cur.first = 4 * VT<V>::SBYTES / VT<V>::WBYTES;
  cur.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
  cur.err = 0;
  S x[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) x[k] = load_state<V>(row, k);
  const int64_t base = b * P.nsym, N = P.nsym;
  int64_t i = 0;
  for (; i < N - 3; i += 4) {
    int32_t kk[4];
    TableInfo tt[4];
    bool ok[4];
    int32_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      kk[j] = __ldg(P.idx + base + i + j);
      tt[j] = tinfo_or_zero(P, kk[j], true);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (kk[j] < 0 || (int64_t)kk[j] >= P.ntables) {
        cur.err |= DEV_BAD_INDEX;
        ok[j] = false;
        v[j] = 0;
        continue;
      }
      v[j] = pop_chain<V, LK, false>(P, x[j], cur, kk[j], tt[j], ok[j]);
    }
    if constexpr (BYPASS) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (ok[j] && v[j] == tt[j].size - 2) {
          const int32_t raw = pop_escape<V>(x[j], cur, P.bp);
          const int32_t h = raw >> 1;
          v[j] = (raw & 1) ? (-h - 1) : (h + tt[j].size - 2);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      P.out[base + i + j] = ok[j] ? (int32_t)((uint32_t)v[j] + (uint32_t)tt[j].offset) : 0;
  }
  for (; i < N; ++i) {
    const int32_t k = __ldg(P.idx + base + i);
    const TableInfo t = tinfo_or_zero(P, k, true);
    switch (i & 3) {
      case 0: pop_elem<V, LK, BYPASS>(P, x[0], cur, base + i, base, base + N, k, t); break;
      case 1: pop_elem<V, LK, BYPASS>(P, x[1], cur, base + i, base, base + N, k, t); break;
      case 2: pop_elem<V, LK, BYPASS>(P, x[2], cur, base + i, base, base + N, k, t); break;
      default: pop_elem<V, LK, BYPASS>(P, x[3], cur, base + i, base, base + N, k, t); break;
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) store_state<V>(row, k, x[k]);
  row[0] = (int32_t)((cur.p + 1) * VT<V>::WBYTES);
  report(P.status, cur.err);
}

// ---------------------------------------------------------------- host side
constexpr int64_t kFusedMaxBytes = 128ll << 20;  // fused tables in global memory up to this size
constexpr int64_t kSplitMaxBytes = 256ll << 20;  // split tables in global memory up to this size
constexpr int64_t kSmemBudget = 200 * 1024;

static int64_t split_stride(int lookup, int64_t cdf_width, int fp) {
  // entries per table in ST: the cdf part of a row (an inverse-cdf row is [cdf | 2^fp inverse])
  int64_t w = lookup == TANS_LOOKUP_INVCDF ? cdf_width - ((int64_t)1 << fp) : cdf_width;
  if (w < 2) w = 2;
  const int64_t cap = ((int64_t)1 << fp) + 1;
  return std::min(w - 1, cap);
}

static int64_t fused_bytes(int64_t ntables, int fp) { return ntables * ((int64_t)6 << fp); }
static int64_t split_bytes(int lookup, int64_t ntables, int64_t cdf_width, int fp) {
  return ntables * ((int64_t)2 << fp) + ntables * split_stride(lookup, cdf_width, fp) * 4;
}

// bucket table: ntables + 1 rows (the last one all markers) of 2^(fp-1) bytes, the first row
// aligned to a row's size (so a row address plus an offset inside the row needs no carry); then a
// 256-byte counter slot and the secondary table of per-cum blocks (128 bytes each) for marker
// buckets, with room for one bucket in 16
static int64_t bucket_row_bytes(int fp) { return (int64_t)8 << (fp - kBucketBits); }
static int64_t bucket_sec_cap(int64_t ntables, int fp) {
  return std::max<int64_t>(64, (ntables << (fp - kBucketBits)) / 16);
}
static int64_t bucket_bytes(int64_t ntables, int fp) {
  return fp >= kBucketBits
             ? (ntables + 2) * bucket_row_bytes(fp) + 256 + bucket_sec_cap(ntables, fp) * (8 << kBucketBits)
             : 0;
}
// level-1 table (ntables + 1 rows of 2^(fp - kL1Bits) entries), padded to 16 bytes
static int64_t level1_bytes(int64_t ntables, int fp, int bits = kL1Bits) {
  return fp >= bits ? (((ntables + 1) * ((int64_t)8 << (fp - bits))) + 15) & ~(int64_t)15 : 0;
}

static bool tables_enabled() {
  const char* e = std::getenv("TORCH_ANS_B200_FUSED");
  return !(e && e[0] == '0');
}

size_t pop_workspace_bytes(int variant, int lookup, int64_t ntables, int64_t cdf_width, int fp) {
  (void)variant;
  size_t n = align_up((size_t)ntables * sizeof(TableInfo));
  if (fp <= 16 && tables_enabled()) {
    size_t extra = 0;
    if (fused_bytes(ntables, fp) <= kFusedMaxBytes)
      extra = align_up((size_t)(ntables << fp) * 4) + align_up((size_t)(ntables << fp) * 2);
    if (lookup != TANS_LOOKUP_ALIAS && split_bytes(lookup, ntables, cdf_width, fp) <= kSplitMaxBytes)
      extra = std::max(extra, align_up((size_t)(ntables << fp) * 2) +
                                  align_up((size_t)ntables * split_stride(lookup, cdf_width, fp) * 4) +
                                  align_up((size_t)bucket_bytes(ntables, fp)) +
                                  align_up((size_t)level1_bytes(ntables, fp)));
    n += extra;
  }
  return n;
}

template <int V, int LK, bool BYPASS>
static void launch_pop(const PopParams& P, int interleave, const LaunchShape& L, cudaStream_t s) {
  note_launch();
  if (interleave == 4) {
    pop_i4_kernel<V, LK, BYPASS><<<L.blocks, L.threads, 0, s>>>(P);
    return;
  }
  size_t smem = (size_t)L.threads * POP_RS * 16 + (P.tin_smem ? (size_t)P.ntables * sizeof(TableInfo) : 0);
  if (P.fD && P.fused_smem) {
    smem += (size_t)(P.ntables << P.fp) * 6;
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(pop_i1_kernel<V, LK, BYPASS, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    pop_i1_kernel<V, LK, BYPASS, 2><<<L.blocks, L.threads, smem, s>>>(P);
  } else if (P.fD) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(pop_i1_kernel<V, LK, BYPASS, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    pop_i1_kernel<V, LK, BYPASS, 1><<<L.blocks, L.threads, smem, s>>>(P);
  } else {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(pop_i1_kernel<V, LK, BYPASS, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    pop_i1_kernel<V, LK, BYPASS, 0><<<L.blocks, L.threads, smem, s>>>(P);
  }
}

template <int V>
static void launch_pop_v(const PopParams& P, int lookup, bool bypass, int interleave, const LaunchShape& L,
                         cudaStream_t s) {
  if (lookup == TANS_LOOKUP_ALIAS) {
    if (bypass) launch_pop<V, LK_ALIAS, true>(P, interleave, L, s);
    else launch_pop<V, LK_ALIAS, false>(P, interleave, L, s);
  } else if (lookup == TANS_LOOKUP_INVCDF) {
    if (bypass) launch_pop<V, LK_INVCDF, true>(P, interleave, L, s);
    else launch_pop<V, LK_INVCDF, false>(P, interleave, L, s);
  } else {
    if (bypass) launch_pop<V, LK_SEARCH, true>(P, interleave, L, s);
    else launch_pop<V, LK_SEARCH, false>(P, interleave, L, s);
  }
}

template <int V>
static void build_tables(const PopParams& P, int lookup, bool fused, uint32_t* D, uint16_t* Sx, uint32_t* ST,
                         int sms, cudaStream_t s) {
  const int64_t m = P.ntables << P.fp;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((m + 255) / 256, 8 * (int64_t)sms));
  note_launch();
  if (fused) {
    if (lookup == TANS_LOOKUP_ALIAS)
      build_fused_kernel<V, LK_ALIAS><<<blocks, 256, 0, s>>>(P.cdfs, P.ntables, P.cdf_width, P.tinfo, P.fp, D, Sx);
    else if (lookup == TANS_LOOKUP_INVCDF)
      build_fused_kernel<V, LK_INVCDF><<<blocks, 256, 0, s>>>(P.cdfs, P.ntables, P.cdf_width, P.tinfo, P.fp, D, Sx);
    else
      build_fused_kernel<V, LK_SEARCH><<<blocks, 256, 0, s>>>(P.cdfs, P.ntables, P.cdf_width, P.tinfo, P.fp, D, Sx);
    return;
  }
  if (lookup == TANS_LOOKUP_INVCDF)
    build_split_s_kernel<V, LK_INVCDF><<<blocks, 256, 0, s>>>(P.cdfs, P.ntables, P.cdf_width, P.tinfo, P.fp,
                                                              P.st_stride, Sx);
  else
    build_split_s_kernel<V, LK_SEARCH><<<blocks, 256, 0, s>>>(P.cdfs, P.ntables, P.cdf_width, P.tinfo, P.fp,
                                                              P.st_stride, Sx);
  const int64_t n = P.ntables * P.st_stride;
  const int b2 = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 8 * (int64_t)sms));
  build_split_st_kernel<<<b2, 256, 0, s>>>(P.cdfs, P.ntables, P.cdf_width, P.st_stride, ST);
  note_launch();
}

// launch shape of the fast kernel: streams spread over all SMs, up to 4 warps per SM, then up to
// 4 streams per thread, then more lanes
static LaunchShape fast_shape(int64_t streams, int sms, int& spt) {
  // lanes of a warp run their chains in lockstep for free, so one stream per thread is the
  // default; TORCH_ANS_B200_POP_WARPS / _LANES / _SPT override the shape for tuning
  LaunchShape L{1, 32, 1};
  const int64_t per_sm = (streams + sms - 1) / sms;
  int64_t sp = 1;
  const int spt_env = env_int("TORCH_ANS_B200_SPT", 0);
  if (spt_env == 1 || spt_env == 2 || spt_env == 4) sp = spt_env;
  const int64_t threads_sm = (per_sm + sp - 1) / sp;
  // measured on B200 (8,192 streams, 55 per SM): 16 warps x 4 lanes beat 4 x 14 by 1.3x, since a
  // warp's step is one dependent L2 access and more warps per scheduler overlap those waits
  int64_t warps = std::min<int64_t>(threads_sm, env_int("TORCH_ANS_B200_POP_WARPS", 16));
  if (warps < 1) warps = 1;
  int64_t lanes = (threads_sm + warps - 1) / warps;
  if (lanes > 32) {
    lanes = 32;
    warps = std::min<int64_t>(16, (threads_sm + 31) / 32);
  }
  const int lanes_env = env_int("TORCH_ANS_B200_POP_LANES", 0);
  if (lanes_env > 0 && lanes_env <= 32) lanes = lanes_env;
  // trim the warp count to the lanes actually needed so that the blocks cover every SM
  // (55.4 streams per SM as 14 warps x 4 lanes: 147 blocks rather than 128 blocks of 16 x 4)
  warps = std::max<int64_t>(1, std::min<int64_t>(warps, (threads_sm + lanes - 1) / lanes));
  spt = (int)sp;
  L.lanes = (int)lanes;
  L.threads = (int)(warps * 32);
  L.blocks = (int)((streams + warps * lanes * sp - 1) / (warps * lanes * sp));
  return L;
}

// launch shape of the lean kernel: one stream per thread, streams spread over every SM
static LaunchShape lean_shape(int64_t streams, int sms) {
  LaunchShape L{1, 32, 1};
  const int64_t per_sm = (streams + sms - 1) / sms;
  int64_t warps = std::min<int64_t>(per_sm, env_int("TORCH_ANS_B200_POPL_WARPS", 16));
  warps = std::max<int64_t>(1, std::min<int64_t>(warps, 16));
  int64_t lanes = std::min<int64_t>(32, (per_sm + warps - 1) / warps);
  const int lanes_env = env_int("TORCH_ANS_B200_POPL_LANES", 0);
  if (lanes_env > 0 && lanes_env <= 32) lanes = lanes_env;
  warps = std::max<int64_t>(1, std::min<int64_t>(16, (per_sm + lanes - 1) / lanes));
  L.lanes = (int)lanes;
  L.threads = (int)(warps * 32);
  L.blocks = (int)((streams + warps * lanes - 1) / (warps * lanes));
  return L;
}

// TORCH_ANS_B200_POP_KERNEL: unset = the lean kernel for tables in L2 read per step (bucket,
// split), the fast kernel for tables in shared memory and the fused table (short table latency,
// so per-step overhead dominates and its branch-free chunks measured faster); "lean", "fast"
// (several streams per thread) or "generic" force one
static int pop_kernel_choice() {
  const char* e = std::getenv("TORCH_ANS_B200_POP_KERNEL");
  if (!e || !*e) return 0;
  const std::string v(e);
  if (v == "fast") return 1;
  if (v == "generic") return 2;
  if (v == "lean") return 3;
  return 0;
}

static int layout_override() {
  const char* e = std::getenv("TORCH_ANS_B200_POP_LAYOUT");
  if (!e || !*e) return -1;
  const std::string v(e);
  if (v == "fused_smem") return TM_FUSED_SMEM;
  if (v == "fused_global") return TM_FUSED_GLOBAL;
  if (v == "split_smem") return TM_SPLIT_SMEM;
  if (v == "split_global") return TM_SPLIT_GLOBAL;
  if (v == "bucket_global") return TM_BUCKET_GLOBAL;
  if (v == "generic") return 100;
  return -1;
}

int pop_impl(int variant, int lookup, int interleave, int32_t* stream, int64_t batch, int64_t width, int32_t* out,
             const int32_t* indexes, int64_t nsym, const int32_t* cdfs, int64_t ntables, int64_t cdf_width,
             const int32_t* sizes, const int32_t* offsets, int fp, int bypass, int bp, void* workspace,
             size_t ws_bytes, uint32_t* status, cudaStream_t s, bool allow_alloc) {
  int rc = check_coding_args(variant, interleave, stream, batch, width, indexes, nsym, cdfs, ntables, cdf_width,
                             sizes, fp, bypass, bp);
  if (rc != TANS_OK) return rc;
  if (lookup < 0 || lookup > 2) return TANS_E_INVALID_ARGUMENT;
  if (nsym > 0 && !out) return TANS_E_INVALID_ARGUMENT;
  if (batch == 0) return TANS_OK;
  const int dev_sms = sm_count();
  const bool vec_idx = (reinterpret_cast<uintptr_t>(indexes) & 15u) == 0;
  const bool vec_out = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  const bool use_tables = interleave == 1 && nsym > 0 && fp <= 16 && tables_enabled();
  const int64_t sstride = split_stride(lookup, cdf_width, fp);

  // ---- plan: fast kernel + table layout, or the generic kernel
  int tm = -1, spt = 1;
  LaunchShape L{};
  size_t smem = 0;
  bool tin_smem = false;
  const int kchoice = pop_kernel_choice();
  const int ov = kchoice == 2 ? 100 : layout_override();
  bool lean = kchoice == 0 || kchoice == 3;
  if (use_tables && ov != 100 && nsym % 4 == 0 && vec_idx && vec_out && nsym / 4 < 0x7fffffff) {
    L = lean ? lean_shape(batch, dev_sms) : fast_shape(batch, dev_sms, spt);
    const int64_t ring = lean ? 0 : (int64_t)(L.threads / 32) * L.lanes * POPF_RS * 16 * spt;
    tin_smem = true;  // the fast kernel always stages the per-table info
    const int64_t avail = (ntables <= 4096) ? kSmemBudget - ring : -1;
    auto fits = [&](int t) {
      switch (t) {
        case TM_FUSED_SMEM: return popf_table_smem(t, ntables, fp, cdf_width, sstride) <= avail;
        case TM_SPLIT_SMEM:
          return lookup != TANS_LOOKUP_ALIAS && popf_table_smem(t, ntables, fp, cdf_width, sstride) <= avail;
        case TM_FUSED_GLOBAL:
          return lookup == TANS_LOOKUP_ALIAS && popf_table_smem(t, ntables, fp, cdf_width, sstride) <= avail &&
                 fused_bytes(ntables, fp) <= kFusedMaxBytes;
        case TM_SPLIT_GLOBAL:
          return lookup != TANS_LOOKUP_ALIAS && popf_table_smem(t, ntables, fp, cdf_width, sstride) <= avail &&
                 split_bytes(lookup, ntables, cdf_width, fp) <= kSplitMaxBytes;
        case TM_BUCKET_GLOBAL:
          return lookup != TANS_LOOKUP_ALIAS && fp >= kBucketBits &&
                 popf_table_smem(t, ntables, fp, cdf_width, sstride) <= avail &&
                 split_bytes(lookup, ntables, cdf_width, fp) <= kSplitMaxBytes;
      }
      return false;
    };
    if (ov >= 0 && fits(ov)) tm = ov;
    else {
      const int order[5] = {TM_FUSED_SMEM, TM_SPLIT_SMEM, TM_FUSED_GLOBAL, TM_BUCKET_GLOBAL, TM_SPLIT_GLOBAL};
      for (int t : order)
        if (fits(t)) {
          tm = t;
          break;
        }
    }
    // alias tables in shared memory with at least one stream per SM: the lean kernel with its index
    // ring (zipf_alias, 1,024 streams: 24.4 vs 28.1 ms for the fast kernel at a quarter length)
    const bool lean_fused = tm == TM_FUSED_SMEM && lookup == TANS_LOOKUP_ALIAS && batch >= (int64_t)dev_sms;
    if ((tm == TM_FUSED_GLOBAL || tm == TM_FUSED_SMEM || tm == TM_SPLIT_SMEM) && kchoice == 0 && !lean_fused) {
      // the fast kernel for this layout; its index ring must fit beside the table info too
      int spt2 = 1;
      const LaunchShape L2 = fast_shape(batch, dev_sms, spt2);
      const int64_t ring2 = (int64_t)(L2.threads / 32) * L2.lanes * POPF_RS * 16 * spt2;
      if (ring2 + popf_table_smem(tm, ntables, fp, cdf_width, sstride) <= kSmemBudget) {
        lean = false;
        L = L2;
        spt = spt2;
        smem = (size_t)ring2 + (size_t)popf_table_smem(tm, ntables, fp, cdf_width, sstride);
      } else {
        smem = (size_t)ring + (size_t)popf_table_smem(tm, ntables, fp, cdf_width, sstride);
      }
    } else if (tm >= 0) {
      smem = (size_t)ring + (size_t)popf_table_smem(tm, ntables, fp, cdf_width, sstride);
    }
  }
  // level-1 table in shared memory in front of the bucket table, one entry per 2^l1_bits cum
  // values (the finest granularity from 2^kL1Bits up that fits beside the records): chosen for at
  // most two streams per SM (one lane per warp, so a level-1 miss costs only its own lane) with
  // entries of at most 2^kL1AutoBits cum values.  Coarser entries are exact for fewer steps (the
  // mixture tables at 2^10: 54 % of steps; the level-1 pop then measured slower than the bucket
  // pop at 1,024 streams).  TORCH_ANS_B200_POP_L1=0|1 forces it off or on,
  // TORCH_ANS_B200_POP_L1_BITS a granularity
  bool use_l1 = false;
  int l1_bits = kL1Bits;
  if (tm == TM_BUCKET_GLOBAL && lean && fp >= kL1Bits) {
    const int env_l1 = env_int("TORCH_ANS_B200_POP_L1", -1);
    const int env_bits = env_int("TORCH_ANS_B200_POP_L1_BITS", 0);
    if (env_bits >= kL1Bits && env_bits <= fp) {
      l1_bits = env_bits;
    } else {
      while (l1_bits < fp && (int64_t)smem + 16 + level1_bytes(ntables, fp, l1_bits) > kSmemBudget) ++l1_bits;
    }
    const bool fits = (int64_t)smem + 16 + level1_bytes(ntables, fp, l1_bits) <= kSmemBudget;
    const bool auto_on = batch <= 2 * (int64_t)dev_sms && l1_bits <= kL1AutoBits;
    use_l1 = fits && (env_l1 == 1 || (env_l1 != 0 && auto_on));
    if (use_l1) smem += 16 + (size_t)level1_bytes(ntables, fp, l1_bits);
  }
  // index ring of the bucket kernel (its bucket and fused-shared launches): per stream two halves
  // of kRingChunks index chunks and two mbarriers, after everything else in shared memory, when
  // it fits; not with the level-1 table for rans32 (byte words), where it measured slower
  // (gaussian_latent pop 9.06 vs 7.09 ms; laplace64, rans64 with the level-1 table: 5.53 with
  // the ring vs 6.29 ms without).  TORCH_ANS_B200_POP_IRING=0|1 forces plain loads or the ring.
  int64_t iring_off = 0;
  bool iring = false;
  const int env_ir = env_int("TORCH_ANS_B200_POP_IRING", -1);
  const bool want_ring = env_ir == 1 || (env_ir != 0 && !(use_l1 && variant == TANS_RANS32));
  if (lean && (tm == TM_BUCKET_GLOBAL || tm == TM_FUSED_SMEM) && want_ring) {
    const int64_t nsl = (int64_t)(L.threads / 32) * L.lanes;
    const int64_t off = ((int64_t)smem + 15) & ~(int64_t)15;
    if (off + nsl * kRingBytesPerStream <= kSmemBudget) {
      iring = true;
      iring_off = off;
      smem = (size_t)(off + nsl * kRingBytesPerStream);
    }
  }
  const bool fast = tm >= 0;
  const bool need_fused = fast ? (tm == TM_FUSED_SMEM || tm == TM_FUSED_GLOBAL)
                               : (use_tables && ov != 100 && fused_bytes(ntables, fp) <= kFusedMaxBytes);
  const bool need_split = fast && (tm == TM_SPLIT_SMEM || tm == TM_SPLIT_GLOBAL || tm == TM_BUCKET_GLOBAL);
  const bool need_bucket = fast && tm == TM_BUCKET_GLOBAL;

  size_t need = align_up((size_t)ntables * sizeof(TableInfo));
  if (need_fused) need += align_up((size_t)(ntables << fp) * 4) + align_up((size_t)(ntables << fp) * 2);
  if (need_split) need += align_up((size_t)(ntables << fp) * 2) + align_up((size_t)ntables * sstride * 4);
  if (need_bucket) need += align_up((size_t)bucket_bytes(ntables, fp));
  if (use_l1) need += align_up((size_t)level1_bytes(ntables, fp, l1_bits));
  void* ws = workspace;
  bool owned = false;
  if (!ws && need > 0) {  // an empty table list needs no scratch at all
    if (!allow_alloc) return TANS_E_WORKSPACE;
    if (cudaMallocAsync(&ws, need, s) != cudaSuccess) return TANS_E_CUDA;
    owned = true;
  } else if (ws_bytes < need) {
    return TANS_E_WORKSPACE;
  }
  char* wsp = reinterpret_cast<char*>(ws);
  TableInfo* tinfo = reinterpret_cast<TableInfo*>(wsp);
  wsp += align_up((size_t)ntables * sizeof(TableInfo));
  PopParams P{};
  P.stream = stream;
  P.batch = batch;
  P.width = width;
  P.out = out;
  P.idx = indexes;
  P.nsym = nsym;
  P.cdfs = cdfs;
  P.ntables = ntables;
  P.cdf_width = cdf_width;
  P.tinfo = tinfo;
  P.fp = fp;
  P.bp = bp;
  P.status = status;
  P.vec = vec_idx;
  P.vec_out = vec_out;
  P.st_stride = sstride;
  if (need_fused) {
    P.fD = reinterpret_cast<uint32_t*>(wsp);
    wsp += align_up((size_t)(ntables << fp) * 4);
    P.fS = reinterpret_cast<uint16_t*>(wsp);
  } else if (need_split) {
    P.fS = reinterpret_cast<uint16_t*>(wsp);
    wsp += align_up((size_t)(ntables << fp) * 2);
    P.fST = reinterpret_cast<uint32_t*>(wsp);
    wsp += align_up((size_t)ntables * sstride * 4);
    if (need_bucket) {
      const uintptr_t rb = (uintptr_t)bucket_row_bytes(fp);
      P.fBK = reinterpret_cast<unsigned long long*>((reinterpret_cast<uintptr_t>(wsp) + rb - 1) & ~(rb - 1));
      char* after = reinterpret_cast<char*>(const_cast<unsigned long long*>(P.fBK)) + (ntables + 1) * rb;
      P.fSEC = reinterpret_cast<unsigned long long*>(after + 256);
      P.sec_cap = bucket_sec_cap(ntables, fp);
      wsp += align_up((size_t)bucket_bytes(ntables, fp));
      if (use_l1) {
        P.fL1 = reinterpret_cast<unsigned long long*>(wsp);
        P.l1_bytes = level1_bytes(ntables, fp, l1_bits);
        P.l1_bits = l1_bits;
      }
    }
  }
  {
    const int blocks = (int)std::min<int64_t>((ntables + 255) / 256, 4 * (int64_t)dev_sms);
    build_table_info_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(sizes, offsets, ntables, fp, tinfo);
    note_launch();
  }
  if (need_fused || need_split) {
    uint32_t* D = const_cast<uint32_t*>(P.fD);
    uint16_t* Sx = const_cast<uint16_t*>(P.fS);
    uint32_t* ST = const_cast<uint32_t*>(P.fST);
    if (variant == TANS_RANS64) build_tables<0>(P, lookup, need_fused, D, Sx, ST, dev_sms, s);
    else if (variant == TANS_RANS32) build_tables<1>(P, lookup, need_fused, D, Sx, ST, dev_sms, s);
    else build_tables<2>(P, lookup, need_fused, D, Sx, ST, dev_sms, s);
  }
  if (need_bucket) {
    unsigned long long* BK = const_cast<unsigned long long*>(P.fBK);
    unsigned long long* SEC = const_cast<unsigned long long*>(P.fSEC);
    unsigned long long* cnt = SEC - 32;  // the counter slot before the secondary table
    // without a zeroed counter no secondary blocks are handed out (type-2 buckets stay type 0)
    const int64_t sc = cudaMemsetAsync(cnt, 0, sizeof(unsigned long long), s) == cudaSuccess ? P.sec_cap : 0;
    const int64_t nbk = (ntables + 1) << (fp - kBucketBits);
    const int bb = (int)std::max<int64_t>(1, std::min<int64_t>((nbk + 127) / 128, 16 * (int64_t)dev_sms));
    note_launch();
    if (lookup == TANS_LOOKUP_INVCDF) {
      if (variant == TANS_RANS64) build_bucket_kernel<0, LK_INVCDF><<<bb, 128, 0, s>>>(cdfs, ntables, cdf_width, tinfo, fp, BK, SEC, sc, cnt);
      else if (variant == TANS_RANS32) build_bucket_kernel<1, LK_INVCDF><<<bb, 128, 0, s>>>(cdfs, ntables, cdf_width, tinfo, fp, BK, SEC, sc, cnt);
      else build_bucket_kernel<2, LK_INVCDF><<<bb, 128, 0, s>>>(cdfs, ntables, cdf_width, tinfo, fp, BK, SEC, sc, cnt);
    } else {
      if (variant == TANS_RANS64) build_bucket_kernel<0, LK_SEARCH><<<bb, 128, 0, s>>>(cdfs, ntables, cdf_width, tinfo, fp, BK, SEC, sc, cnt);
      else if (variant == TANS_RANS32) build_bucket_kernel<1, LK_SEARCH><<<bb, 128, 0, s>>>(cdfs, ntables, cdf_width, tinfo, fp, BK, SEC, sc, cnt);
      else build_bucket_kernel<2, LK_SEARCH><<<bb, 128, 0, s>>>(cdfs, ntables, cdf_width, tinfo, fp, BK, SEC, sc, cnt);
    }
    if (use_l1) {
      const int64_t n1 = (ntables + 1) << (fp - l1_bits);
      const int b1 = (int)std::max<int64_t>(1, std::min<int64_t>((n1 + 127) / 128, 16 * (int64_t)dev_sms));
      build_level1_kernel<<<b1, 128, 0, s>>>(BK, ntables, fp, l1_bits, const_cast<unsigned long long*>(P.fL1));
      note_launch();
    }
  }
  if (fast) {
    P.lanes = L.lanes;
    P.tin_smem = tin_smem ? 1 : 0;
    P.spt = spt;
    P.iring = iring ? 1 : 0;
    P.iring_off = iring_off;
    bool launched;
    if (lean) {
      if (variant == TANS_RANS64) launched = launch_pop_lean<0>(P, lookup, bypass != 0, tm, L.blocks, L.threads, smem, s);
      else if (variant == TANS_RANS32) launched = launch_pop_lean<1>(P, lookup, bypass != 0, tm, L.blocks, L.threads, smem, s);
      else launched = launch_pop_lean<2>(P, lookup, bypass != 0, tm, L.blocks, L.threads, smem, s);
    } else if (variant == TANS_RANS64) launched = launch_pop_fast<0>(P, lookup, bypass != 0, tm, spt, L.blocks, L.threads, smem, s);
    else if (variant == TANS_RANS32) launched = launch_pop_fast<1>(P, lookup, bypass != 0, tm, spt, L.blocks, L.threads, smem, s);
    else launched = launch_pop_fast<2>(P, lookup, bypass != 0, tm, spt, L.blocks, L.threads, smem, s);
    if (!launched) rc = TANS_E_INVALID_ARGUMENT;
  } else {
    L = pick_launch(batch, dev_sms);
    P.lanes = L.lanes;
    const int64_t ring = (int64_t)L.threads * POP_RS * 16;
    P.tin_smem = (ntables <= kPopTinfoSmemMax && ring + ntables * 16 <= kSmemBudget) ? 1 : 0;
    P.fused_smem =
        (P.fD && ring + (P.tin_smem ? ntables * 16 : 0) + (ntables << fp) * 6 <= kSmemBudget) ? 1 : 0;
    if (variant == TANS_RANS64) launch_pop_v<0>(P, lookup, bypass != 0, interleave, L, s);
    else if (variant == TANS_RANS32) launch_pop_v<1>(P, lookup, bypass != 0, interleave, L, s);
    else launch_pop_v<2>(P, lookup, bypass != 0, interleave, L, s);
  }
  if (owned) cudaFreeAsync(ws, s);
  if (rc != TANS_OK) return rc;
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}

}  // namespace tans

extern "C" size_t tans_pop_workspace_size(int variant, int lookup, int64_t num_tables, int64_t cdf_width,
                                          int freq_precision) {
  return tans::pop_workspace_bytes(variant, lookup, num_tables, cdf_width, freq_precision);
}

extern "C" int tans_pop(int variant, int lookup, int num_interleaves, int32_t* stream, int64_t batch,
                        int64_t stream_width, int32_t* out_symbols, const int32_t* indexes, int64_t num_symbols,
                        const int32_t* cdfs, int64_t num_tables, int64_t cdf_width, const int32_t* cdf_sizes,
                        const int32_t* offsets, int freq_precision, int bypass_coding, int bypass_precision,
                        void* workspace, size_t workspace_bytes, uint32_t* dev_status, void* cuda_stream) {
  return tans::pop_impl(variant, lookup, num_interleaves, stream, batch, stream_width, out_symbols, indexes,
                        num_symbols, cdfs, num_tables, cdf_width, cdf_sizes, offsets, freq_precision, bypass_coding,
                        bypass_precision, workspace, workspace_bytes, dev_status,
                        reinterpret_cast<cudaStream_t>(cuda_stream), true);
}
