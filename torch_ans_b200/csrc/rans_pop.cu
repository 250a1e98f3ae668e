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

#include "../../include/torch_ans_b200.h"
#include "launch.cuh"
#include "rans_device.cuh"
#include "rans_host.h"

namespace tans {

__global__ void build_table_info_kernel(const int32_t* sizes, const int32_t* offsets, int64_t ntables, int fp,
                                        TableInfo* out);

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
  const uint32_t* fD;  // fused decode table (nullptr: direct lookups)
  const uint16_t* fS;
  int fused_smem;      // fused table staged in shared memory
  int tin_smem;        // per-table info staged in shared memory
  int vec_out;         // out is 16-byte aligned
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

// Symbol lookup of rans_utils.hpp:401-449 for one cum value of table row `row`: sets s and the
// offset cum - start (alias: cum - alias_start) and the symbol's frequency.  Returns false where
// the reference would index outside the row (then nothing is read out of bounds).
template <int V, int LK>
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
    const int32_t cut_cdf = __ldg(row + at);
    const int32_t other = __ldg(row + at + 1);
    const int32_t self_off = __ldg(row + at + 2);
    const int32_t other_off = __ldg(row + at + 3);
    const bool hi = cum >= cut_cdf;
    s = hi ? other : id;
    cum_off -= hi ? other_off : self_off;
  } else if constexpr (LK == LK_INVCDF) {
    if ((int64_t)size + cum >= cdf_width) return false;
    s = __ldg(row + size + cum);
  } else {
    // probe (cdf_size * cum) >> fp, then bisection on [0, cdf_size - 1] (rans_utils.hpp:427-448)
    S ix = to_state<S>((int32_t)((uint32_t)size * (uint32_t)cum) >> fp);
    uint32_t low = 0, high = (uint32_t)(size - 1);
    while (high > low) {
      if ((unsigned long long)ix >= (unsigned long long)size) return false;
      if (cum >= __ldg(row + ix)) low = (uint32_t)ix + 1u;
      else high = (uint32_t)ix;
      ix = (S)((low + high) / 2u);
    }
    s = (int64_t)(unsigned long long)(S)(ix - 1);
  }
  if (s < 0 || s >= (int64_t)size - 1) return false;
  const int32_t lo_c = __ldg(row + s), hi_c = __ldg(row + s + 1);
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

__device__ __forceinline__ int4 load_idx_chunk(const int32_t* a, int64_t c, int64_t lo, int64_t hi, bool vec) {
  const int64_t g = c * 4;
  if (vec && g >= lo && g + 4 <= hi) return __ldg(reinterpret_cast<const int4*>(a) + c);
  int4 r = make_int4(0, 0, 0, 0);
  if (g >= lo && g < hi) r.x = __ldg(a + g);
  if (g + 1 >= lo && g + 1 < hi) r.y = __ldg(a + g + 1);
  if (g + 2 >= lo && g + 2 < hi) r.z = __ldg(a + g + 2);
  if (g + 3 >= lo && g + 3 < hi) r.w = __ldg(a + g + 3);
  return r;
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
constexpr int64_t kFusedMaxBytes = 128ll << 20;  // fused decode tables up to this size
constexpr int64_t kSmemBudget = 200 * 1024;

static bool fused_enabled(int64_t ntables, int fp) {
  const char* e = std::getenv("TORCH_ANS_B200_FUSED");
  if (e && e[0] == '0') return false;
  return fp <= 16 && ntables * ((int64_t)6 << fp) <= kFusedMaxBytes;
}

size_t pop_workspace_bytes(int variant, int lookup, int64_t ntables, int64_t cdf_width, int fp) {
  (void)variant;
  (void)lookup;
  (void)cdf_width;
  size_t n = align_up((size_t)ntables * sizeof(TableInfo));
  if (fused_enabled(ntables, fp)) {
    const size_t m = (size_t)ntables << fp;
    n += align_up(m * 4) + align_up(m * 2);
  }
  return n;
}

template <int V, int LK, bool BYPASS>
static void launch_pop(const PopParams& P, int interleave, const LaunchShape& L, cudaStream_t s) {
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
static void launch_fused_build(const PopParams& P, int lookup, uint32_t* D, uint16_t* Sx, int sms, cudaStream_t s) {
  const int64_t m = P.ntables << P.fp;
  const int blocks = (int)std::min<int64_t>((m + 255) / 256, 8 * (int64_t)sms);
  if (lookup == TANS_LOOKUP_ALIAS)
    build_fused_kernel<V, LK_ALIAS><<<blocks, 256, 0, s>>>(P.cdfs, P.ntables, P.cdf_width, P.tinfo, P.fp, D, Sx);
  else if (lookup == TANS_LOOKUP_INVCDF)
    build_fused_kernel<V, LK_INVCDF><<<blocks, 256, 0, s>>>(P.cdfs, P.ntables, P.cdf_width, P.tinfo, P.fp, D, Sx);
  else
    build_fused_kernel<V, LK_SEARCH><<<blocks, 256, 0, s>>>(P.cdfs, P.ntables, P.cdf_width, P.tinfo, P.fp, D, Sx);
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
  const bool fused = interleave == 1 && nsym > 0 && fused_enabled(ntables, fp);
  size_t need = align_up((size_t)ntables * sizeof(TableInfo));
  if (fused) need += align_up(((size_t)ntables << fp) * 4) + align_up(((size_t)ntables << fp) * 2);
  void* ws = workspace;
  bool owned = false;
  if (!ws) {
    if (!allow_alloc) return TANS_E_WORKSPACE;
    if (cudaMallocAsync(&ws, need, s) != cudaSuccess) return TANS_E_CUDA;
    owned = true;
  } else if (ws_bytes < need) {
    return TANS_E_WORKSPACE;
  }
  char* wsp = reinterpret_cast<char*>(ws);
  TableInfo* tinfo = reinterpret_cast<TableInfo*>(wsp);
  wsp += align_up((size_t)ntables * sizeof(TableInfo));
  uint32_t* D = nullptr;
  uint16_t* Sx = nullptr;
  if (fused) {
    D = reinterpret_cast<uint32_t*>(wsp);
    wsp += align_up(((size_t)ntables << fp) * 4);
    Sx = reinterpret_cast<uint16_t*>(wsp);
  }
  const int dev_sms = sm_count();
  {
    const int blocks = (int)std::min<int64_t>((ntables + 255) / 256, 4 * (int64_t)dev_sms);
    build_table_info_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(sizes, offsets, ntables, fp, tinfo);
  }
  PopParams P;
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
  P.vec = (reinterpret_cast<uintptr_t>(indexes) & 15u) == 0;
  P.vec_out = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  P.fD = D;
  P.fS = Sx;
  const LaunchShape L = pick_launch(batch, dev_sms);
  P.lanes = L.lanes;
  const int64_t ring = (int64_t)L.threads * POP_RS * 16;
  P.tin_smem = (ntables <= kPopTinfoSmemMax && ring + ntables * 16 <= kSmemBudget) ? 1 : 0;
  P.fused_smem = (fused && ring + (P.tin_smem ? ntables * 16 : 0) + (ntables << fp) * 6 <= kSmemBudget) ? 1 : 0;
  if (fused) {
    if (variant == TANS_RANS64) launch_fused_build<0>(P, lookup, D, Sx, dev_sms, s);
    else if (variant == TANS_RANS32) launch_fused_build<1>(P, lookup, D, Sx, dev_sms, s);
    else launch_fused_build<2>(P, lookup, D, Sx, dev_sms, s);
  }
  if (variant == TANS_RANS64) launch_pop_v<0>(P, lookup, bypass != 0, interleave, L, s);
  else if (variant == TANS_RANS32) launch_pop_v<1>(P, lookup, bypass != 0, interleave, L, s);
  else launch_pop_v<2>(P, lookup, bypass != 0, interleave, L, s);
  if (owned) cudaFreeAsync(ws, s);
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
