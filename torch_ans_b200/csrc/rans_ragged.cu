// rans_ragged.cu -- ragged coding: streams of different lengths over one flat symbol array, each
// symbol with its own table row if wanted (tans_push_ragged / tans_pop_ragged).
//
// The reference codes rectangular (batch, N) tensors only; per-element distributions (every
// symbol its own cdf row, the pattern of TorchANSInterface.encode_with_freqs, utils.py:704-760)
// over streams of different lengths take one reference call per stream (B = 1, indexes
// arange(n_b), tables = that stream's rows).  Here stream b codes symbols
// [row_starts[b], row_starts[b+1]) of the flat array with table indexes[i] (or table i when
// indexes is NULL), and its row holds exactly the bytes that per-stream call produces.
//
// push: a fully parallel prep pass resolves every symbol to its encode entry (reciprocal, freq,
//   start, escape value, flags) straight from its table row -- per-element tables are used once,
//   so a per-table entry table would cost more than it saves -- then one thread per stream runs
//   the serial chain over its entries (last symbol first), prefetched by cp.async.
// pop: one thread per stream; table indexes are fetched D1 + D2 steps ahead and each step's table
//   row (with its size and offset) is copied into a per-thread shared-memory ring D2 steps ahead,
//   so the bisection of rans_utils.hpp:424-450 reads shared memory only.
#include <cuda_runtime.h>

#include <algorithm>

#include "../../include/torch_ans_b200.h"
#include "launch.cuh"
#include "rans_device.cuh"
#include "rans_host.h"
#include "rans_pop.cuh"
#include "rans_push_common.cuh"

namespace tans {

struct RaggedArgs {
  int32_t* stream;
  int64_t batch, width;
  const int32_t* sym;     // push: flat symbols
  int32_t* out;           // pop: flat decoded symbols
  const int32_t* idx;     // flat table indexes or nullptr (symbol i uses table i)
  const int64_t* rows;    // batch + 1 row starts
  int64_t total;
  const int32_t* cdfs;
  int64_t ntables, cdf_width;
  const int32_t* sizes;
  const int32_t* offsets;  // or nullptr
  int fp, bp;
  uint32_t* status;
  uint4* ent;  // push workspace: per-symbol entry
  int2* aux;   // push workspace: per-symbol {escape value, flags}
};

__device__ __forceinline__ bool ragged_row(const RaggedArgs& R, int64_t b, int64_t& lo, int64_t& hi) {
  lo = R.rows[b];
  hi = R.rows[b + 1];
  return lo >= 0 && hi >= lo && hi <= R.total;
}

// ---------------------------------------------------------------- push
// per symbol: the work of push_prepare (rans_utils.hpp:186-215) plus the entry the push builds
// per table elsewhere (reciprocal of freq, start), from the symbol's own row
// LEAN (32-bit states, no bypass coding): the chain's own entry {reciprocal m, (2^fp - freq) |
// (l - 1) << 24, bound = freq << (31 - fp), start}, with bit 31 of y set (and the rest unused) when
// the step must take the exact code (flags, freq < 2 or freq > 2^fp); the second array then keeps
// {the standard entry's z word, flags} for that code.
template <int V, bool BYPASS, bool LEAN = false>
__global__ void ragged_push_prep_kernel(const RaggedArgs R) {
  uint32_t err = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < R.total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = R.idx ? (int64_t)R.idx[i] : i;
    uint4 e = make_uint4(0, 0, 0, 0);
    int2 a = make_int2(0, (int)PREP_SKIP);
    if (k < 0 || k >= R.ntables) {
      err |= DEV_BAD_INDEX;
    } else {
      const int32_t size = R.sizes[k];
      const int32_t off = R.offsets ? R.offsets[k] : 0;
      int32_t v = (int32_t)((uint32_t)R.sym[i] - (uint32_t)off);
      const int32_t maxv = size - 2;
      uint32_t flags = 0;
      int32_t raw = 0;
      if constexpr (BYPASS) {
        if (v < 0) {
          raw = -2 * v - 1;
          v = maxv;
        } else if (v >= maxv) {
          raw = 2 * (v - maxv);
          v = maxv;
        }
        if (v == maxv) flags |= PREP_ESC;
      }
      if (v < 0 || v >= size - 1 || (int64_t)v + 1 >= R.cdf_width) {
        err |= DEV_BAD_VALUE;
      } else {
        const int32_t* row = R.cdfs + k * R.cdf_width;
        const int32_t start = row[v];
        const int32_t freq = (int32_t)((uint32_t)row[v + 1] - (uint32_t)start);
        e.w = (uint32_t)start;
        // same entry rule as the per-table builder: freq <= 0 (or too wide to pack at fp <= 23)
        // leaves z = 0, which the chain reports as a bad frequency
        if (freq > 0 && !(R.fp <= 23 && freq >= (1 << 24))) {
          const uint32_t d = (uint32_t)freq;
          e.z = R.fp <= 23 ? (d | (ceil_log2(d) << 24)) : d;
          if constexpr (V == 0) {
            const unsigned long long m = recip64(d);
            e.x = (uint32_t)m;
            e.y = (uint32_t)(m >> 32);
          } else {
            e.x = recip32(d);
          }
        }
        a = make_int2(raw, (int)flags);
      }
    }
    if constexpr (LEAN) {
      const uint32_t freq = e.z & 0xFFFFFFu, l = e.z >> 24;
      const bool fast = a.y == 0 && freq >= 2u && freq <= (1u << R.fp);
      uint4 le;
      le.x = e.x;
      le.y = fast ? (((1u << R.fp) - freq) | ((l - 1u) << 24)) : 0x80000000u;
      le.z = fast ? freq << (VT<V>::USED - R.fp) : 0u;
      le.w = e.w;
      R.ent[i] = le;
      R.aux[i] = make_int2((int)e.z, a.y);
    } else {
      R.ent[i] = e;
      R.aux[i] = a;
    }
  }
  report(R.status, err);
}

constexpr int RG_RS = 32;  // push chain: entry ring slots per thread
constexpr int RG_D = 24;   // push chain: steps between an entry copy and its use

template <int V, bool BYPASS>
__global__ void __launch_bounds__(256) ragged_push_chain_kernel(const RaggedArgs R, const PushParams P) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  uint4* ering = reinterpret_cast<uint4*>(smem_raw);
  int2* aring = reinterpret_cast<int2*>(ering + RG_RS * T);
  const int64_t b = (int64_t)blockIdx.x * T + tid;
  if (b >= R.batch) return;
  int64_t lo, hi;
  if (!ragged_row(R, b, lo, hi)) {
    report(R.status, DEV_BAD_VALUE);
    return;
  }
  int32_t* row = R.stream + b * R.width;
  PushCursor<V> cur;
  cur.payload = reinterpret_cast<uint8_t*>(row + 1);
  cur.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
  cur.cap = (R.width - 1) * 4 / VT<V>::WBYTES;
  cur.err = 0;
  using S = typename VT<V>::State;
  using W = typename VT<V>::Word;
  constexpr int MR = VT<V>::MAX_RENORM;
  S x = load_state<V>(row, 0);
  const int64_t n = hi - lo;
  const bool packed = P.fp <= 23;
  const int shift = VT<V>::USED - P.fp;
  W* words = reinterpret_cast<W*>(cur.payload);
  for (int64_t t = 0; t < n + RG_D; ++t) {
    if (t < n) {  // step t codes symbol hi - 1 - t
      const int64_t i = hi - 1 - t;
      const int sl = (int)(t & (RG_RS - 1)) * T + tid;
      cp_async16(ering + sl, R.ent + i, 16);
      cp_async8(aring + sl, R.aux + i);
    }
    cp_async_commit();
    cp_async_wait<RG_D - 1>();
    const int64_t tc = t - RG_D;
    if (tc < 0) continue;
    const int sl = (int)(tc & (RG_RS - 1)) * T + tid;
    PushPrep r;
    r.e = ering[sl];
    const int2 a = aring[sl];
    r.raw = a.x;
    r.flags = (uint32_t)a.y;
    r.rbase = 0;
    r.rcap = 0;
    const uint32_t freq = packed ? entry_freq(r.e, true) : 0u;
    if (r.flags == 0u && freq - 1u < (1u << P.fp) && cur.p >= -1 && cur.p + MR < cur.cap) {
      // every word this step can emit lands inside the row: the store is predicated on the word
      // being kept, so the renormalisation has no branch and slots past the row's final length
      // keep what they held
      const S bound = (S)((S)freq << shift);
#pragma unroll
      for (int u = 0; u < MR; ++u) {
        const bool rn = x >= bound;
        st_global_if<W>(words + (cur.p + 1), (uint32_t)x, rn);
        cur.p += rn ? 1 : 0;
        x = rn ? (S)(x >> VT<V>::WB) : x;
      }
      const S q = quotient<V>(x, r.e, true);
      x = (S)(x + to_state<S>((int32_t)r.e.w) + q * (S)((S)((S)1 << P.fp) - (S)freq));
    } else {
      push_chain<V, false, BYPASS>(P, x, cur, r);  // flagged steps, rows near their end, wide precision
    }
  }
  cp_async_wait<0>();
  store_state<V>(row, 0, x);
  row[0] = (int32_t)((cur.p + 1) * VT<V>::WBYTES);
  report(R.status, cur.err);
}

// Lean chain for 32-bit states without bypass coding (entries from the LEAN prep).  Each
// thread's entries arrive in a ring of four 16-entry quarters, each filled by one 1D bulk copy
// (copy engine, completing on the quarter's mbarrier) three quarters ahead of its use; the next
// step's entry is read from the ring during the current step.  A step whose entry is usable
// (2 <= freq <= 2^fp) and whose words fit the row takes the fast form: the renormalisation count
// from MR comparisons made at once ((x >> WB*t) >= bound for t < MR: the reference's loop of
// rans_utils.hpp:45-49 runs exactly that many times, the conditions being nested), the words
// stored by predicated stores (the kept ones only, no branch), the reciprocal quotient
// mulhi(x, m) >> (l - 1) = floor(x * m / 2^(31+l)) (exact there: the renormalised state is below
// bound <= 2^31) and C(s, x) of rans_utils.hpp:292.  Any other step runs push_chain, the
// reference-exact step code, on the standard entry rebuilt from the second array.
constexpr int RQ_ENT = 16;                             // entries per quarter (one bulk copy)
constexpr int RQ_Q = 4;                                // quarters per thread
constexpr int RQ_STRIDE = RQ_Q * RQ_ENT * 16 + 16;     // ring bytes per thread (+16: threads on distinct banks)
constexpr int RQ_SMEM = RQ_STRIDE + RQ_Q * 8;          // + one mbarrier per quarter
constexpr unsigned RQ_WAIT_LIMIT = 1u << 20;           // tries of a copy-completion wait

template <int V>
__global__ void __launch_bounds__(256) ragged_push_lean_kernel(const RaggedArgs R, const PushParams P) {
  static_assert(V == 1 || V == 2, "32-bit states only");
  using W = typename VT<V>::Word;
  constexpr int MR = VT<V>::MAX_RENORM;
  constexpr int WB = VT<V>::WB;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  uint4* ring = reinterpret_cast<uint4*>(smem_raw + (size_t)tid * RQ_STRIDE);
  unsigned long long* bar = reinterpret_cast<unsigned long long*>(smem_raw + (size_t)T * RQ_STRIDE) + tid * RQ_Q;
  const int64_t b = (int64_t)blockIdx.x * T + tid;
  if (b >= R.batch) return;
  int64_t lo, hi;
  if (!ragged_row(R, b, lo, hi)) {
    report(R.status, DEV_BAD_VALUE);
    return;
  }
  int32_t* row = R.stream + b * R.width;
  uint8_t* payload = reinterpret_cast<uint8_t*>(row + 1);
  W* words = reinterpret_cast<W*>(payload);
  int64_t p = (int64_t)row[0] / VT<V>::WBYTES - 1;  // last written word
  const int64_t cap = (R.width - 1) * 4 / VT<V>::WBYTES;
  // fast steps need p >= -1 (a length outside the row sends every step the exact way) and room for
  // MR words after p
  const int64_t pfast = p >= -1 ? cap - MR : INT64_MIN;
  uint32_t x = (uint32_t)load_state<V>(row, 0);
  uint32_t err = 0;
  const int64_t n = hi - lo;
  const int64_t nch = (n + RQ_ENT - 1) / RQ_ENT;
  // quarter c & 3 <- the entries of steps [16c, 16c + 16), last step first in memory order, so
  // step 16c + j reads slot 15 - j
  auto issue = [&](int64_t c) {
    const int cnt = (int)min((int64_t)RQ_ENT, n - c * RQ_ENT);
    const int q = (int)(c & (RQ_Q - 1));
    mbar_arrive_expect_tx(bar + q, (unsigned)cnt * 16u);
    bulk_copy_g2s(ring + q * RQ_ENT + (RQ_ENT - cnt), R.ent + (hi - c * RQ_ENT - cnt), (unsigned)cnt * 16u, bar + q);
  };
  auto wait = [&](int64_t c) -> bool {
    const int q = (int)(c & (RQ_Q - 1));
    const unsigned par = (unsigned)((c >> 2) & 1);
    for (unsigned it = 0; it < RQ_WAIT_LIMIT; ++it)
      if (mbar_try_wait(bar + q, par)) return true;
    return false;
  };
  if (nch > 0) {
    for (int q = 0; q < RQ_Q; ++q) mbar_init(bar + q, 1u);
    mbar_init_fence();
    for (int64_t c = 0; c < min(nch, (int64_t)RQ_Q); ++c) issue(c);
  }
  int64_t c = 0;
  for (; c < nch; ++c) {
    if (!wait(c)) {
      err |= DEV_STALLED;
      break;
    }
    const int cnt = (int)min((int64_t)RQ_ENT, n - c * RQ_ENT);
    const uint4* ch = ring + (c & (RQ_Q - 1)) * RQ_ENT + (RQ_ENT - 1);
    uint4 e = ch[0];
#pragma unroll 1
    for (int j = 0; j < cnt; ++j) {
      const uint4 en = j + 1 < cnt ? ch[-(j + 1)] : e;
      if ((int32_t)e.y >= 0 && p < pfast) {
        const uint32_t bound = e.z;
        W* wp = words + (p + 1);
        int k;
        if constexpr (V == 1) {
          const uint32_t x8 = x >> 8, x16 = x >> 16;
          const bool e0 = x >= bound, e1 = x8 >= bound, e2 = x16 >= bound;
          k = (e0 ? 1 : 0) + (e1 ? 1 : 0) + (e2 ? 1 : 0);
          st_global_if<W>(wp, x, e0);
          st_global_if<W>(wp + 1, x8, e1);
          st_global_if<W>(wp + 2, x16, e2);
        } else {
          k = x >= bound ? 1 : 0;
          st_global_if<W>(wp, x, k != 0);
        }
        x >>= WB * k;
        p += k;
        const uint32_t qt = __umulhi(x, e.x) >> (e.y >> 24);
        x = x + e.w + qt * (e.y & 0xFFFFFFu);
      } else {
        const int2 a = R.aux[hi - 1 - (c * RQ_ENT + j)];
        PushCursor<V> cur;
        cur.payload = payload;
        cur.p = p;
        cur.cap = cap;
        cur.err = err;
        PushPrep r;
        r.e = make_uint4(e.x, 0u, (uint32_t)a.x, e.w);
        r.flags = (uint32_t)a.y;
        r.raw = 0;
        r.rbase = 0;
        r.rcap = 0;
        typename VT<V>::State xs = x;
        push_chain<V, false, false>(P, xs, cur, r);
        x = (uint32_t)xs;
        p = cur.p;
        err = cur.err;
      }
      e = en;
    }
    if (c + RQ_Q < nch) {
      fence_proxy_async_shared();  // this thread's reads of the quarter come before the copy's writes
      issue(c + RQ_Q);
    }
  }
  // a wait that gave up leaves copies in flight: wait (bounded) for them before leaving
  for (int64_t d = c; d < min(nch, c + RQ_Q); ++d) wait(d);
  store_state<V>(row, 0, (typename VT<V>::State)x);
  row[0] = (int32_t)((p + 1) * VT<V>::WBYTES);
  report(R.status, err);
}

// ---------------------------------------------------------------- pop
// cp.async groups complete in order, so one wait depth serves both copies: a row is copied RP_DR
// steps before its use and an index RP_DI = 2 RP_DR steps before, so the index a row copy needs
// has landed by the same wait that lands the rows (a short index lead would force young row
// copies to land early too and cut the row prefetch short)
constexpr int RP_DR = 12;             // steps between a row copy and its use
constexpr int RP_DI = 2 * RP_DR;      // steps between an index copy and its use
constexpr int RP_WAIT = RP_DR - 1;    // groups allowed in flight after each iteration's commit
constexpr int RP_RI = 32;             // index ring slots (> RP_DI)
constexpr int RP_RR = 16;             // row ring slots (> RP_DR)

// 16-byte units of shared memory one staged row occupies (the row rounded out to 16-byte bounds)
inline int64_t ragged_row_units(int64_t cdf_width) { return (cdf_width + 3) / 4 + 1; }

template <int V, bool BYPASS, bool STAGE>
__global__ void __launch_bounds__(256) ragged_pop_kernel(const RaggedArgs R, const PopParams P, int units) {
  using S = typename VT<V>::State;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  int4* rring = reinterpret_cast<int4*>(smem_raw);                                       // [RR][T][units]
  int32_t* kring = reinterpret_cast<int32_t*>(rring + (STAGE ? (size_t)RP_RR * T * units : 0));  // [RI][T]
  int2* tring = reinterpret_cast<int2*>(kring + RP_RI * T);                               // [RR][T]
  const int64_t b = (int64_t)blockIdx.x * T + tid;
  if (b >= R.batch) return;
  int64_t lo, hi;
  if (!ragged_row(R, b, lo, hi)) {
    report(R.status, DEV_BAD_VALUE);
    return;
  }
  int32_t* row = R.stream + b * R.width;
  PopCursor<V> cur;
  cur.payload = reinterpret_cast<const uint8_t*>(row + 1);
  cur.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
  cur.first = VT<V>::SBYTES / VT<V>::WBYTES;
  cur.cap = (R.width - 1) * 4 / VT<V>::WBYTES;
  cur.err = 0;
  S x = load_state<V>(row, 0);
  const int64_t n = hi - lo;
  const int64_t total_words = R.ntables * R.cdf_width;
  // table index of step t (staged in the index ring when the caller gave indexes)
  auto table_of = [&](int64_t t) -> int64_t {
    return R.idx ? (int64_t)kring[(int)(t & (RP_RI - 1)) * T + tid] : lo + t;
  };
  // iteration j: copy the index of step j, copy the row (and size, offset) of step j - (DI - DR),
  // commit, wait, decode step j - DI
  for (int64_t j = 0; j < n + RP_DI; ++j) {
    if (R.idx && j < n) cp_async4(kring + (int)(j & (RP_RI - 1)) * T + tid, R.idx + lo + j);
    const int64_t tr = j - (RP_DI - RP_DR);
    if (tr >= 0 && tr < n) {
      const int64_t k = table_of(tr);
      const int sl = (int)(tr & (RP_RR - 1));
      int2* td = tring + sl * T + tid;
      if (k >= 0 && k < R.ntables) {
        if constexpr (STAGE) {
          // the row rounded out to 16-byte bounds; the tail past the table array reads nothing
          const int64_t e0 = k * R.cdf_width, base = e0 & ~(int64_t)3;
          const int64_t nu = (e0 + R.cdf_width - base + 3) / 4;
          int4* dst = rring + ((size_t)sl * T + tid) * units;
          for (int64_t u = 0; u < nu; ++u) {
            const int64_t w0 = base + 4 * u;
            const int64_t avail = total_words - w0;
            cp_async16(dst + u, R.cdfs + w0, avail >= 4 ? 16 : (int)(avail > 0 ? avail * 4 : 0));
          }
        }
        cp_async4(&td->x, R.sizes + k);
        if (R.offsets) cp_async4(&td->y, R.offsets + k);
        else td->y = 0;
      }
    }
    cp_async_commit();
    cp_async_wait<RP_WAIT>();
    const int64_t tc = j - RP_DI;
    if (tc < 0) continue;
    const int64_t k = table_of(tc);
    const int64_t i = lo + tc;
    if (k < 0 || k >= R.ntables) {
      cur.err |= DEV_BAD_INDEX;
      R.out[i] = 0;
      continue;
    }
    const int sl = (int)(tc & (RP_RR - 1));
    const int2 so = tring[sl * T + tid];
    TableInfo tinf;
    tinf.size = so.x;
    tinf.offset = so.y;
    tinf.cut = 0;
    tinf.cut_log2 = -1;
    const int32_t cum = (int32_t)(uint32_t)(x & (S)((1ull << R.fp) - 1ull));
    int64_t s;
    int32_t cum_off, freq;
    bool found;
    if constexpr (STAGE) {
      const int64_t e0 = k * R.cdf_width;
      const int32_t* srow =
          reinterpret_cast<const int32_t*>(rring + ((size_t)sl * T + tid) * units) + (e0 - (e0 & ~(int64_t)3));
      found = lookup_symbol<V, LK_SEARCH, false>(srow, tinf, cum, R.cdf_width, R.fp, s, cum_off, freq);
    } else {
      found = lookup_symbol<V, LK_SEARCH, true>(R.cdfs + k * R.cdf_width, tinf, cum, R.cdf_width, R.fp, s, cum_off,
                                                freq);
    }
    if (!found) {
      cur.err |= DEV_BAD_VALUE;
      R.out[i] = 0;
      continue;
    }
    const int32_t v = pop_finish<V, BYPASS>(P, x, cur, (int32_t)s, cum_off, freq, tinf.size - 2);
    R.out[i] = (int32_t)((uint32_t)v + (uint32_t)tinf.offset);
  }
  cp_async_wait<0>();
  store_state<V>(row, 0, x);
  row[0] = (int32_t)((cur.p + 1) * VT<V>::WBYTES);
  report(R.status, cur.err);
}

// One warp per stream, for rows of at most 64 entries (the per-element tables: 33 entries).  Lane
// l stages entries l and l + 32 of each step's row with 4-byte cp.async RW_D steps ahead (lane 0
// also the row's size and offset); after its own copies land each lane meets the others at a
// __syncwarp, so entries staged by another lane are visible.  The search is one ballot of
// P(j) = row[j] <= cum over the row's entries j < size: the reference's bisection
// (rans_utils.hpp:424-450) keeps low <= c <= high for every probe whenever P is true exactly on
// the first c entries and false on entry size - 1, so it ends at s = c - 1 whatever the row's
// values are; the ballot mask shows that case directly (bit 0 set, bit size - 1 clear, set bits a
// prefix: m & (m + 1) == 0), s = popc(m) - 1 and (start, freq) come from two shuffles.  Any other
// mask takes the reference bisection itself (on the staged row).  Every lane carries the same
// state; the decoded symbols of 32 steps leave as one coalesced store.
constexpr int RW_D = 12;   // steps between a row copy and its use
constexpr int RW_R = 16;   // row ring slots per warp (> RW_D)
constexpr int RW_E = 66;   // staged words per slot: 64 entries + size + offset

// shared-memory words per warp: a ring of RW_R row slots, or (consecutive rows) two buffers of
// 32 rows with their sizes and offsets
__host__ __device__ inline size_t ragged_warp_words(bool contig, int64_t cdf_width) {
  return contig ? 2 * (32 * (size_t)cdf_width + 64) : (size_t)RW_R * RW_E;
}

template <int V, bool BYPASS, bool WIDE, bool CONTIG>
__global__ void __launch_bounds__(256) ragged_pop_warp_kernel(const RaggedArgs R, const PopParams P) {
  using S = typename VT<V>::State;
  using Wd = typename VT<V>::Word;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warps = blockDim.x >> 5, wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* ring = reinterpret_cast<int32_t*>(smem_raw) + (size_t)wib * ragged_warp_words(CONTIG, R.cdf_width);
  const int64_t b = (int64_t)blockIdx.x * warps + wib;
  if (b >= R.batch) return;
  int64_t lo, hi;
  if (!ragged_row(R, b, lo, hi) || hi - lo > 0x7fffff00) {
    if (lane == 0) report(R.status, DEV_BAD_VALUE);
    return;
  }
  int32_t* row = R.stream + b * R.width;
  // word cursor (every lane holds the same copy): next word index p, its word prefetched in nextw
  const Wd* pw = reinterpret_cast<const Wd*>(row + 1);
  const int64_t p64 = (int64_t)row[0] / VT<V>::WBYTES - 1;
  const int first = VT<V>::SBYTES / VT<V>::WBYTES;
  const int capw = (int)min((R.width - 1) * 4 / VT<V>::WBYTES, (int64_t)0x7fffffff);
  int p = (int)min(max(p64, (int64_t)-0x7fffffff), (int64_t)0x7fffffff);
  S nextw = (p >= first && p < capw) ? (S)__ldg(pw + p) : (S)0;
  uint32_t err = 0;
  S x = load_state<V>(row, 0);
  const int n = (int)(hi - lo);
  const int W = (int)R.cdf_width;
  const int32_t cmask = (int32_t)((1u << R.fp) - 1u);
  // one step decoded from a staged row (`slot`: the row's entries in shared memory)
  auto decode = [&](const int32_t* slot, int32_t size, int32_t offset) -> int32_t {
    int32_t v = 0;
    const int32_t cum = (int32_t)((uint32_t)x & (uint32_t)cmask);
    const int32_t c0 = lane < W ? slot[lane] : 0;
    int64_t s;
    int32_t cum_off = 0, freq = 0;
    bool found;
    bool fast;
    int32_t st = 0, en = 0;
    if constexpr (!WIDE) {
      // rows of at most 33 entries: lane l holds entry l, every lane reads entry 32
      const int32_t e32 = W > 32 ? slot[32] : 0;
      const unsigned m = __ballot_sync(0xffffffffu, lane < size && c0 <= cum);
      // P(size - 1) must be false: bit size - 1 of the mask, or entry 32 for 33-entry rows
      const bool last_false = size <= 32 ? ((m >> ((size - 1) & 31)) & 1u) == 0u : cum < e32;
      fast = size >= 2 && size <= W && (m & 1u) != 0u && (m & (m + 1u)) == 0u && last_false;
      if (fast) {
        s = __popc(m) - 1;
        st = __shfl_sync(0xffffffffu, c0, (int)s);
        const int32_t en0 = __shfl_sync(0xffffffffu, c0, (int)(s + 1) & 31);
        en = s + 1 == 32 ? e32 : en0;
      }
    } else {
      const int32_t c1 = lane + 32 < W ? slot[32 + lane] : 0;
      const unsigned m0 = __ballot_sync(0xffffffffu, lane < size && c0 <= cum);
      const unsigned m1 = __ballot_sync(0xffffffffu, lane + 32 < size && c1 <= cum);
      const unsigned long long mm = (unsigned long long)m0 | ((unsigned long long)m1 << 32);
      fast = size >= 2 && size <= W && (mm & 1ull) != 0ull && (mm & (mm + 1ull)) == 0ull &&
             ((mm >> ((size - 1) & 63)) & 1ull) == 0ull;
      if (fast) {
        s = __popcll(mm) - 1;
        st = __shfl_sync(0xffffffffu, s < 32 ? c0 : c1, (int)(s & 31));
        en = __shfl_sync(0xffffffffu, s + 1 < 32 ? c0 : c1, (int)((s + 1) & 31));
      }
    }
    if (fast) {
      cum_off = cum - st;
      freq = (int32_t)((uint32_t)en - (uint32_t)st);
      found = true;
    } else {
      TableInfo tinf;
      tinf.size = size;
      tinf.offset = offset;
      tinf.cut = 0;
      tinf.cut_log2 = -1;
      found = lookup_symbol<V, LK_SEARCH, false>(slot, tinf, cum, R.cdf_width, R.fp, s, cum_off, freq);
    }
    if (!found) {
      err |= DEV_BAD_VALUE;
    } else {
      // x = D(x) and the refill (rans_utils.hpp:473-475), the first word from the prefetch
      x = (S)((x >> R.fp) * to_state<S>(freq) + to_state<S>(cum_off));
#pragma unroll
      for (int t = 0; t < VT<V>::MAX_RENORM; ++t) {
        if ((unsigned long long)x < VT<V>::LB) {
          if (p < first || p >= capw) err |= DEV_UNDERFLOW;
          x = (S)((x << VT<V>::WB) | nextw);
          --p;
          nextw = (p >= first && p < capw) ? (S)__ldg(pw + p) : (S)0;
        }
      }
      int32_t value = (int32_t)s;
      if constexpr (BYPASS) {
        if (value == size - 2) {  // escape (rare): the cursor-based reference code
          PopCursor<V> cur;
          cur.payload = reinterpret_cast<const uint8_t*>(row + 1);
          cur.p = p;
          cur.first = first;
          cur.cap = (R.width - 1) * 4 / VT<V>::WBYTES;
          cur.err = err;
          const int32_t raw = pop_escape<V>(x, cur, R.bp);
          value = raw >> 1;
          value = (raw & 1) ? (-value - 1) : (value + size - 2);
          p = (int)min(max(cur.p, (int64_t)-0x7fffffff), (int64_t)0x7fffffff);
          err = cur.err;
          nextw = (p >= first && p < capw) ? (S)__ldg(pw + p) : (S)0;
        }
      }
      v = (int32_t)((uint32_t)value + (uint32_t)offset);
    }
    return v;
  };
  int32_t kcur = 0;   // table index held by this lane for steps [32 m, 32 m + 32)
  int32_t outv = 0;   // decoded symbol of step 32 m + lane
  if constexpr (CONTIG) {
    // rows of consecutive symbols are consecutive: stage 32 steps' rows (with their sizes and
    // offsets) at once into one of two buffers, one block ahead of the decode
    int32_t* bufs[2] = {ring, ring + (32 * W + 64)};
    const int nblk = (n + 31) >> 5;
    auto stage = [&](int blk) {
      int32_t* buf = bufs[blk & 1];
      const int64_t t0 = lo + ((int64_t)blk << 5);
      const int nr = min(32, n - (blk << 5));
      const int vr = (int)max((int64_t)0, min((int64_t)nr, R.ntables - t0));  // rows inside the table list
      const int32_t* src = R.cdfs + t0 * R.cdf_width;
      for (int i = lane; i < vr * W; i += 32) cp_async4(buf + i, src + i);
      if (lane < vr) {
        cp_async4(buf + 32 * W + lane, R.sizes + t0 + lane);
        if (R.offsets) cp_async4(buf + 32 * W + 32 + lane, R.offsets + t0 + lane);
      }
    };
    if (nblk > 0) stage(0);
    cp_async_commit();
    for (int blk = 0; blk < nblk; ++blk) {
      if (blk + 1 < nblk) stage(blk + 1);
      cp_async_commit();
      cp_async_wait<1>();
      __syncwarp();  // every lane's staged words are visible to the whole warp
      const int32_t* buf = bufs[blk & 1];
      const int t0 = blk << 5;
      const int nr = min(32, n - t0);
#pragma unroll 1
      for (int r = 0; r < nr; ++r) {
        int32_t v = 0;
        if (lo + t0 + r >= R.ntables) {
          err |= DEV_BAD_INDEX;
        } else {
          const int32_t size = buf[32 * W + r];
          const int32_t offset = R.offsets ? buf[32 * W + 32 + r] : 0;
          v = decode(buf + r * W, size, offset);
        }
        if (r == lane) outv = v;
      }
      if (lane < nr) R.out[lo + t0 + lane] = outv;  // one coalesced store per block
      __syncwarp();  // the buffer is restaged only after every lane has read it
    }
  } else {
    auto table_at = [&](int t, int32_t kreg) -> int64_t {
      return R.idx ? (int64_t)__shfl_sync(0xffffffffu, kreg, t & 31) : lo + t;
    };
    int32_t kahead = (R.idx && lane < n) ? R.idx[lo + lane] : 0;           // indexes of steps [0, 32)
    int32_t kahead2 = (R.idx && 32 + lane < n) ? R.idx[lo + 32 + lane] : 0;  // steps [32, 64)
    // iteration j: stage the row of step j, decode step j - RW_D
    for (int j = 0; j < n + RW_D; ++j) {
      if ((j & 31) == 0 && j > 0) {  // rotate the index registers every 32 steps
        kahead = kahead2;
        kahead2 = (R.idx && j + 32 + lane < n) ? R.idx[lo + j + 32 + lane] : 0;
      }
      if (j < n) {
        const int64_t k = table_at(j, kahead);
        int32_t* slot = ring + (j & (RW_R - 1)) * RW_E;
        if (k >= 0 && k < R.ntables) {
          const int32_t* src = R.cdfs + k * R.cdf_width;
          if (lane < W) cp_async4(slot + lane, src + lane);
          if (lane + 32 < W) cp_async4(slot + 32 + lane, src + 32 + lane);
          if (lane == 0) {
            cp_async4(slot + 64, R.sizes + k);
            if (R.offsets) cp_async4(slot + 65, R.offsets + k);
          }
        }
      }
      cp_async_commit();
      const int tc = j - RW_D;
      if (tc < 0) continue;
      if ((tc & 31) == 0) {
        if (tc > 0) R.out[lo + tc - 32 + lane] = outv;  // the previous 32 steps: one coalesced store
        // indexes of steps [tc, tc + 32): the staging side (RW_D < 32 steps ahead) holds them now
        kcur = kahead;
      }
      cp_async_wait<RW_D - 1>();
      __syncwarp();  // every lane's staged words are visible to the whole warp
      const int64_t k = table_at(tc, kcur);
      int32_t v = 0;
      if (k < 0 || k >= R.ntables) {
        err |= DEV_BAD_INDEX;
      } else {
        const int32_t* slot = ring + (tc & (RW_R - 1)) * RW_E;
        const int32_t size = __shfl_sync(0xffffffffu, lane == 0 ? slot[64] : 0, 0);
        const int32_t offset = R.offsets ? __shfl_sync(0xffffffffu, lane == 0 ? slot[65] : 0, 0) : 0;
        v = decode(slot, size, offset);
      }
      if ((tc & 31) == lane) outv = v;
    }
    // the last group of decoded symbols (full or partial)
    const int last = n > 0 ? ((n - 1) & ~31) : 0;
    if (n > 0 && last + lane < n) R.out[lo + last + lane] = outv;
  }
  cp_async_wait<0>();
  if (lane == 0) {
    store_state<V>(row, 0, x);
    row[0] = (int32_t)((int64_t)(p + 1) * VT<V>::WBYTES);
    report(R.status, err);
  }
}

// Lean warp pop for the common per-element case: consecutive rows (no table indexes) of at most 33
// entries, no bypass coding.  Same results as ragged_pop_warp_kernel; the step is rebuilt around a
// short dependent chain:
//   * lane l compares entry l + 1 (l + 1 < size) with cum, so s = popc(ballot) directly, and every
//     lane forms the candidate state (x >> fp) * (row[l+1] - row[l]) + cum - row[l] beside the
//     vote; one shuffle from lane s gives D(x) (rans_utils.hpp:466-471).
//   * the exactness test of ragged_pop_warp_kernel in three comparisons: the mask is a prefix
//     (m & (m + 1) == 0, so m = 2^s - 1), entry size - 1 is above cum (s <= size - 2, with a
//     usable size folded into the bound) and entry 0 is not.  Then the reference bisection
//     (rans_utils.hpp:424-450) ends at s; any other step runs that bisection on the staged row.
//   * the words ahead of the cursor sit in a 64-bit register window (two 32-bit halves moved by
//     funnel shifts, refilled one aligned 32-bit unit at a time, the next unit already loaded), so
//     the renormalisation of rans_utils.hpp:473-475 is a count of the words needed and a funnel
//     shift.
//   * the next step's row entries are read from shared memory during the current step (without a
//     branch: the last step of a block reads a row it does not use), and 16 rows are staged per
//     copy round so that every warp of a 4,096-stream call is resident at once.
constexpr int RL_ROWS = 16;  // rows per staging buffer

__host__ __device__ inline size_t ragged_lean_words(int64_t cdf_width) {
  return 2 * (RL_ROWS * (size_t)cdf_width + 2 * RL_ROWS);
}

template <int V>
__global__ void __launch_bounds__(256, 4) ragged_pop_lean_kernel(const RaggedArgs R, const PopParams P) {
  using S = typename VT<V>::State;
  constexpr int WB = VT<V>::WB;
  constexpr int WPU = 32 / WB;  // words per 32-bit unit
  constexpr int LWPU = WPU == 4 ? 2 : (WPU == 2 ? 1 : 0);
  constexpr int MR = VT<V>::MAX_RENORM;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warps = blockDim.x >> 5, wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = (int)R.cdf_width;
  int32_t* ring = reinterpret_cast<int32_t*>(smem_raw) + (size_t)wib * ragged_lean_words(W);
  const int64_t b = (int64_t)blockIdx.x * warps + wib;
  if (b >= R.batch) return;
  int64_t lo, hi;
  if (!ragged_row(R, b, lo, hi) || hi - lo > 0x7fffff00) {
    if (lane == 0) report(R.status, DEV_BAD_VALUE);
    return;
  }
  int32_t* row = R.stream + b * R.width;
  const uint32_t* pu = reinterpret_cast<const uint32_t*>(row + 1);
  const int first = VT<V>::SBYTES / VT<V>::WBYTES;  // words below hold the state
  const int ufirst = VT<V>::SBYTES / 4;
  const int capw = (int)min((R.width - 1) * 4 / VT<V>::WBYTES, (int64_t)0x7fffffff);
  const int capu = (int)min(R.width - 1, (int64_t)0x7fffffff);
  // a word outside [first, capw) reads as 0, as the reference-order cursor of the other pops does
  auto unit = [&](int u) -> uint32_t { return (u >= ufirst && u < capu) ? __ldg(pu + u) : 0u; };
  const int64_t p64 = (int64_t)row[0] / VT<V>::WBYTES - 1;
  int p = (int)min(max(p64, (int64_t)-0x7fffffff), (int64_t)0x7fffffff);  // next word to read
  // window wh:wl: the next words to read, the first in the top bits of wh, nbits of them (> 32
  // before every step); nu = unit q, merged when nbits drops to 32 or below
  int q = p >> LWPU;
  uint32_t wh = unit(q) << (WB * (WPU - 1 - (p & (WPU - 1))));
  int nbits = WB * ((p & (WPU - 1)) + 1);
  const uint32_t u1 = unit(q - 1);
  wh |= __funnelshift_rc(u1, 0u, nbits);  // u1 >> nbits (nothing for nbits = 32)
  uint32_t wl = u1 << (32 - nbits);
  nbits += 32;
  q -= 2;
  uint32_t nu = unit(q);
  uint32_t err = 0;
  S x = load_state<V>(row, 0);
  const int n = (int)(hi - lo);
  const uint32_t cmask = (1u << R.fp) - 1u;
  const int fp = R.fp;
  const int bstride = RL_ROWS * W + 2 * RL_ROWS;
  const int nblk = (n + RL_ROWS - 1) / RL_ROWS;
  // rows [t0, t0 + 16) of the stream with their sizes and offsets into one buffer
  auto stage = [&](int blk) {
    int32_t* buf = ring + (blk & 1) * bstride;
    const int64_t t0 = lo + (int64_t)blk * RL_ROWS;
    const int nr = min(RL_ROWS, n - blk * RL_ROWS);
    const int vr = (int)max((int64_t)0, min((int64_t)nr, R.ntables - t0));
    const int32_t* src = R.cdfs + t0 * R.cdf_width;
    for (int i = lane; i < vr * W; i += 32) cp_async4(buf + i, src + i);
    if (lane < vr) {
      cp_async4(buf + RL_ROWS * W + lane, R.sizes + t0 + lane);
      if (R.offsets) cp_async4(buf + RL_ROWS * W + RL_ROWS + lane, R.offsets + t0 + lane);
    }
  };
  if (nblk > 0) stage(0);
  cp_async_commit();
  for (int blk = 0; blk < nblk; ++blk) {
    if (blk + 1 < nblk) stage(blk + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();  // every lane's staged words are visible to the whole warp
    const int32_t* buf = ring + (blk & 1) * bstride;
    const int t0 = blk * RL_ROWS;
    const int nr = min(RL_ROWS, n - t0);
    const int vr = (int)max((int64_t)0, min((int64_t)nr, R.ntables - (lo + t0)));
    // lane l < vr: the offset of this block's row l (its decoded symbol leaves from lane l)
    const int32_t myoff = (R.offsets && lane < vr) ? buf[RL_ROWS * W + RL_ROWS + lane] : 0;
    int32_t outv = 0;
    // the step's row: entries l and l + 1 of this lane, entry 0, size
    int32_t c0 = buf[lane], c1 = buf[lane + 1], r0 = buf[0];
    int32_t size = buf[RL_ROWS * W];
#pragma unroll 1
    for (int r = 0; r < vr; ++r) {
      const int rn = min(r + 1, RL_ROWS - 1);  // the next step's row, read off the chain
      const int32_t* sn = buf + rn * W;
      const int32_t c0n = sn[lane], c1n = sn[lane + 1], r0n = sn[0];
      const int32_t sizen = buf[RL_ROWS * W + rn];
      const int32_t lim = (size >= 2 && size <= W) ? size - 2 : -1;
      const int32_t c1m = lane + 1 < size ? c1 : 0x7fffffff;
      const int32_t cum = (int32_t)((uint32_t)x & cmask);
      const unsigned m = __ballot_sync(0xffffffffu, c1m <= cum);
      const int s = __popc(m);
      const S cand = (S)((x >> fp) * to_state<S>((int32_t)((uint32_t)c1 - (uint32_t)c0)) +
                         to_state<S>((int32_t)((uint32_t)cum - (uint32_t)c0)));
      S xn = __shfl_sync(0xffffffffu, cand, s & 31);
      int32_t sym = s;
      bool ok = true;
      if (!((m & (m + 1u)) == 0u && s <= lim && cum >= r0)) {
        TableInfo tinf;
        tinf.size = size;
        tinf.offset = 0;
        tinf.cut = 0;
        tinf.cut_log2 = -1;
        int64_t s64;
        int32_t cum_off, freq;
        ok = lookup_symbol<V, LK_SEARCH, false>(buf + r * W, tinf, cum, R.cdf_width, fp, s64, cum_off, freq);
        if (ok) {
          xn = (S)((x >> fp) * to_state<S>(freq) + to_state<S>(cum_off));
          sym = (int32_t)s64;
        } else {
          err |= DEV_BAD_VALUE;  // the state stays, the step decodes 0
        }
      }
      if (ok) {
        // words needed: the reference's renormalisation loop count (at most MR)
        int k = 0;
#pragma unroll
        for (int t = 0; t < MR; ++t) k += (xn < (S)(VT<V>::LB >> (WB * t))) ? 1 : 0;
        const int bits = WB * k;
        if constexpr (V == 0) {
          x = bits ? (S)((xn << 32) | wh) : xn;
          wh = bits ? wl : wh;
          wl = bits ? 0u : wl;
        } else {
          x = __funnelshift_lc(wh, xn, bits);
          wh = __funnelshift_l(wl, wh, bits);
          wl <<= bits;
        }
        if (k > 0 && (p >= capw || p < first + k - 1)) err |= DEV_UNDERFLOW;
        p = (int)((unsigned)p - (unsigned)k);
        nbits -= bits;
        if (nbits <= 32) {
          wh |= __funnelshift_rc(nu, 0u, nbits);
          wl = nu << ((32 - nbits) & 31);
          nbits += 32;
          nu = unit(--q);
        }
      }
      outv = lane == r ? (ok ? (int32_t)((uint32_t)sym + (uint32_t)myoff) : 0) : outv;
      c0 = c0n;
      c1 = c1n;
      r0 = r0n;
      size = sizen;
    }
    if (vr < nr) err |= DEV_BAD_INDEX;  // rows past the table list decode as 0
    if (lane < nr) R.out[lo + t0 + lane] = outv;
    __syncwarp();  // the buffer is restaged only after every lane has read it
  }
  cp_async_wait<0>();
  if (lane == 0) {
    store_state<V>(row, 0, x);
    row[0] = (int32_t)((int64_t)(p + 1) * VT<V>::WBYTES);
    report(R.status, err);
  }
}

// ---------------------------------------------------------------- host side
static int ragged_threads(int64_t batch, int sms, int64_t smem_per_thread, int max_threads) {
  int64_t t = (batch + sms - 1) / sms;
  t = ((t + 31) / 32) * 32;
  t = std::max<int64_t>(32, std::min<int64_t>(t, max_threads));
  while (t > 32 && t * smem_per_thread > 200 * 1024) t -= 32;
  return (int)t;
}

template <int V, bool BY>
static void ragged_push_launch(const RaggedArgs& R, const PushParams& P, int sms, cudaStream_t s) {
  const int pb = (int)std::max<int64_t>(1, std::min<int64_t>((R.total + 255) / 256, 16 * (int64_t)sms));
  if constexpr (V != 0 && !BY) {
    // the entry array must be 16-byte aligned for the bulk copies (the library's own workspace
    // and any aligned caller buffer are)
    if (R.fp <= 23 && (reinterpret_cast<uintptr_t>(R.ent) & 15u) == 0 &&
        env_int("TORCH_ANS_B200_RAGGED_PUSH_LEAN", 1) != 0) {
      if (R.total > 0) {
        ragged_push_prep_kernel<V, false, true><<<pb, 256, 0, s>>>(R);
        note_launch();
      }
      const int T = ragged_threads(R.batch, sms, RQ_SMEM, 256);
      const size_t smem = (size_t)T * RQ_SMEM;
      if (smem > 48 * 1024)
        cudaFuncSetAttribute(ragged_push_lean_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      ragged_push_lean_kernel<V><<<(int)((R.batch + T - 1) / T), T, smem, s>>>(R, P);
      note_launch();
      return;
    }
  }
  if (R.total > 0) {
    ragged_push_prep_kernel<V, BY><<<pb, 256, 0, s>>>(R);
    note_launch();
  }
  const int T = ragged_threads(R.batch, sms, RG_RS * 24, 256);
  const size_t smem = (size_t)T * RG_RS * 24;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(ragged_push_chain_kernel<V, BY>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  ragged_push_chain_kernel<V, BY><<<(int)((R.batch + T - 1) / T), T, smem, s>>>(R, P);
  note_launch();
}

template <int V, bool BY, bool WIDE, bool CONTIG>
static void ragged_pop_warp_go(const RaggedArgs& R, const PopParams& P, int sms, cudaStream_t s) {
  int64_t warps = (R.batch + sms - 1) / sms;
  warps = std::max<int64_t>(1, std::min<int64_t>(warps, 8));
  const size_t smem = (size_t)warps * ragged_warp_words(CONTIG, R.cdf_width) * sizeof(int32_t);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(ragged_pop_warp_kernel<V, BY, WIDE, CONTIG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  ragged_pop_warp_kernel<V, BY, WIDE, CONTIG>
      <<<(int)((R.batch + warps - 1) / warps), (int)(warps * 32), smem, s>>>(R, P);
  note_launch();
}

template <int V>
static void ragged_pop_lean_go(const RaggedArgs& R, const PopParams& P, int sms, cudaStream_t s) {
  int64_t warps = (R.batch + sms - 1) / sms;
  warps = std::max<int64_t>(1, std::min<int64_t>(warps, 8));
  const size_t smem = (size_t)warps * ragged_lean_words(R.cdf_width) * sizeof(int32_t);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(ragged_pop_lean_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  ragged_pop_lean_kernel<V><<<(int)((R.batch + warps - 1) / warps), (int)(warps * 32), smem, s>>>(R, P);
  note_launch();
}

// without table indexes the rows of consecutive symbols are consecutive: block staging
template <int V, bool BY>
static void ragged_pop_warp_launch(const RaggedArgs& R, const PopParams& P, int sms, cudaStream_t s) {
  const bool contig = R.idx == nullptr;
  if constexpr (!BY) {
    if (contig && R.cdf_width <= 33 && env_int("TORCH_ANS_B200_RAGGED_POP_LEAN", 1) != 0) {
      ragged_pop_lean_go<V>(R, P, sms, s);
      return;
    }
  }
  if (R.cdf_width <= 33) {
    if (contig) ragged_pop_warp_go<V, BY, false, true>(R, P, sms, s);
    else ragged_pop_warp_go<V, BY, false, false>(R, P, sms, s);
  } else {
    if (contig) ragged_pop_warp_go<V, BY, true, true>(R, P, sms, s);
    else ragged_pop_warp_go<V, BY, true, false>(R, P, sms, s);
  }
}

template <int V, bool BY, bool STAGE>
static void ragged_pop_launch(const RaggedArgs& R, const PopParams& P, int units, int sms, cudaStream_t s) {
  const int64_t per = (STAGE ? (int64_t)RP_RR * units * 16 : 0) + RP_RI * 4 + RP_RR * 8;
  const int T = ragged_threads(R.batch, sms, per, 256);
  const size_t smem = (size_t)T * per;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(ragged_pop_kernel<V, BY, STAGE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  ragged_pop_kernel<V, BY, STAGE><<<(int)((R.batch + T - 1) / T), T, smem, s>>>(R, P, units);
  note_launch();
}

static int check_ragged(int variant, const int32_t* stream, int64_t batch, int64_t width, const int64_t* rows,
                        int64_t total, const int32_t* cdfs, int64_t ntables, int64_t cdf_width, const int32_t* sizes,
                        int fp, int bypass, int bp) {
  if (variant < 0 || variant > 2 || batch < 0 || total < 0 || ntables < 0 || cdf_width < 0)
    return TANS_E_INVALID_ARGUMENT;
  if (fp < 1 || fp > max_precision(variant)) return TANS_E_INVALID_ARGUMENT;
  if (bypass && (bp < 1 || bp > max_precision(variant))) return TANS_E_INVALID_ARGUMENT;
  if (batch == 0) return TANS_OK;
  if (!stream || !rows || width < 1 + (int64_t)state_bytes(variant) / 4) return TANS_E_INVALID_ARGUMENT;
  if (total > 0 && (!cdfs || !sizes || ntables < 1 || cdf_width < 2)) return TANS_E_INVALID_ARGUMENT;
  return TANS_OK;
}

}  // namespace tans

extern "C" size_t tans_push_ragged_workspace_size(int64_t total_symbols) {
  return total_symbols > 0 ? tans::align_up((size_t)total_symbols * 16) + tans::align_up((size_t)total_symbols * 8)
                           : 0;
}

extern "C" int tans_push_ragged(int variant, int32_t* stream, int64_t batch, int64_t stream_width,
                                const int32_t* symbols, const int32_t* indexes, const int64_t* row_starts,
                                int64_t total_symbols, const int32_t* cdfs, int64_t num_tables, int64_t cdf_width,
                                const int32_t* cdf_sizes, const int32_t* offsets, int freq_precision,
                                int bypass_coding, int bypass_precision, void* workspace, size_t workspace_bytes,
                                uint32_t* dev_status, void* cuda_stream) {
  using namespace tans;
  int rc = check_ragged(variant, stream, batch, stream_width, row_starts, total_symbols, cdfs, num_tables, cdf_width,
                        cdf_sizes, freq_precision, bypass_coding, bypass_precision);
  if (rc != TANS_OK) return rc;
  if (batch == 0) return TANS_OK;
  if (total_symbols > 0 && !symbols) return TANS_E_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(cuda_stream);
  const size_t need = tans_push_ragged_workspace_size(total_symbols);
  void* ws = workspace;
  bool owned = false;
  if (need > 0) {
    if (!ws) {
      if (cudaMallocAsync(&ws, need, s) != cudaSuccess) return TANS_E_CUDA;
      owned = true;
    } else if (workspace_bytes < need) {
      return TANS_E_WORKSPACE;
    }
  }
  RaggedArgs R{};
  R.stream = stream;
  R.batch = batch;
  R.width = stream_width;
  R.sym = symbols;
  R.idx = indexes;
  R.rows = row_starts;
  R.total = total_symbols;
  R.cdfs = cdfs;
  R.ntables = num_tables;
  R.cdf_width = cdf_width;
  R.sizes = cdf_sizes;
  R.offsets = offsets;
  R.fp = freq_precision;
  R.bp = bypass_precision;
  R.status = dev_status;
  R.ent = reinterpret_cast<uint4*>(ws);
  R.aux = reinterpret_cast<int2*>(reinterpret_cast<char*>(ws) + align_up((size_t)std::max<int64_t>(total_symbols, 0) * 16));
  PushParams P{};
  P.fp = freq_precision;
  P.bp = bypass_precision;
  P.status = dev_status;
  const int sms = sm_count();
  const bool by = bypass_coding != 0;
  if (variant == TANS_RANS64) {
    if (by) ragged_push_launch<0, true>(R, P, sms, s);
    else ragged_push_launch<0, false>(R, P, sms, s);
  } else if (variant == TANS_RANS32) {
    if (by) ragged_push_launch<1, true>(R, P, sms, s);
    else ragged_push_launch<1, false>(R, P, sms, s);
  } else {
    if (by) ragged_push_launch<2, true>(R, P, sms, s);
    else ragged_push_launch<2, false>(R, P, sms, s);
  }
  if (owned) cudaFreeAsync(ws, s);
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}

extern "C" int tans_pop_ragged(int variant, int32_t* stream, int64_t batch, int64_t stream_width,
                               int32_t* out_symbols, const int32_t* indexes, const int64_t* row_starts,
                               int64_t total_symbols, const int32_t* cdfs, int64_t num_tables, int64_t cdf_width,
                               const int32_t* cdf_sizes, const int32_t* offsets, int freq_precision,
                               int bypass_coding, int bypass_precision, uint32_t* dev_status, void* cuda_stream) {
  using namespace tans;
  int rc = check_ragged(variant, stream, batch, stream_width, row_starts, total_symbols, cdfs, num_tables, cdf_width,
                        cdf_sizes, freq_precision, bypass_coding, bypass_precision);
  if (rc != TANS_OK) return rc;
  if (batch == 0) return TANS_OK;
  if (total_symbols > 0 && !out_symbols) return TANS_E_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(cuda_stream);
  RaggedArgs R{};
  R.stream = stream;
  R.batch = batch;
  R.width = stream_width;
  R.out = out_symbols;
  R.idx = indexes;
  R.rows = row_starts;
  R.total = total_symbols;
  R.cdfs = cdfs;
  R.ntables = num_tables;
  R.cdf_width = cdf_width;
  R.sizes = cdf_sizes;
  R.offsets = offsets;
  R.fp = freq_precision;
  R.bp = bypass_precision;
  R.status = dev_status;
  PopParams P{};
  P.fp = freq_precision;
  P.bp = bypass_precision;
  P.status = dev_status;
  const int sms = sm_count();
  const int units = (int)ragged_row_units(cdf_width);
  const bool by = bypass_coding != 0;
  // rows of at most 64 entries: one warp per stream, ballot search
  if (cdf_width <= 64 && env_int("TORCH_ANS_B200_RAGGED_POP_WARP", 1) != 0) {
    if (variant == TANS_RANS64) {
      if (by) ragged_pop_warp_launch<0, true>(R, P, sms, s);
      else ragged_pop_warp_launch<0, false>(R, P, sms, s);
    } else if (variant == TANS_RANS32) {
      if (by) ragged_pop_warp_launch<1, true>(R, P, sms, s);
      else ragged_pop_warp_launch<1, false>(R, P, sms, s);
    } else {
      if (by) ragged_pop_warp_launch<2, true>(R, P, sms, s);
      else ragged_pop_warp_launch<2, false>(R, P, sms, s);
    }
    return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
  }
  // otherwise one thread per stream; rows are staged in shared memory when the table array is
  // 16-byte aligned and a row is small
  const bool stage = ((reinterpret_cast<uintptr_t>(cdfs) & 15u) == 0) && units <= 32;
#define TANS_RAGGED_POP(VV)                                                     \
  if (stage) {                                                                  \
    if (by) ragged_pop_launch<VV, true, true>(R, P, units, sms, s);             \
    else ragged_pop_launch<VV, false, true>(R, P, units, sms, s);               \
  } else {                                                                      \
    if (by) ragged_pop_launch<VV, true, false>(R, P, units, sms, s);            \
    else ragged_pop_launch<VV, false, false>(R, P, units, sms, s);              \
  }
  if (variant == TANS_RANS64) {
    TANS_RAGGED_POP(0)
  } else if (variant == TANS_RANS32) {
    TANS_RAGGED_POP(1)
  } else {
    TANS_RAGGED_POP(2)
  }
#undef TANS_RAGGED_POP
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}
