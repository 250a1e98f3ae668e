// rans_push_ws.cuh -- warp-specialised single-state push (rows 16-byte aligned, length % 4 == 0,
// at most 4096 tables, frequency precision <= 23).
//
// The encode of a stream is one serial chain (rans_utils.hpp:168-323 per symbol), so a block's
// throughput is set by how fast that chain turns over.  Here the chain warps run nothing but the
// chain, and separate prep warps of the same block feed them through a shared-memory ring:
//
//   prep warps   raw symbols/indexes: cp.async two groups ahead into a raw ring;
//                per (stream, chunk of 4 symbols): table info from shared memory, value =
//                symbol - offset, bounds checks, and a cp.async gather of the four 16-byte encode
//                entries {reciprocal, freq | shift << 24, start} into the entry ring slot; a chunk
//                the straight-line chain cannot code (bad index, symbol outside its table, escape,
//                zero frequency) is flagged;
//                arrive on full[slot] twice per thread: once with release semantics (flag bytes,
//                alias table indexes) and once when its cp.async gathers have landed.
//   chain warps  one lane per stream: wait full[slot], run the slot's chunks (last chunk of the
//                row first, last symbol of a chunk first): flagged chunks (or chunks whose words
//                might not fit the row) through the reference-exact step code, the rest as four
//                straight-line steps (compare, word store, multiply-high quotient, multiply-add);
//                then arrive on empty[slot] so the prep warps may refill it.
//
// A group is WS_G chunks of every stream of the block; slot = group % WS_R.  Every wait is a
// bounded try_wait loop: a wait that runs out sets TANS_DEV_STALLED, tells the other warps of
// the block through a shared flag, and every warp leaves (prep warps after their copies land).
#pragma once

#include "rans_push_common.cuh"

namespace tans {

constexpr int WS_G = 4;           // chunks per group (the flag bytes of a group are one word)
constexpr int WS_R = 4;           // entry ring slots
constexpr int WS_D = 2;           // groups of raw symbols/indexes in flight ahead of the prep
constexpr int WS_RR = WS_D + 2;   // raw ring slots
// tries before a wait gives up: at least ~25 ms even when every try returns at once, far beyond
// any real hand-over (a few microseconds).  The launch passes it as PushParams::wait_limit; the
// diagnostic variable TORCH_ANS_B200_WAIT_LIMIT sets another count (failure-detection tests use 0:
// the first wait of each warp gives up at once and the block leaves through the stall path).
constexpr unsigned WS_WAIT_LIMIT = 1u << 20;
constexpr int WS_HEADER = 128;    // barriers + abort flag

static_assert(WS_G == 4, "the flag bytes of one stream's group are read as one 32-bit word");

// shared-memory bytes per stream of a block
inline int64_t pushws_stream_bytes(bool alias) {
  return (int64_t)WS_R * 4 * WS_G * 16            // entry ring
         + (int64_t)WS_RR * WS_G * 32               // raw ring (symbols + indexes)
         + (int64_t)WS_R * 4                        // flag words
         + (alias ? (int64_t)WS_R * 4 * WS_G * 4 : 0);  // alias: table index per symbol
}
inline int64_t pushws_smem_bytes(int64_t sb, bool alias, int64_t ntables, int64_t remap_entries, int tcopies) {
  return WS_HEADER + sb * pushws_stream_bytes(alias) + ntables * (16 + 8 * (int64_t)tcopies) + remap_entries * 4;
}
// Copies of the per-table {size, offset} records the prep warps gather at random table indexes:
// with 16 interleaved copies, lane l reads copy l % 16, so the 16 lanes of a half warp always read
// 16 different 8-byte bank pairs (no bank conflicts); one copy when 16 would take over 32 KB.
inline int pushws_tcopies(int64_t ntables) { return ntables * 8 * 16 <= 32 * 1024 ? 16 : 1; }

// chain state the rare exact path reads and writes, passed by value both ways so that the kernel
// never takes the address of its state or of its parameters (both stay in registers)
template <int V> struct WsState {
  typename VT<V>::State x;
  int p;
  uint32_t err;
};

// A flagged chunk, or one whose words might not fit the row: the reference-exact steps, with the
// symbols and indexes read again from global memory (rare path, kept out of line).
template <int V, bool ALIAS, bool BYPASS>
__device__ __noinline__ WsState<V> pushws_exact_chunk(const PushParams P, WsState<V> st, int64_t b, int cr) {
  PushCursor<V> cur;
  int32_t* row = P.stream + b * P.width;
  cur.payload = reinterpret_cast<uint8_t*>(row + 1);
  cur.p = st.p;
  cur.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
  cur.err = 0;
  const int32_t* srow = P.sym + b * P.nsym;
  const int32_t* irow = P.idx + b * P.nsym;
  uint32_t perr = 0;
  typename VT<V>::State x = st.x;
  for (int q = 3; q >= 0; --q) {
    const int64_t i = 4 * (int64_t)cr + q;
    const PushPrep r = push_prepare<V, ALIAS, BYPASS>(P, __ldg(srow + i), __ldg(irow + i), true, perr);
    push_chain<V, ALIAS, BYPASS>(P, x, cur, r);
  }
  // past the row end the cursor only counts (the row's length then reports every word, as the
  // reference's does); later chunks see p + 4 * MAX_RENORM >= cap and stay on this path
  st.x = x;
  st.p = (int)(cur.p < 0x3FFFFFFF ? cur.p : 0x3FFFFFFF);
  st.err |= cur.err | perr;
  return st;
}

template <int V, bool ALIAS, bool BYPASS, bool RSMEM>
__global__ void __launch_bounds__(512) push_ws_kernel(const PushParams P, int sb, int chain_warps) {
  using S = typename VT<V>::State;
  using W = typename VT<V>::Word;
  constexpr int MR = VT<V>::MAX_RENORM;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned long long* full = reinterpret_cast<unsigned long long*>(smem_raw);
  unsigned long long* empty = full + WS_R;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + WS_R);
  uint4* ent = reinterpret_cast<uint4*>(smem_raw + WS_HEADER);                 // [R][4G][sb]
  int4* rsym = reinterpret_cast<int4*>(ent + (size_t)WS_R * 4 * WS_G * sb);    // [RR][G][sb]
  int4* ridx = rsym + (size_t)WS_RR * sb * WS_G;                               // [RR][G][sb]
  TableInfo* tsm = reinterpret_cast<TableInfo*>(ridx + (size_t)WS_RR * sb * WS_G);
  int2* tso = reinterpret_cast<int2*>(tsm + P.ntables);                          // [K][copies] {size, offset}
  const int tcl = P.ws_tcopies == 16 ? 4 : 0;                                    // log2 of the copies
  uint32_t* flg = reinterpret_cast<uint32_t*>(tso + (P.ntables << tcl));        // [R][sb]
  int32_t* kix = reinterpret_cast<int32_t*>(flg + (size_t)WS_R * sb);          // [R][4G][sb]
  int32_t* rsm = kix + (ALIAS ? (size_t)WS_R * 4 * WS_G * sb : 0);

  const int T = blockDim.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nprep = T - chain_warps * 32;
  const int64_t M = (int64_t)1 << P.fp;
  const int64_t b0 = (int64_t)blockIdx.x * sb;
  const int64_t N = P.nsym;
  const int nch = (int)(N >> 2);
  const int ngr = (nch + WS_G - 1) / WS_G;

  for (int64_t k = tid; k < P.ntables; k += T) tsm[k] = P.tinfo[k];
  for (int64_t i = tid; i < (P.ntables << tcl); i += T) {
    const TableInfo ti = P.tinfo[i >> tcl];
    tso[i] = make_int2(ti.size, ti.offset);
  }
  if constexpr (ALIAS && RSMEM) {
    for (int64_t i = tid; i < P.ntables * M; i += T) {
      const int64_t k = i >> P.fp, r = i & (M - 1);
      const int32_t sz = P.tinfo[k].size;
      const int64_t col = (int64_t)sz + r;
      rsm[i] = (sz >= 0 && col < P.cdf_width) ? P.cdfs[k * P.cdf_width + col] : 0;
    }
  }
  if (tid == 0) {
    for (int r = 0; r < WS_R; ++r) {
      mbar_init(full + r, 2u * (unsigned)nprep);
      mbar_init(empty + r, (unsigned)chain_warps);
    }
    *abort_flag = 0;
  }
  __syncthreads();

  if (warp < chain_warps) {
    // ------------------------------------------------------------------ chain warps
    const int lanes = (sb + chain_warps - 1) / chain_warps;
    const int s = warp * lanes + lane;
    const int64_t b = b0 + s;
    const bool active = lane < lanes && s < sb && b < P.batch;
    int32_t* row = P.stream + (active ? b : 0) * P.width;
    W* words = reinterpret_cast<W*>(row + 1);
    const int cap = (int)((P.width - 1) * 4 / VT<V>::WBYTES);
    int p = 0;
    S x = 0;
    bool row_ok = false;
    if (active) {
      const int64_t p64 = (int64_t)row[0] / VT<V>::WBYTES - 1;
      row_ok = p64 >= -1 && p64 < cap;  // a length outside the row sends every chunk the exact way
      p = (int)(p64 < -0x3FFFFFFF ? -0x3FFFFFFF : (p64 > 0x3FFFFFFF ? 0x3FFFFFFF : p64));
      x = load_state<V>(row, 0);
    }
    uint32_t err = 0;
    const int shift = VT<V>::USED - P.fp;
    const long long rstride = P.cdf_width;
    bool stalled = false;
    for (int g = 0; g < ngr; ++g) {
      const int slot = g % WS_R;
      if (!warp_wait(full + slot, (unsigned)(g / WS_R) & 1u, abort_flag, P.wait_limit)) {
        stalled = true;
        break;
      }
      if (active) {
        const uint32_t fw = flg[(size_t)slot * sb + s];
        const uint4* es = ent + (size_t)slot * 4 * WS_G * sb + s;
#pragma unroll 1
        for (int c = 0; c < WS_G; ++c) {
          const int gc = g * WS_G + c;
          if (gc >= nch) break;
          const int cr = nch - 1 - gc;
          uint4 e[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) e[q] = es[(size_t)(4 * c + q) * sb];
          bool exact = ((fw >> (8 * c)) & 0xFFu) != 0u || !row_ok || p + 4 * MR >= cap;
#pragma unroll
          for (int q = 0; q < 4; ++q) exact |= entry_freq(e[q], true) - 1u >= (1u << P.fp);  // 0 or above 2^fp
          if (exact) {
            const WsState<V> st = pushws_exact_chunk<V, ALIAS, BYPASS>(P, WsState<V>{x, p, err}, b, cr);
            x = st.x;
            p = st.p;
            err = st.err;
            continue;
          }
          int32_t kq[4] = {0, 0, 0, 0};
          if constexpr (ALIAS) {
#pragma unroll
            for (int q = 0; q < 4; ++q) kq[q] = kix[((size_t)slot * 4 * WS_G + 4 * c + q) * sb + s];
          }
#pragma unroll
          for (int q = 3; q >= 0; --q) {
            const uint32_t freq = e[q].z & 0xFFFFFFu;
            const unsigned long long bound = (unsigned long long)freq << shift;
            if constexpr (!ALIAS) {
              // the store is predicated on the word being kept (no branch; the chunk check above
              // keeps p + 1 inside the row): slots past the row's length keep what they held, as
              // the reference leaves them
#pragma unroll
              for (int u = 0; u < MR; ++u) {
                const bool r = (unsigned long long)x >= bound;
                st_global_if<W>(words + (p + 1), (uint32_t)x, r);
                p += r ? 1 : 0;
                x = r ? (S)(x >> VT<V>::WB) : x;
              }
            } else {
#pragma unroll
              for (int u = 0; u < MR; ++u) {
                if ((unsigned long long)x >= bound) {
                  ++p;
                  words[p] = (W)x;
                  x >>= VT<V>::WB;
                }
              }
            }
            const S qt = quotient<V>(x, e[q], true);
            const S start = to_state<S>((int32_t)e[q].w);
            if constexpr (ALIAS) {
              // same bounds rule as push_chain: a remap index outside the row skips the step
              const uint32_t kc = (uint32_t)kq[q];
              const S ri = (S)(x - qt * (S)freq + start);
              const int32_t sz = tsm[kc].size;
              const long long rcap = rstride - (long long)sz;
              int32_t rv = 0;
              const bool ok = (unsigned long long)ri < (unsigned long long)(rcap > 0 ? rcap : 0);
              if constexpr (RSMEM) {
                if ((unsigned long long)ri < (unsigned long long)M) rv = rsm[((int64_t)kc << P.fp) + (int64_t)ri];
                else if (ok) rv = __ldg(P.cdfs + (int64_t)kc * rstride + sz + (int64_t)ri);
              } else {
                if (ok) rv = __ldg(P.cdfs + (int64_t)kc * rstride + sz + (int64_t)ri);
              }
              if (ok) x = (S)((qt << P.fp) + to_state<S>(rv));
              else err |= DEV_BAD_VALUE;
            } else {
              const S cmpl = (S)((S)1 << P.fp) - (S)freq;
              x = (S)(x + start + qt * cmpl);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + slot);
    }
    if (stalled) {
      if (lane == 0) *abort_flag = 1;
      if (lane == 0) report(P.status, DEV_STALLED);
      return;
    }
    if (active) {
      store_state<V>(row, 0, x);
      row[0] = (int32_t)((int64_t)(p + 1) * VT<V>::WBYTES);
      report(P.status, err);
    }
    return;
  }

  // -------------------------------------------------------------------- prep warps
  const int ptid = tid - chain_warps * 32;
  const uint32_t kmax = (uint32_t)(P.ntables - 1);
  const int64_t emax = P.enc_stride - 1;
  // Tasks run stream-fastest across the lanes (task t: chunk t / sbp of stream t % sbp), in the
  // copies of the raw symbols and indexes and in the prep alike: every thread reads back only the
  // raw chunks its own cp.async copies brought in (its cp.async wait covers them), and a warp's
  // raw-ring reads, entry-ring copies and flag bytes fall on consecutive slots (no bank conflicts).
  // From 32 streams per block up, sbp = sb rounded up to whole warps, so that every warp works on
  // one chunk of consecutive streams; below that sbp = sb (padding would leave most lanes idle:
  // the prep warps' instructions, not bank conflicts, then set their pace).
  const int sbp = sb >= 32 ? (sb + 31) & ~31 : sb;
  const int ntaskp = WS_G * sbp;
  // t / sbp as a multiply-shift: exact for t * sbp < 2^20 (t < 4 sbp, sbp <= 128 streams)
  const uint32_t sbm = ((1u << 20) + (uint32_t)sbp - 1u) / (uint32_t)sbp;
  const int tcm = (1 << tcl) - 1;
  auto issue_raw = [&](int gr) {
    const int rs = gr % WS_RR;
    for (int t = ptid; t < ntaskp; t += nprep) {
      const int c = (int)(((uint32_t)t * sbm) >> 20), s = t - c * sbp;
      const int64_t b = b0 + s;
      const int gc = gr * WS_G + c;
      if (s < sb && b < P.batch && gc < nch) {
        const int64_t off = b * N + 4 * (int64_t)(nch - 1 - gc);
        cp_async16(rsym + ((size_t)rs * WS_G + c) * sb + s, P.sym + off, 16);
        cp_async16(ridx + ((size_t)rs * WS_G + c) * sb + s, P.idx + off, 16);
      }
    }
    cp_async_commit();  // one group per call, empty or not, so the wait depths below hold
  };
  for (int gr = 0; gr < WS_D; ++gr) issue_raw(gr);
  bool stalled = false;
  int g_done = 0;  // groups this thread has arrived on
  for (int g = 0; g < ngr; ++g) {
    // raw group g: committed WS_D calls ago; 2 (WS_D - 1) younger groups may still be in flight
    if (g < WS_D - 1) cp_async_wait<0>();
    else cp_async_wait<2 * (WS_D - 1)>();
    const int slot = g % WS_R;
    __syncwarp();
    if (g >= WS_R && !warp_wait(empty + slot, ((unsigned)(g / WS_R) & 1u) ^ 1u, abort_flag, P.wait_limit)) {
      stalled = true;
      break;
    }
    const int rs = g % WS_RR;
    uint8_t* fb = reinterpret_cast<uint8_t*>(flg + (size_t)slot * sb);
    for (int t = ptid; t < ntaskp; t += nprep) {  // the same task order as issue_raw
      const int c = (int)(((uint32_t)t * sbm) >> 20), s = t - c * sbp;
      const int64_t b = b0 + s;
      const int gc = g * WS_G + c;
      if (s >= sb || b >= P.batch || gc >= nch) continue;
      const int4 s4 = rsym[((size_t)rs * WS_G + c) * sb + s];
      const int4 k4 = ridx[((size_t)rs * WS_G + c) * sb + s];
      const int32_t sv[4] = {s4.x, s4.y, s4.z, s4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
      bool exact = false;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t kc = min((uint32_t)kv[q], kmax);
        exact |= (uint32_t)kv[q] > kmax;
        const int2 ti = tso[((int)kc << tcl) + (lane & tcm)];  // {size, offset}, this lane's copy
        const int32_t v = (int32_t)((uint32_t)sv[q] - (uint32_t)ti.y);
        exact |= v < 0 || v >= ti.x - 1 || (int64_t)v > emax;
        if constexpr (BYPASS) exact |= v >= ti.x - 2;  // escape slot or beyond: escape coding
        const int64_t vc = min((int64_t)max(v, 0), emax);
        const size_t eo = ((size_t)slot * 4 * WS_G + 4 * c + q) * sb + s;
        cp_async16(ent + eo, P.enc + (int64_t)kc * P.enc_stride + vc, 16);
        if constexpr (ALIAS) kix[eo] = (int32_t)kc;
      }
      fb[(size_t)s * 4 + c] = exact ? 1 : 0;
    }
    cp_async_commit();
    mbar_arrive(full + slot);
    mbar_arrive_cp_async(full + slot);
    issue_raw(g + WS_D);
    g_done = g + 1;
  }
  if (stalled) {
    if (lane == 0) *abort_flag = 1;
    if (lane == 0) report(P.status, DEV_STALLED);
  }
  cp_async_wait<0>();
  if (*abort_flag) {
    // the chain warps may have left already: before this thread leaves, wait (bounded) until the
    // arrivals its copies trigger on the last groups' full barriers have landed, so that none of
    // them reaches the block's shared memory after the block is gone
    for (int g2 = g_done > WS_R ? g_done - WS_R : 0; g2 < g_done; ++g2)
      for (unsigned it = 0; it < (1u << 16) && !mbar_try_wait(full + g2 % WS_R, (unsigned)(g2 / WS_R) & 1u); ++it) {
      }
  }
}

template <int V>
bool launch_push_ws(const PushParams& P, bool alias, bool bypass, bool rsmem, int blocks, int threads, int sb,
                    int chain_warps, size_t smem, cudaStream_t s);

template <int V, bool A, bool B, bool R>
void pushws_go(const PushParams& P, int blocks, int threads, int sb, int chain_warps, size_t smem, cudaStream_t s) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(push_ws_kernel<V, A, B, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  push_ws_kernel<V, A, B, R><<<blocks, threads, smem, s>>>(P, sb, chain_warps);
  note_launch();
}

#define TANS_DEFINE_PUSH_WS(VV)                                                                              \
  template <>                                                                                                \
  bool launch_push_ws<VV>(const PushParams& P, bool alias, bool bypass, bool rsmem, int blocks, int threads, \
                          int sb, int cw, size_t smem, cudaStream_t s) {                                     \
    if (alias) {                                                                                             \
      if (bypass) {                                                                                          \
        if (rsmem) pushws_go<VV, true, true, true>(P, blocks, threads, sb, cw, smem, s);                     \
        else pushws_go<VV, true, true, false>(P, blocks, threads, sb, cw, smem, s);                          \
      } else {                                                                                               \
        if (rsmem) pushws_go<VV, true, false, true>(P, blocks, threads, sb, cw, smem, s);                    \
        else pushws_go<VV, true, false, false>(P, blocks, threads, sb, cw, smem, s);                         \
      }                                                                                                      \
    } else {                                                                                                 \
      if (bypass) pushws_go<VV, false, true, false>(P, blocks, threads, sb, cw, smem, s);                    \
      else pushws_go<VV, false, false, false>(P, blocks, threads, sb, cw, smem, s);                          \
    }                                                                                                        \
    return true;                                                                                             \
  }

}  // namespace tans
