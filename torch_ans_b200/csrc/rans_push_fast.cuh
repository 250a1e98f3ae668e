// rans_push_fast.cuh -- the fast single-state push kernel (rows 16-byte aligned, length % 4 == 0,
// at most 4096 tables, frequency precision <= 23 so entries carry their packed shift).
//
// Per thread one stream, walked from its last 4-symbol chunk to its first in time steps:
//   (1) cp.async the symbol and index chunk PF_L1 + PF_L2 steps ahead of its chain;
//   (2) prep the chunk PF_L2 steps ahead: table info from shared memory, value = symbol - offset,
//       and a cp.async gather of the four 16-byte encode entries {reciprocal, freq, start};
//       anything the straight-line chain cannot do (bad index, symbol outside the table, an
//       escape, a zero frequency, a stream row too short) marks the chunk "exact";
//   (3) commit, wait for the group PF_L2 - 1 steps old;
//   (4) run the chunk: a marked chunk goes through the reference-exact step code, otherwise four
//       straight-line steps (compare, predicated word store, multiply-high quotient,
//       multiply-add).
// The alias remap rows are staged in shared memory when they fit.
#pragma once

#include "rans_push_common.cuh"

namespace tans {

constexpr int PF_L1 = 4;   // raw chunk -> prep
constexpr int PF_L2 = 4;   // prep -> chain (FIFO deadline of both loads)
constexpr int PF_RS = 16;  // raw ring slots (> PF_L1 + PF_L2: the exact path rereads from global)
constexpr int PF_ES = 8;   // entry ring slots (> PF_L2)

inline int64_t pushf_smem_bytes(int64_t nact, int64_t ntables, int64_t remap_entries) {
  return nact * (PF_RS * 32 + PF_ES * 64 + PF_ES * 4) + ntables * 16 + remap_entries * 4;
}

template <int V, bool ALIAS, bool BYPASS, bool RSMEM>
__global__ void __launch_bounds__(512) push_fast_kernel(const PushParams P) {
  using S = typename VT<V>::State;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  const int warps = T >> 5, warp = tid >> 5, lane = tid & 31;
  const int nact = warps * P.lanes;
  const int at = warp * P.lanes + lane;
  int4* rsym = reinterpret_cast<int4*>(smem_raw);
  int4* ridx = rsym + PF_RS * nact;
  uint4* ent = reinterpret_cast<uint4*>(ridx + PF_RS * nact);
  uint32_t* flg = reinterpret_cast<uint32_t*>(ent + PF_ES * 4 * nact);
  TableInfo* tsm = reinterpret_cast<TableInfo*>(flg + PF_ES * nact);
  int32_t* rsm = reinterpret_cast<int32_t*>(tsm + P.ntables);  // alias remap rows (RSMEM)
  const int64_t M = (int64_t)1 << P.fp;
  for (int64_t k = tid; k < P.ntables; k += T) tsm[k] = P.tinfo[k];
  if constexpr (ALIAS && RSMEM) {
    for (int64_t i = tid; i < P.ntables * M; i += T) {
      const int64_t k = i >> P.fp, r = i & (M - 1);
      const int32_t sz = P.tinfo[k].size;
      const int64_t col = (int64_t)sz + r;
      rsm[i] = (sz >= 0 && col < P.cdf_width) ? P.cdfs[k * P.cdf_width + col] : 0;
    }
  }
  __syncthreads();
  if (lane >= P.lanes) return;
  const int64_t b = ((int64_t)blockIdx.x * warps + warp) * P.lanes + lane;
  if (b >= P.batch) return;

  int32_t* row = P.stream + b * P.width;
  PushCursor<V> cur;
  cur.payload = reinterpret_cast<uint8_t*>(row + 1);
  cur.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
  cur.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
  cur.err = 0;
  S x = load_state<V>(row, 0);
  uint32_t perr = 0;
  const int64_t N = P.nsym;
  const int nch = (int)(N >> 2);
  const int32_t* srow = P.sym + b * N;
  const int32_t* irow = P.idx + b * N;
  const uint32_t kmax = (uint32_t)(P.ntables - 1);
  const int64_t emax = P.enc_stride - 1;
  // a row whose length points outside it is coded by the exact path only
  const bool row_ok = cur.p >= -1 && cur.p < cur.cap;

  for (int t = 0; t < nch + PF_L1 + PF_L2; ++t) {
    const int cr = nch - 1 - t;  // raw chunk issued now
    if (cr >= 0) {
      const int rs = cr & (PF_RS - 1);
      cp_async16(rsym + rs * nact + at, srow + 4 * (int64_t)cr, 16);
      cp_async16(ridx + rs * nact + at, irow + 4 * (int64_t)cr, 16);
    }
    const int cp = cr + PF_L1;  // chunk prepped now
    if (cp >= 0 && cp < nch) {
      const int rs = cp & (PF_RS - 1), es = cp & (PF_ES - 1);
      const int4 s4 = rsym[rs * nact + at], k4 = ridx[rs * nact + at];
      const int32_t sv[4] = {s4.x, s4.y, s4.z, s4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
      bool exact = !row_ok;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t kc = min((uint32_t)kv[q], kmax);
        exact |= (uint32_t)kv[q] > kmax;
        const TableInfo ti = tsm[kc];
        const int32_t v = (int32_t)((uint32_t)sv[q] - (uint32_t)ti.offset);
        exact |= v < 0 || v >= ti.size - 1 || (int64_t)v > emax;
        if constexpr (BYPASS) exact |= v >= ti.size - 2;  // escape slot or beyond: escape coding
        const int64_t vc = min((int64_t)max(v, 0), emax);
        cp_async16(ent + (es * 4 + q) * nact + at, P.enc + (int64_t)kc * P.enc_stride + vc, 16);
      }
      flg[es * nact + at] = exact ? 1u : 0u;
    }
    cp_async_commit();
    cp_async_wait<PF_L2 - 1>();
    const int cc = cp + PF_L2;  // chunk coded now
    if (cc < 0 || cc >= nch) continue;
    const int es = cc & (PF_ES - 1);
    uint4 e[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) e[q] = ent[(es * 4 + q) * nact + at];
    bool exact = flg[es * nact + at] != 0u;
#pragma unroll
    for (int q = 0; q < 4; ++q) exact |= entry_freq(e[q], true) - 1u >= (1u << P.fp);  // 0 or above 2^fp
    if (exact) {
      // reference-exact steps, last symbol of the chunk first
#pragma unroll 1
      for (int q = 3; q >= 0; --q) {
        const int64_t i = 4 * (int64_t)cc + q;
        const PushPrep r = push_prepare<V, ALIAS, BYPASS>(P, __ldg(srow + i), __ldg(irow + i), true, perr);
        push_chain<V, ALIAS, BYPASS>(P, x, cur, r);
      }
      continue;
    }
    int32_t kq[4] = {0, 0, 0, 0};
    if constexpr (ALIAS) {
      const int4 k4 = ridx[(cc & (PF_RS - 1)) * nact + at];
      kq[0] = k4.x;
      kq[1] = k4.y;
      kq[2] = k4.z;
      kq[3] = k4.w;
    }
#pragma unroll
    for (int q = 3; q >= 0; --q) {
      const uint32_t freq = entry_freq(e[q], true);
      const unsigned long long bound = (unsigned long long)freq << (VT<V>::USED - P.fp);
#pragma unroll
      for (int u = 0; u < VT<V>::MAX_RENORM; ++u) {
        const bool r = (unsigned long long)x >= bound;
        if (r) cur.emit(x);
      }
      const S qt = quotient<V>(x, e[q], true);
      const S start = to_state<S>((int32_t)e[q].w);
      if constexpr (ALIAS) {
        // the raw ring still holds this chunk's indexes (PF_RS > PF_L1 + PF_L2)
        // same bounds rule as push_chain: a remap index outside the row skips the step
        const uint32_t kc = min((uint32_t)kq[q], kmax);
        const S ri = (S)(x - qt * (S)freq + start);
        const int32_t sz = tsm[kc].size;
        const long long rcap = P.cdf_width - (long long)sz;
        int32_t rv = 0;
        bool ok = (unsigned long long)ri < (unsigned long long)(rcap > 0 ? rcap : 0);
        if constexpr (RSMEM) {
          if ((unsigned long long)ri < (unsigned long long)M) rv = rsm[((int64_t)kc << P.fp) + (int64_t)ri];
          else if (ok) rv = __ldg(P.cdfs + (int64_t)kc * P.cdf_width + sz + (int64_t)ri);
        } else {
          if (ok) rv = __ldg(P.cdfs + (int64_t)kc * P.cdf_width + sz + (int64_t)ri);
        }
        if (ok) x = (S)((qt << P.fp) + to_state<S>(rv));
        else cur.err |= DEV_BAD_VALUE;
      } else {
        const S cmpl = (S)((S)1 << P.fp) - (S)freq;
        x = (S)(x + start + qt * cmpl);
      }
    }
  }
  cp_async_wait<0>();
  store_state<V>(row, 0, x);
  row[0] = (int32_t)((cur.p + 1) * VT<V>::WBYTES);
  report(P.status, cur.err | perr);
}

template <int V>
bool launch_push_fast(const PushParams& P, bool alias, bool bypass, bool rsmem, int blocks, int threads, size_t smem,
                      cudaStream_t s);

template <int V, bool A, bool B, bool R>
void pushf_go(const PushParams& P, int blocks, int threads, size_t smem, cudaStream_t s) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(push_fast_kernel<V, A, B, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  push_fast_kernel<V, A, B, R><<<blocks, threads, smem, s>>>(P);
  note_launch();
}

#define TANS_DEFINE_PUSH_FAST(VV)                                                                             \
  template <>                                                                                                 \
  bool launch_push_fast<VV>(const PushParams& P, bool alias, bool bypass, bool rsmem, int blocks, int threads, \
                            size_t smem, cudaStream_t s) {                                                    \
    if (alias) {                                                                                              \
      if (bypass) {                                                                                           \
        if (rsmem) pushf_go<VV, true, true, true>(P, blocks, threads, smem, s);                               \
        else pushf_go<VV, true, true, false>(P, blocks, threads, smem, s);                                    \
      } else {                                                                                                \
        if (rsmem) pushf_go<VV, true, false, true>(P, blocks, threads, smem, s);                              \
        else pushf_go<VV, true, false, false>(P, blocks, threads, smem, s);                                   \
      }                                                                                                       \
    } else {                                                                                                  \
      if (bypass) pushf_go<VV, false, true, false>(P, blocks, threads, smem, s);                              \
      else pushf_go<VV, false, false, false>(P, blocks, threads, smem, s);                                    \
    }                                                                                                         \
    return true;                                                                                              \
  }

}  // namespace tans
