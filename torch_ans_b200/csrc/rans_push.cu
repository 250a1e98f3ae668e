// rans_push.cu -- encode (push) kernels and the tans_push C entry point.
//
// Replaces the reference's rans_push_indexed_cpu / rans_push_indexed_cuda
// (torch_ans/rans_cpu.cpp:44-189, torch_ans/rans_cuda.cu:20-167): per stream, symbols are pushed
// last-first onto the stream row with the step of torch_ans/rans_utils.hpp:168-323.
//
// B200 design:
//  * one thread per stream (launch.cuh spreads streams over all SMs);
//  * a per-call prep kernel turns every (table, symbol) of the cdf list into a 16-byte entry
//    {reciprocal, freq, start}, so the serial chain of a step is compare/emit + multiply-high
//    + multiply-add instead of a 64-bit division (rans_device.cuh);
//  * symbol/index rows are read with 16-byte vector loads four chunks (16 symbols) ahead of the
//    chain, and table entries two chunks ahead, so no memory latency sits on the chain except
//    the alias remap lookup, which is part of the algorithm.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <string>

#include "../../include/torch_ans_b200.h"
#include "launch.cuh"
#include "rans_device.cuh"
#include "rans_host.h"
#include "rans_push_common.cuh"
#include "rans_push_fast.cuh"
#include "rans_push_ws.cuh"

namespace tans {

// ---------------------------------------------------------------- prep: table info + entries
__global__ void build_table_info_kernel(const int32_t* sizes, const int32_t* offsets, int64_t ntables,
                                        int fp, TableInfo* out) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < ntables;
       k += (int64_t)gridDim.x * blockDim.x) {
    TableInfo t;
    t.size = sizes[k];
    t.offset = offsets ? offsets[k] : 0;
    // alias cut width of rans_utils.hpp:413: (1 << fp) / (cdf_size - 1); 0 marks "unusable"
    t.cut = (t.size - 1 > 0) ? (int32_t)((1 << fp) / (t.size - 1)) : 0;
    t.cut_log2 = (t.cut > 0 && (t.cut & (t.cut - 1)) == 0) ? (31 - __clz(t.cut)) : -1;
    out[k] = t;
  }
}

template <int V>
__global__ void build_push_entries_kernel(const int32_t* cdfs, int64_t ntables, int64_t cdf_width,
                                          int64_t stride, int fp, uint4* enc) {
  const int64_t total = ntables * stride;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = e / stride, v = e - k * stride;
    const int32_t* row = cdfs + k * cdf_width;
    const int32_t start = row[v];
    const int32_t freq = (int32_t)((uint32_t)row[v + 1] - (uint32_t)start);
    uint4 out;
    out.w = (uint32_t)start;
    // at fp <= 23 the shift is packed above a 24-bit frequency; a step of 2^24 or more there is
    // larger than the whole cdf range (no quantised cdf has one) and is reported as a bad frequency
    if (freq <= 0 || (fp <= 23 && freq >= (1 << 24))) {
      out.x = out.y = out.z = 0u;
    } else {
      const uint32_t d = (uint32_t)freq;
      out.z = fp <= 23 ? (d | (ceil_log2(d) << 24)) : d;
      if constexpr (V == 0) {
        const unsigned long long m = recip64(d);
        out.x = (uint32_t)m;
        out.y = (uint32_t)(m >> 32);
      } else {
        out.x = recip32(d);
        out.y = 0u;
      }
    }
    enc[e] = out;
  }
}

// ---------------------------------------------------------------- single-state kernel
// Software pipeline over chunks of 4 symbols (walked from the end of the row to its start), all
// staging in shared memory so nothing in flight is ever held in a register:
//   time t: (1) cp.async the symbol/index chunk x = c_hi - t                      (raw ring)
//           (2) prep chunk x + L1: table info, escape transform, cp.async of the  (entry ring)
//               four 16-byte encode entries
//           (3) commit; wait until at most L2-1 groups are pending
//           (4) run the serial chain over chunk x + L1 + L2 (its entries landed)
// Ring slots are laid out [slot][thread] so a warp's 16-byte accesses hit distinct banks.
constexpr int PUSH_RS = 8;  // raw slots (> L1)
constexpr int PUSH_ES = 4;  // entry slots (> L2)
constexpr int PUSH_L1 = 4;
constexpr int PUSH_L2 = 3;
constexpr int64_t kTinfoSmemMax = 4096;  // tables whose info is staged in shared memory

__host__ __device__ constexpr int push_smem_per_thread(bool alias, bool bypass) {
  return 2 * PUSH_RS * 16 + PUSH_ES * 4 * 16 + PUSH_ES * 4 + (bypass ? PUSH_ES * 16 : 0) + (alias ? PUSH_ES * 16 : 0);
}

__device__ __forceinline__ void issue_raw_chunk(int4* dst, const int32_t* a, int64_t c, int64_t total, bool vec) {
  const int64_t g = c * 4;
  if (vec && g >= 0 && g + 4 <= total) {
    cp_async16(dst, a + g, 16);
    return;
  }
  int32_t* d = reinterpret_cast<int32_t*>(dst);
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (g + e >= 0 && g + e < total) cp_async4(d + e, a + g + e);
}

template <int V, bool ALIAS, bool BYPASS>
__global__ void __launch_bounds__(256) push_i1_kernel(const PushParams P) {
  using S = typename VT<V>::State;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int T = blockDim.x, tid = threadIdx.x;
  int4* raw_sym = reinterpret_cast<int4*>(smem_raw);
  int4* raw_idx = raw_sym + PUSH_RS * T;
  uint4* ent = reinterpret_cast<uint4*>(raw_idx + PUSH_RS * T);
  uint32_t* flg = reinterpret_cast<uint32_t*>(ent + PUSH_ES * 4 * T);
  int4* escv = reinterpret_cast<int4*>(flg + PUSH_ES * T);
  int4* kslot = escv + (BYPASS ? PUSH_ES * T : 0);
  TableInfo* tsm = reinterpret_cast<TableInfo*>(kslot + (ALIAS ? PUSH_ES * T : 0));
  const bool tin_smem = P.tin_smem != 0;
  if (tin_smem) {
    for (int64_t k = tid; k < P.ntables; k += T) tsm[k] = P.tinfo[k];
    __syncthreads();
  }
  const TableInfo* tin = tin_smem ? tsm : P.tinfo;

  const int64_t b = my_stream(P.lanes, P.batch);
  if (b < 0) return;
  int32_t* row = P.stream + b * P.width;
  PushCursor<V> cur;
  cur.payload = reinterpret_cast<uint8_t*>(row + 1);
  cur.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
  cur.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
  cur.err = 0;
  S x = load_state<V>(row, 0);
  uint32_t perr = 0;
  const int64_t lo = b * P.nsym, hi = lo + P.nsym, total = P.batch * P.nsym;
  const bool vec = P.vec != 0;

  if (P.nsym > 0) {
    const int64_t c_hi = (hi - 1) >> 2, c_lo = lo >> 2;
    const int64_t t_end = (c_hi - c_lo) + PUSH_L1 + PUSH_L2;
    for (int64_t t = 0; t <= t_end; ++t) {
      // (1) raw chunk
      const int64_t xr = c_hi - t;
      if (xr >= c_lo) {
        const int rs = (int)(xr & (PUSH_RS - 1));
        issue_raw_chunk(raw_sym + rs * T + tid, P.sym, xr, total, vec);
        issue_raw_chunk(raw_idx + rs * T + tid, P.idx, xr, total, vec);
      }
      // (2) prep
      const int64_t xp = xr + PUSH_L1;
      if (xp >= c_lo && xp <= c_hi) {
        const int rs = (int)(xp & (PUSH_RS - 1)), es = (int)(xp & (PUSH_ES - 1));
        const int4 s4 = raw_sym[rs * T + tid], k4 = raw_idx[rs * T + tid];
        const int32_t sv[4] = {s4.x, s4.y, s4.z, s4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
        uint32_t flags = 0;
        int32_t esc[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t g = xp * 4 + j;
          uint32_t f = PREP_SKIP;
          if (g >= lo && g < hi) {
            const int32_t k = kv[j];
            if (k < 0 || (int64_t)k >= P.ntables) {
              perr |= DEV_BAD_INDEX;
            } else {
              const TableInfo ti = tin_smem ? tin[k] : load_tinfo(P.tinfo, k);
              int32_t v = (int32_t)((uint32_t)sv[j] - (uint32_t)ti.offset);
              const int32_t maxv = ti.size - 2;
              f = 0;
              if constexpr (BYPASS) {
                if (v < 0) {
                  esc[j] = -2 * v - 1;
                  v = maxv;
                } else if (v >= maxv) {
                  esc[j] = 2 * (v - maxv);
                  v = maxv;
                }
                if (v == maxv) f = PREP_ESC;
              }
              if (v < 0 || v >= ti.size - 1 || (int64_t)v >= P.enc_stride) {
                perr |= DEV_BAD_VALUE;
                f = PREP_SKIP;
              } else {
                cp_async16(ent + (es * 4 + j) * T + tid, P.enc + (int64_t)k * P.enc_stride + v, 16);
              }
            }
          }
          flags |= f << (8 * j);
        }
        flg[es * T + tid] = flags;
        if constexpr (BYPASS) escv[es * T + tid] = make_int4(esc[0], esc[1], esc[2], esc[3]);
        if constexpr (ALIAS) kslot[es * T + tid] = k4;
      }
      // (3)
      cp_async_commit();
      cp_async_wait<PUSH_L2 - 1>();
      // (4) chain, last symbol of the chunk first
      const int64_t xc = xp + PUSH_L2;
      if (xc >= c_lo && xc <= c_hi) {
        const int es = (int)(xc & (PUSH_ES - 1));
        const uint32_t flags = flg[es * T + tid];
        int4 escq = make_int4(0, 0, 0, 0), kq = make_int4(0, 0, 0, 0);
        if constexpr (BYPASS) escq = escv[es * T + tid];
        if constexpr (ALIAS) kq = kslot[es * T + tid];
        const int32_t escs[4] = {escq.x, escq.y, escq.z, escq.w};
        const int32_t ks[4] = {kq.x, kq.y, kq.z, kq.w};
#pragma unroll
        for (int j = 3; j >= 0; --j) {
          const uint32_t f = (flags >> (8 * j)) & 0xffu;
          if (f & PREP_SKIP) continue;
          PushPrep r;
          r.flags = f;
          r.raw = escs[j];
          r.e = ent[(es * 4 + j) * T + tid];
          r.rbase = 0;
          r.rcap = 0;
          if constexpr (ALIAS) {
            const TableInfo ti = tin_smem ? tin[ks[j]] : load_tinfo(P.tinfo, ks[j]);
            r.rbase = (int64_t)ks[j] * P.cdf_width + ti.size;
            const int64_t cap = P.cdf_width - ti.size;
            r.rcap = cap <= 0 ? 0 : (cap > 0x7fffffff ? 0x7fffffff : (int32_t)cap);
          }
          push_chain<V, ALIAS, BYPASS>(P, x, cur, r);
        }
      }
    }
    cp_async_wait<0>();
  }
  store_state<V>(row, 0, x);
  row[0] = (int32_t)((cur.p + 1) * VT<V>::WBYTES);
  report(P.status, cur.err | perr);
}

// ---------------------------------------------------------------- four-state (i4) kernel
// rans_cpu.cpp:89-160: the last N % 4 symbols first (state i % 4, escapes inline), then blocks
// [i-3, i] with i = 3 (mod 4): escapes of the whole block first (symbol i-j -> state 3-j, j=0..3),
// then the four symbols.  The four states are independent chains, so a block has 4-way ILP.
template <int V, bool ALIAS, bool BYPASS>
__global__ void __launch_bounds__(256) push_i4_kernel(const PushParams P) {
  using S = typename VT<V>::State;
  const int64_t b = my_stream(P.lanes, P.batch);
  if (b < 0) return;
  int32_t* row = P.stream + b * P.width;
  PushCursor<V> cur;
  cur.payload = reinterpret_cast<uint8_t*>(row + 1);
  cur.p = (int64_t)row[0] / VT<V>::WBYTES - 1;
  cur.cap = (P.width - 1) * 4 / VT<V>::WBYTES;
  cur.err = 0;
  S x[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) x[k] = load_state<V>(row, k);
  uint32_t perr = 0;
  const int32_t* sym = P.sym + b * P.nsym;
  const int32_t* idx = P.idx + b * P.nsym;
  const int64_t N = P.nsym;
  const int64_t first = N % 4;
  int64_t i = N - 1;
  for (; i >= N - first; --i) {
    const PushPrep r = push_prepare<V, ALIAS, BYPASS>(P, __ldg(sym + i), __ldg(idx + i), true, perr);
    switch (i & 3) {  // state index i % 4 (i >= 0)
      case 0: push_chain<V, ALIAS, BYPASS>(P, x[0], cur, r); break;
      case 1: push_chain<V, ALIAS, BYPASS>(P, x[1], cur, r); break;
      case 2: push_chain<V, ALIAS, BYPASS>(P, x[2], cur, r); break;
      default: push_chain<V, ALIAS, BYPASS>(P, x[3], cur, r); break;
    }
  }
  for (; i >= 0; i -= 4) {
    PushPrep r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = push_prepare<V, ALIAS, BYPASS>(P, __ldg(sym + i - j), __ldg(idx + i - j), true, perr);
    if constexpr (BYPASS) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (!(r[j].flags & PREP_SKIP) && (r[j].flags & PREP_ESC)) {
          push_escape<V>(x[3 - j], cur, r[j].raw, P.bp);
        }
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j].flags &= ~PREP_ESC;  // escapes already pushed
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) push_chain<V, ALIAS, BYPASS>(P, x[3 - j], cur, r[j]);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) store_state<V>(row, k, x[k]);
  row[0] = (int32_t)((cur.p + 1) * VT<V>::WBYTES);
  report(P.status, cur.err | perr);
}

// ---------------------------------------------------------------- host side
size_t push_workspace_bytes(int variant, int64_t ntables, int64_t enc_stride) {
  (void)variant;
  return align_up((size_t)ntables * sizeof(TableInfo)) + align_up((size_t)ntables * enc_stride * sizeof(uint4));
}

template <int V, bool ALIAS, bool BYPASS>
static void launch_push(const PushParams& P, int interleave, const LaunchShape& L, cudaStream_t s) {
  note_launch();
  if (interleave == 4) {
    push_i4_kernel<V, ALIAS, BYPASS><<<L.blocks, L.threads, 0, s>>>(P);
    return;
  }
  size_t smem = (size_t)L.threads * push_smem_per_thread(ALIAS, BYPASS);
  if (P.tin_smem) smem += (size_t)P.ntables * sizeof(TableInfo);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(push_i1_kernel<V, ALIAS, BYPASS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  push_i1_kernel<V, ALIAS, BYPASS><<<L.blocks, L.threads, smem, s>>>(P);
}

template <int V>
static void launch_push_v(const PushParams& P, bool alias, bool bypass, int interleave, const LaunchShape& L,
                          cudaStream_t s) {
  if (alias) {
    if (bypass) launch_push<V, true, true>(P, interleave, L, s);
    else launch_push<V, true, false>(P, interleave, L, s);
  } else {
    if (bypass) launch_push<V, false, true>(P, interleave, L, s);
    else launch_push<V, false, false>(P, interleave, L, s);
  }
}

// TORCH_ANS_B200_PUSH_KERNEL: "ws" (warp-specialised, default), "chunk" (single-role fast kernel)
// or "generic"; each falls through to the next when its preconditions do not hold
static int push_kernel_choice() {
  const char* e = std::getenv("TORCH_ANS_B200_PUSH_KERNEL");
  if (!e || !*e) return 0;
  const std::string v(e);
  if (v == "chunk") return 1;
  if (v == "generic") return 2;
  return 0;
}

int64_t push_entry_stride(int64_t cdf_width, int fp) {
  // entries exist for v < cdf_width - 1, and no usable table has more than 2^fp + 1 symbols;
  // an empty row (cdf_width 0 or 1) has no entries
  const int64_t a = cdf_width > 1 ? cdf_width - 1 : 0, b = ((int64_t)1 << fp) + 1;
  return a < b ? a : b;
}

int push_impl(int variant, int use_alias, int interleave, int32_t* stream, int64_t batch, int64_t width,
              const int32_t* symbols, const int32_t* indexes, int64_t nsym, const int32_t* cdfs, int64_t ntables,
              int64_t cdf_width, const int32_t* sizes, const int32_t* offsets, int fp, int bypass, int bp,
              void* workspace, size_t ws_bytes, uint32_t* status, cudaStream_t s, bool allow_alloc) {
  int rc = check_coding_args(variant, interleave, stream, batch, width, indexes, nsym, cdfs, ntables, cdf_width,
                             sizes, fp, bypass, bp);
  if (rc != TANS_OK) return rc;
  if (nsym > 0 && !symbols) return TANS_E_INVALID_ARGUMENT;
  if (batch == 0) return TANS_OK;
  const int64_t stride = push_entry_stride(cdf_width, fp);
  const size_t need = push_workspace_bytes(variant, ntables, stride);
  void* ws = workspace;
  bool owned = false;
  if (!ws && need > 0) {  // an empty table list needs no scratch at all
    if (!allow_alloc) return TANS_E_WORKSPACE;
    if (cudaMallocAsync(&ws, need, s) != cudaSuccess) return TANS_E_CUDA;
    owned = true;
  } else if (ws_bytes < need) {
    return TANS_E_WORKSPACE;
  }
  TableInfo* tinfo = reinterpret_cast<TableInfo*>(ws);
  uint4* enc = reinterpret_cast<uint4*>(reinterpret_cast<char*>(ws) + align_up((size_t)ntables * sizeof(TableInfo)));
  const int dev_sms = sm_count();
  {
    const int64_t n = ntables;
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4 * (int64_t)dev_sms);
    build_table_info_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(sizes, offsets, ntables, fp, tinfo);
    note_launch();
    const int64_t m = ntables * stride;
    const int eb = (int)std::min<int64_t>((m + 255) / 256, 16 * (int64_t)dev_sms);
    if (m > 0) {
      if (variant == TANS_RANS64) build_push_entries_kernel<0><<<eb, 256, 0, s>>>(cdfs, ntables, cdf_width, stride, fp, enc);
      else if (variant == TANS_RANS32) build_push_entries_kernel<1><<<eb, 256, 0, s>>>(cdfs, ntables, cdf_width, stride, fp, enc);
      else build_push_entries_kernel<2><<<eb, 256, 0, s>>>(cdfs, ntables, cdf_width, stride, fp, enc);
      note_launch();
    }
  }
  PushParams P;
  P.stream = stream;
  P.batch = batch;
  P.width = width;
  P.sym = symbols;
  P.idx = indexes;
  P.nsym = nsym;
  P.enc = enc;
  P.enc_stride = stride;
  P.tinfo = tinfo;
  P.ntables = ntables;
  P.cdfs = cdfs;
  P.cdf_width = cdf_width;
  P.fp = fp;
  P.bp = bp;
  P.status = status;
  P.vec = ((reinterpret_cast<uintptr_t>(symbols) | reinterpret_cast<uintptr_t>(indexes)) & 15u) == 0;
  const int choice = push_kernel_choice();
  const bool fast_ok = interleave == 1 && nsym > 0 && nsym % 4 == 0 && P.vec && ntables <= 4096 && fp <= 23 &&
                       nsym / 4 < 0x7fffffff;
  // ---- warp-specialised kernel: chain warps fed by prep warps through a shared-memory ring
  if (fast_ok && choice == 0 && (width - 1) * 4 / ((variant == TANS_RANS64) ? 4 : (variant == TANS_RANS32 ? 1 : 2)) <
                                     (int64_t)0x7fffff00) {
    const int64_t M = (int64_t)1 << fp;
    const int64_t remap = use_alias ? ntables * M : 0;
    const int64_t budget = 200 * 1024;
    const int tc_env = env_int("TORCH_ANS_B200_PUSHWS_TCOPIES", 0);
    const int tcopies = (tc_env == 1 || tc_env == 16) ? tc_env : pushws_tcopies(ntables);
    const bool rsmem = use_alias && pushws_smem_bytes(1, true, ntables, remap, tcopies) <= budget;
    const int64_t fixed = pushws_smem_bytes(0, use_alias != 0, ntables, rsmem ? remap : 0, tcopies);
    const int64_t per = pushws_stream_bytes(use_alias != 0);
    const int64_t sb_max = fixed < budget ? (budget - fixed) / per : 0;
    int64_t sb = (batch + dev_sms - 1) / dev_sms;
    const int sb_env = env_int("TORCH_ANS_B200_PUSHWS_STREAMS", 0);
    if (sb_env > 0) sb = sb_env;
    sb = std::min<int64_t>(sb, std::min<int64_t>(sb_max, 128));
    if (sb >= 1) {
      // chain warps: up to 4, with about 7 lanes or more each (mixture tables at a quarter length:
      // 7 streams per block 4.88 ms on 1 warp vs 4.97 on 2; 14 streams 5.01 on 2 warps vs 5.28 on
      // 4; 28 streams 5.30 on 4 vs 5.31 on 2; 56 streams: 4 warps best)
      int64_t cw = std::min<int64_t>(env_int("TORCH_ANS_B200_PUSHWS_CHAIN_WARPS", (int)std::min<int64_t>(4, (sb + 6) / 7)), sb);
      cw = std::max<int64_t>(1, std::min<int64_t>(cw, 8));
      // whole lanes per chain warp, then only the warps those lanes need
      const int64_t lanes = std::min<int64_t>(32, (sb + cw - 1) / cw);
      cw = (sb + lanes - 1) / lanes;
      int64_t pw = env_int("TORCH_ANS_B200_PUSHWS_PREP_WARPS", 0);
      if (pw <= 0) pw = std::max<int64_t>(1, std::min<int64_t>(4, (WS_G * sb + 31) / 32));
      pw = std::min<int64_t>(pw, 8);
      const int blocks = (int)((batch + sb - 1) / sb);
      const size_t smem = (size_t)(fixed + sb * per);
      P.lanes = (int)lanes;
      P.ws_tcopies = tcopies;
      const int wl = env_int("TORCH_ANS_B200_WAIT_LIMIT", -1);
      P.wait_limit = wl >= 0 ? (unsigned)wl : WS_WAIT_LIMIT;
      bool ok;
      if (variant == TANS_RANS64)
        ok = launch_push_ws<0>(P, use_alias != 0, bypass != 0, rsmem, blocks, (int)((cw + pw) * 32), (int)sb, (int)cw, smem, s);
      else if (variant == TANS_RANS32)
        ok = launch_push_ws<1>(P, use_alias != 0, bypass != 0, rsmem, blocks, (int)((cw + pw) * 32), (int)sb, (int)cw, smem, s);
      else
        ok = launch_push_ws<2>(P, use_alias != 0, bypass != 0, rsmem, blocks, (int)((cw + pw) * 32), (int)sb, (int)cw, smem, s);
      if (owned) cudaFreeAsync(ws, s);
      if (!ok) return TANS_E_INVALID_ARGUMENT;
      return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
    }
  }
  // ---- fast kernel: aligned rows, length % 4 == 0, table info in shared memory
  if (fast_ok && choice <= 1) {
    const int64_t per_sm = (batch + dev_sms - 1) / dev_sms;
    int64_t warps = std::min<int64_t>(per_sm, env_int("TORCH_ANS_B200_PUSH_WARPS", 4));
    if (warps < 1) warps = 1;
    int64_t lanes = (per_sm + warps - 1) / warps;
    if (lanes > 32) {
      lanes = 32;
      warps = std::min<int64_t>(16, (per_sm + 31) / 32);
    }
    const int lanes_env = env_int("TORCH_ANS_B200_PUSH_LANES", 0);
    if (lanes_env > 0 && lanes_env <= 32) lanes = lanes_env;
    const int64_t nact = warps * lanes;
    const int64_t M = (int64_t)1 << fp;
    const int64_t base = pushf_smem_bytes(nact, ntables, 0);
    const bool rsmem = use_alias && base + ntables * M * 4 <= 200 * 1024;
    const int64_t smem = rsmem ? base + ntables * M * 4 : base;
    if (smem <= 200 * 1024) {
      P.lanes = (int)lanes;
      const int blocks = (int)((batch + nact - 1) / nact);
      bool ok;
      if (variant == TANS_RANS64) ok = launch_push_fast<0>(P, use_alias != 0, bypass != 0, rsmem, blocks, (int)(warps * 32), (size_t)smem, s);
      else if (variant == TANS_RANS32) ok = launch_push_fast<1>(P, use_alias != 0, bypass != 0, rsmem, blocks, (int)(warps * 32), (size_t)smem, s);
      else ok = launch_push_fast<2>(P, use_alias != 0, bypass != 0, rsmem, blocks, (int)(warps * 32), (size_t)smem, s);
      if (owned) cudaFreeAsync(ws, s);
      if (!ok) return TANS_E_INVALID_ARGUMENT;
      return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
    }
  }
  const LaunchShape L = pick_launch(batch, dev_sms);
  P.lanes = L.lanes;
  P.tin_smem = (ntables <= kTinfoSmemMax &&
                (size_t)L.threads * push_smem_per_thread(use_alias != 0, bypass != 0) + (size_t)ntables * sizeof(TableInfo) <=
                    200 * 1024)
                   ? 1
                   : 0;
  if (variant == TANS_RANS64) launch_push_v<0>(P, use_alias != 0, bypass != 0, interleave, L, s);
  else if (variant == TANS_RANS32) launch_push_v<1>(P, use_alias != 0, bypass != 0, interleave, L, s);
  else launch_push_v<2>(P, use_alias != 0, bypass != 0, interleave, L, s);
  if (owned) cudaFreeAsync(ws, s);
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}

}  // namespace tans

extern "C" size_t tans_push_workspace_size(int variant, int64_t num_tables, int64_t cdf_width) {
  // the entry stride depends on fp only through the 2^fp + 1 cap; size for the widest case
  return tans::push_workspace_bytes(variant, num_tables, cdf_width > 1 ? cdf_width - 1 : 0);
}

extern "C" int tans_push(int variant, int use_alias, int num_interleaves, int32_t* stream, int64_t batch,
                         int64_t stream_width, const int32_t* symbols, const int32_t* indexes, int64_t num_symbols,
                         const int32_t* cdfs, int64_t num_tables, int64_t cdf_width, const int32_t* cdf_sizes,
                         const int32_t* offsets, int freq_precision, int bypass_coding, int bypass_precision,
                         void* workspace, size_t workspace_bytes, uint32_t* dev_status, void* cuda_stream) {
  return tans::push_impl(variant, use_alias, num_interleaves, stream, batch, stream_width, symbols, indexes,
                         num_symbols, cdfs, num_tables, cdf_width, cdf_sizes, offsets, freq_precision, bypass_coding,
                         bypass_precision, workspace, workspace_bytes, dev_status,
                         reinterpret_cast<cudaStream_t>(cuda_stream), true);
}
