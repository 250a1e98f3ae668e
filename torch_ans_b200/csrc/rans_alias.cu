// rans_alias.cu -- alias-table build on the device (tans_alias_build_table).
//
// Replaces rans_alias_build_table (torch_ans/rans.cpp:56-95) with build_alias_mapping
// (torch_ans/rans_utils.hpp:537-651) for tables that already live on the GPU.  One block per
// table: the block copies the cdf prefix into both output rows and zero-fills the rest; thread 0
// then runs the two inherently sequential passes (Vose-style pairing of the 2^symbol_precision
// cuts, then the alias offsets, whose running "used" counts depend on every earlier cut) in the
// reference's order, writing the same entries in the same order as the host builder (so a table
// that fails midway leaves the same partial rows); finally the whole block fills the remap row
// over all 2^fp cum values.  Two cum values mapping to one remap slot would leave the last one
// (the largest cum) in the sequential builder; atomicMax keeps exactly that one here.
#include <cuda_runtime.h>

#include <algorithm>

#include "../../include/torch_ans_b200.h"
#include "launch.cuh"
#include "rans_host.h"

namespace tans {

__global__ void alias_build_kernel(const int32_t* cdfs, int64_t ntables, int64_t cdf_width, const int32_t* sizes,
                                   int sp, int fp, int32_t* remap, int64_t rw, int32_t* table, int64_t tw,
                                   int32_t* scratch) {
  const int64_t k = blockIdx.x;
  if (k >= ntables) return;
  const int T = blockDim.x, tid = threadIdx.x;
  const int32_t* cdf = cdfs + k * cdf_width;
  int32_t* rrow = remap + k * rw;
  int32_t* trow = table + k * tw;
  const int32_t n = sizes[k];
  const int64_t nc = n < 0 ? 0 : ((int64_t)n < cdf_width ? (int64_t)n : cdf_width);  // cdf entries the rows start with
  for (int64_t i = tid; i < rw; i += T) rrow[i] = i < nc ? cdf[i] : 0;
  for (int64_t i = tid; i < tw; i += T) trow[i] = i < nc ? cdf[i] : 0;
  __syncthreads();
  __shared__ int ok;
  if (tid == 0) {
    ok = 0;
    const int32_t nsym = n - 1;
    const int32_t total_range = 1 << fp;
    const int32_t ncuts = 1 << sp;
    int32_t* tab = trow + nc;
    int32_t* rem = rrow + nc;
    const int64_t tab_cap = (tw - nc) / 4, remap_cap = rw - nc;
    int32_t* order = scratch + k * 3 * (int64_t)ncuts;
    int32_t* mass = order + ncuts;
    int32_t* used = mass + ncuts;
    (void)rem;
    bool good = nsym > 0 && n <= cdf_width;
    const int32_t cut = good ? total_range / nsym : 0;
    good = good && (int64_t)ncuts * cut == total_range && ncuts >= nsym && ncuts <= tab_cap &&
           total_range <= remap_cap;
    int small_end = 0, large_begin = ncuts;
    if (good) {
      int64_t sum = 0;
      for (int i = 0; i < ncuts; ++i) {
        mass[i] = i < nsym ? cdf[i + 1] - cdf[i] : 0;
        used[i] = 0;
        sum += mass[i];
        if (mass[i] >= cut) order[--large_begin] = i;
        else order[small_end++] = i;
      }
      good = sum == total_range;
    }
    // element layout: {cut_cdf, other_symbol, self_alias_offset, other_alias_offset}
    while (good && small_end > 0) {
      if (large_begin >= ncuts) {
        good = false;
        break;
      }
      const int sm = order[--small_end];
      const int lg = order[large_begin++];
      const int32_t cc = mass[sm] + sm * cut;
      tab[4 * sm] = cc >= total_range ? total_range : cc;
      tab[4 * sm + 1] = lg;
      mass[lg] -= cut - mass[sm];
      if (mass[lg] >= cut) --large_begin;
      else order[small_end++] = lg;
      if (large_begin == ncuts) good = false;
    }
    if (good) {
      while (large_begin < ncuts) {
        const int lg = order[large_begin++];
        tab[4 * lg + 1] = lg;
        const int32_t cc = cut + lg * cut;
        tab[4 * lg] = cc >= total_range ? total_range : cc;
      }
      for (int s = 0; s < ncuts && (int64_t)s * cut < total_range; ++s) {
        const int other = tab[4 * s + 1];
        const int32_t cc = tab[4 * s];
        const int32_t own = cc - s * cut;
        const int32_t lent = ((int64_t)(s + 1) * cut >= total_range) ? (total_range - cc) : (cut - own);
        tab[4 * s + 2] = s * cut - used[s];
        tab[4 * s + 3] = s * cut + own - used[other];
        used[s] += own;
        used[other] += lent;
      }
      ok = cut;
    }
  }
  __syncthreads();
  const int32_t cut = ok;
  if (cut == 0) return;
  const int32_t total_range = 1 << fp;
  const int32_t* tab = trow + nc;
  int32_t* rem = rrow + nc;
  const int64_t remap_cap = rw - nc;
  for (int32_t r = tid; r < total_range; r += T) {
    const int32_t id = r / cut;
    const bool hi = r >= tab[4 * id];
    const int32_t sidx = hi ? tab[4 * id + 1] : id;
    const int32_t a0 = hi ? tab[4 * id + 3] : tab[4 * id + 2];
    const int64_t at = (int64_t)r - a0 + ((sidx >= 0 && sidx < cdf_width) ? cdf[sidx] : 0);
    if (at >= 0 && at < remap_cap) atomicMax(rem + at, r);
  }
}

}  // namespace tans

extern "C" size_t tans_alias_workspace_size(int64_t num_tables, int symbol_precision) {
  if (num_tables <= 0 || symbol_precision < 0 || symbol_precision > 24) return 0;
  return tans::align_up((size_t)num_tables * 3 * ((size_t)1 << symbol_precision) * sizeof(int32_t));
}

extern "C" int tans_alias_build_table(const int32_t* cdfs, int64_t num_tables, int64_t cdf_width,
                                      const int32_t* cdf_sizes, int symbol_precision, int freq_precision,
                                      int32_t* remap_out, int32_t* table_out, void* workspace, size_t workspace_bytes,
                                      void* cuda_stream) {
  if (num_tables < 0 || cdf_width < 0 || symbol_precision < 0 || symbol_precision > 24 || freq_precision < 1 ||
      freq_precision > 31)
    return TANS_E_INVALID_ARGUMENT;
  if (num_tables == 0) return TANS_OK;
  if (!cdfs || !cdf_sizes || !remap_out || !table_out) return TANS_E_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(cuda_stream);
  const size_t need = tans_alias_workspace_size(num_tables, symbol_precision);
  void* ws = workspace;
  bool owned = false;
  if (!ws) {
    if (cudaMallocAsync(&ws, need, s) != cudaSuccess) return TANS_E_CUDA;
    owned = true;
  } else if (workspace_bytes < need) {
    return TANS_E_WORKSPACE;
  }
  const int64_t rw = cdf_width + ((int64_t)1 << freq_precision), tw = cdf_width * 5;
  tans::alias_build_kernel<<<(unsigned)num_tables, 256, 0, s>>>(cdfs, num_tables, cdf_width, cdf_sizes,
                                                                 symbol_precision, freq_precision, remap_out, rw,
                                                                 table_out, tw, reinterpret_cast<int32_t*>(ws));
  tans::note_launch();
  if (owned) cudaFreeAsync(ws, s);
  return cudaGetLastError() == cudaSuccess ? TANS_OK : TANS_E_CUDA;
}
