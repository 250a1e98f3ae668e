/*
 * torch_ans_b200.h -- C ABI of the B200 rANS coding engine (libtorch_ans_b200.so).
 *
 * Every entry point takes plain device pointers, element counts and a CUDA stream handle
 * (cudaStream_t passed as void*; NULL = the legacy default stream).  No torch types cross this
 * boundary.  All coding calls are asynchronous on the given stream; nothing here synchronises the
 * device unless its comment says so.  All tensors are int32, row-major and densely packed.
 *
 * Stream rows use the reference's layout (torch_ans/rans_cpu.cpp:81-84,181): an int32 matrix of
 * shape (batch, stream_width); row[0] holds the payload length in bytes, row[1..] the payload:
 * the coder state(s) little-endian, then the emitted words appended upward.
 *
 * Return value of every int function: TANS_OK (0) or one of the TANS_E_* codes.  Problems that
 * can only be seen on the device (an index outside the table list, a symbol outside its table
 * without escape coding, a zero frequency, a row that is too short) never cause an out-of-bounds
 * access: the kernel skips that step and ORs a TANS_DEV_* bit into *dev_status (when non-NULL).
 */
#ifndef TORCH_ANS_B200_H
#define TORCH_ANS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Coder variants: (state bits, word bits).  The three template instantiations bound at
 * torch_ans/rans.hpp:297-322 (rans64 = <uint64_t,uint32_t>, rans32 = <uint32_t,uint8_t>,
 * rans32_16 = <uint32_t,uint16_t>). */
#define TANS_RANS64 0
#define TANS_RANS32 1
#define TANS_RANS32_16 2

/* Symbol lookup used by pop (torch_ans/rans_utils.hpp:412-450): bisection on the cdf row,
 * inverse-cdf table at row + cdf_size, or alias table at row + cdf_size. */
#define TANS_LOOKUP_SEARCH 0
#define TANS_LOOKUP_INVCDF 1
#define TANS_LOOKUP_ALIAS 2

/* Host-visible return codes. */
#define TANS_OK 0
#define TANS_E_INVALID_ARGUMENT 1
#define TANS_E_CUDA 2
#define TANS_E_WORKSPACE 3
#define TANS_E_TOO_LARGE 4

/* Device-side error bits (ORed into *dev_status). */
#define TANS_DEV_BAD_INDEX 1u
#define TANS_DEV_BAD_VALUE 2u
#define TANS_DEV_OVERFLOW 4u
#define TANS_DEV_UNDERFLOW 8u
#define TANS_DEV_BAD_FREQ 16u
#define TANS_DEV_BAD_ESCAPE 32u
/* A kernel whose warps hand work to one another gave up waiting (every such wait is bounded);
 * the rows of that call are not valid.  Not expected in normal operation. */
#define TANS_DEV_STALLED 64u

/* Library version, (major << 16) | (minor << 8) | patch. */
int tans_version(void);

/* Human-readable name of a return code. */
const char* tans_status_string(int code);

/* Number of kernels this library has launched in this process so far (all devices and streams).
 * A diagnostic with no counterpart in the reference: benchmarks read it around a timed region to
 * report how many of the library's kernels ran in it. */
uint64_t tans_launch_count(void);

/* Latency probes behind the kernel design: cycles of one dependent step, measured with clock64 on
 * the device (no counterpart in the reference; a diagnostic that allocates, runs one kernel and
 * synchronises).  kind:
 *   TANS_PROBE_SMEM_CHASE    dependent loads around a random cycle in 48 KB of shared memory
 *   TANS_PROBE_L2_CHASE      dependent 8-byte loads around a random cycle in an 8 MB buffer held in
 *                            L2 (the bucket table's size), one thread
 *   TANS_PROBE_L2_CHASE_BUSY the same with 56 chasing lanes per SM on every SM (14 warps x 4 lanes)
 *   TANS_PROBE_POP32_STEP / TANS_PROBE_PUSH32_STEP / TANS_PROBE_POP64_STEP / TANS_PROBE_PUSH64_STEP
 *                            the dependent instructions of one rans32 / rans64 pop or push step
 *                            (16-bit precision, table entry in shared memory, words in registers,
 *                            renormalising every step), one thread: the floor under a kernel that
 *                            codes one stream per SM.
 * *cycles_per_step receives the mean over the probe's chains. */
#define TANS_PROBE_SMEM_CHASE 0
#define TANS_PROBE_L2_CHASE 1
#define TANS_PROBE_L2_CHASE_BUSY 2
#define TANS_PROBE_POP32_STEP 3
#define TANS_PROBE_PUSH32_STEP 4
#define TANS_PROBE_POP64_STEP 5
#define TANS_PROBE_PUSH64_STEP 6
int tans_probe(int kind, int64_t steps, double* cycles_per_step);

/* Bytes of device scratch that tans_push needs for a table list of num_tables rows of cdf_width
 * entries (a per-entry reciprocal table plus per-table size/offset pairs). */
size_t tans_push_workspace_size(int variant, int64_t num_tables, int64_t cdf_width);

/* Encode: push num_symbols symbols per stream row onto `stream`, last symbol first.
 * Replaces the reference's rans_push<State, Word, USE_ALIAS, I> (torch_ans/rans.hpp:84-217) after
 * its resize step, i.e. rans_push_indexed_cpu (torch_ans/rans_cpu.cpp:44-189) /
 * rans_push_indexed_cuda (torch_ans/rans_cuda.cu:115-167).
 *   stream      [batch, stream_width] int32, updated in place (length, state, appended words);
 *               the caller sizes stream_width for the worst case, as rans.hpp:105-124 does.
 *   symbols     [batch, num_symbols], indexes [batch, num_symbols]: table index per symbol.
 *   cdfs        [num_tables, cdf_width]: quantised cdf rows (with use_alias: the remap rows made
 *               by rans_alias_build_table, remap at row + cdf_size).
 *   cdf_sizes   [num_tables], offsets [num_tables] (offsets may be NULL = all zero).
 *   num_interleaves 1, or 4 for the 4-state format of the *_i4 ops (rans_cpu.cpp:89-160).
 *   workspace   device scratch of tans_push_workspace_size() bytes, 256-byte aligned; NULL makes
 *               the call allocate and free it stream-ordered (cudaMallocAsync / cudaFreeAsync).
 *   dev_status  device uint32 receiving TANS_DEV_* bits, or NULL. */
int tans_push(int variant, int use_alias, int num_interleaves,
              int32_t* stream, int64_t batch, int64_t stream_width,
              const int32_t* symbols, const int32_t* indexes, int64_t num_symbols,
              const int32_t* cdfs, int64_t num_tables, int64_t cdf_width,
              const int32_t* cdf_sizes, const int32_t* offsets,
              int freq_precision, int bypass_coding, int bypass_precision,
              void* workspace, size_t workspace_bytes, uint32_t* dev_status, void* cuda_stream);

/* tans_push without any device allocation, for callers that cannot allocate device memory
 * (hosts whose memory is owned by another allocator or budget, plugins that may only use the
 * buffers they are handed, serving loops that must not allocate after start-up).  This entry
 * point has no counterpart in the reference.  Arguments and results are those of tans_push; the
 * encode-table scratch comes from a fixed 8 MiB array inside the library (held on every GPU that
 * loads it until the process exits).  The scratch a table list needs is 16 bytes per table plus
 * 16 bytes per table entry, with min(cdf_width - 1, 2^freq_precision + 1) entries per table, each
 * part rounded up to 256 bytes (tans_push_workspace_size gives the same figure while
 * cdf_width <= 2^freq_precision + 2); it must be at most 8 MiB (about 524,000 table entries), else
 * TANS_E_TOO_LARGE is returned and nothing runs.  Invalid arguments are reported first, with the
 * codes tans_push returns.  The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress); make that first call before any stream
 * capture.  All calls share the array: calls whose GPU work may overlap (different streams,
 * unordered threads) must be serialised by the caller. */
int tans_push_noalloc(int variant, int use_alias, int num_interleaves,
                      int32_t* stream, int64_t batch, int64_t stream_width,
                      const int32_t* symbols, const int32_t* indexes, int64_t num_symbols,
                      const int32_t* cdfs, int64_t num_tables, int64_t cdf_width,
                      const int32_t* cdf_sizes, const int32_t* offsets,
                      int freq_precision, int bypass_coding, int bypass_precision,
                      uint32_t* dev_status, void* cuda_stream);

/* Bytes of device scratch that tans_pop needs (per-table size/offset pairs and, for the lookup
 * tables it builds, their device copies). */
size_t tans_pop_workspace_size(int variant, int lookup, int64_t num_tables, int64_t cdf_width,
                               int freq_precision);

/* Decode: pop num_symbols symbols per stream row, first symbol first, writing them to
 * out_symbols [batch, num_symbols] and updating each row's length and state in place.
 * Replaces rans_pop<State, Word, USE_ALIAS, USE_INVCDF, I> (torch_ans/rans.hpp:220-276), i.e.
 * rans_pop_indexed_cpu (torch_ans/rans_cpu.cpp:191-322) / rans_pop_indexed_cuda
 * (torch_ans/rans_cuda.cu:236-286).  With TANS_LOOKUP_ALIAS, cdfs are the table rows made by
 * rans_alias_build_table; with TANS_LOOKUP_INVCDF each row is [cdf | inverse cdf (2^fp)]. */
int tans_pop(int variant, int lookup, int num_interleaves,
             int32_t* stream, int64_t batch, int64_t stream_width,
             int32_t* out_symbols, const int32_t* indexes, int64_t num_symbols,
             const int32_t* cdfs, int64_t num_tables, int64_t cdf_width,
             const int32_t* cdf_sizes, const int32_t* offsets,
             int freq_precision, int bypass_coding, int bypass_precision,
             void* workspace, size_t workspace_bytes, uint32_t* dev_status, void* cuda_stream);

/* Ragged coding.  No single reference function corresponds: the reference codes rectangular
 * (batch, N) tensors only, so streams of different lengths -- typically with one table row per
 * symbol, the per-element pattern of TorchANSInterface.encode_with_freqs (torch_ans/utils.py:
 * 704-760) -- take one rans_push / rans_pop call per stream (B = 1, indexes arange(n_b), tables =
 * that stream's rows).  Here stream row b codes symbols [row_starts[b], row_starts[b+1]) of the
 * flat arrays, symbol i with table indexes[i] (indexes NULL: table i), and ends up with exactly
 * the bytes of that per-stream call (rans_push_indexed_cpu / rans_pop_indexed_cpu,
 * torch_ans/rans_cpu.cpp:44-322, single state).  row_starts: device int64[batch + 1]; a row whose
 * range is invalid is skipped and flags TANS_DEV_BAD_VALUE.  Pop uses the bisection lookup only.
 *   workspace: tans_push_ragged_workspace_size(total_symbols) bytes, or NULL to allocate it
 *   stream-ordered. */
size_t tans_push_ragged_workspace_size(int64_t total_symbols);
int tans_push_ragged(int variant, int32_t* stream, int64_t batch, int64_t stream_width,
                     const int32_t* symbols, const int32_t* indexes, const int64_t* row_starts,
                     int64_t total_symbols, const int32_t* cdfs, int64_t num_tables, int64_t cdf_width,
                     const int32_t* cdf_sizes, const int32_t* offsets, int freq_precision, int bypass_coding,
                     int bypass_precision, void* workspace, size_t workspace_bytes, uint32_t* dev_status,
                     void* cuda_stream);
int tans_pop_ragged(int variant, int32_t* stream, int64_t batch, int64_t stream_width, int32_t* out_symbols,
                    const int32_t* indexes, const int64_t* row_starts, int64_t total_symbols,
                    const int32_t* cdfs, int64_t num_tables, int64_t cdf_width, const int32_t* cdf_sizes,
                    const int32_t* offsets, int freq_precision, int bypass_coding, int bypass_precision,
                    uint32_t* dev_status, void* cuda_stream);

/* Alias tables on the device: rans_alias_build_table (torch_ans/rans.cpp:56-95, build_alias_mapping
 * torch_ans/rans_utils.hpp:537-651) for cdf rows already on the GPU.  remap_out [num_tables,
 * cdf_width + 2^freq_precision] and table_out [num_tables, 5 cdf_width] are written whole (cdf
 * prefix, then the remap / alias elements, zeros elsewhere), exactly as the reference builds them,
 * including the rows it leaves unbuilt when its power-of-two cut condition fails.  workspace:
 * tans_alias_workspace_size() bytes or NULL (allocated stream-ordered). */
size_t tans_alias_workspace_size(int64_t num_tables, int symbol_precision);
int tans_alias_build_table(const int32_t* cdfs, int64_t num_tables, int64_t cdf_width, const int32_t* cdf_sizes,
                           int symbol_precision, int freq_precision, int32_t* remap_out, int32_t* table_out,
                           void* workspace, size_t workspace_bytes, void* cuda_stream);

/* Maximum of column 0 (payload length) over the batch rows, written to *out_max (device int32).
 * The device half of the worst-case resize at torch_ans/rans.hpp:105-107. */
int tans_stream_max_length(const int32_t* stream, int64_t batch, int64_t stream_width,
                           int32_t* out_max, void* cuda_stream);

/* Fill `stream` [batch, stream_width] as a fresh stream: row[0] = num_interleaves*state bytes,
 * each state = the lower bound, zeros elsewhere.  Device version of rans_init_stream
 * (torch_ans/rans_cpu.cpp:22-41). */
int tans_init_stream(int variant, int num_interleaves, int32_t* stream, int64_t batch,
                     int64_t stream_width, void* cuda_stream);

/* Concatenated-bitstream assembly, the device form of rans_stream_to_byte_strings followed by
 * merge_bytes (torch_ans/rans.cpp:5-21, torch_ans/utils.py:47-72).  Given the exclusive byte
 * offsets of each row's record in `out` (record = optional little-endian length prefix of
 * prefix_bytes (0, 1, 2, 4 or 8) followed by the row's payload[0:len]), writes all records.
 * `prefix_rows` says how many leading rows get a prefix (rows >= prefix_rows get none). */
int tans_gather_payloads(const int32_t* stream, int64_t batch, int64_t stream_width,
                         const int64_t* record_offsets, int prefix_bytes, int64_t prefix_rows,
                         uint8_t* out, void* cuda_stream);

/* Inverse of tans_gather_payloads: rows of `stream` [batch, stream_width] are zeroed and filled
 * with payload bytes taken from `in` at payload_offsets[b] (lengths[b] bytes each), row[0] set to
 * lengths[b].  Device form of rans_byte_strings_to_stream (torch_ans/rans.cpp:23-53). */
int tans_scatter_payloads(const uint8_t* in, const int64_t* payload_offsets,
                          const int32_t* lengths, int32_t* stream, int64_t batch,
                          int64_t stream_width, void* cuda_stream);

/* Zero-frequency repair of quantised cdf rows (the per-row loop of
 * rans_pmf_to_quantized_cdf_cpu, torch_ans/rans_cpu.cpp:351-379): for every symbol whose
 * frequency is 0, borrow one count from the first symbol holding the smallest frequency > 1.
 * cdfs [rows, n + 1] updated in place; rows with nothing to borrow set TANS_DEV_BAD_FREQ. */
int tans_cdf_fix_zero_freqs(int32_t* cdfs, int64_t rows, int64_t n, uint32_t* dev_status,
                            void* cuda_stream);

#ifdef __cplusplus
}
#endif

#endif /* TORCH_ANS_B200_H */
