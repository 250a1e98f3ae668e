/*
 * oracle/rans_oracle.c -- CPU restatement of torch_ans's rANS coding path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle that the CUDA path of torch_ans_b200 is
 * compared against; nothing in the product imports, links or executes it.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it (through oracle/oracle.py).
 *
 * It restates, in plain C, the per-stream loops and step arithmetic of the reference CPU backend:
 *   - constants / renorm macros          torch_ans/rans_utils.hpp:32-71
 *   - escape ("bypass") value push       torch_ans/rans_utils.hpp:106-164
 *   - symbol push  x = C(s, x)           torch_ans/rans_utils.hpp:168-323
 *   - escape value pop                   torch_ans/rans_utils.hpp:327-375
 *   - symbol pop   s, x = D(x)           torch_ans/rans_utils.hpp:379-532
 *   - alias table construction           torch_ans/rans_utils.hpp:537-651, torch_ans/rans.cpp:56-95
 *   - per-stream push loop (1 / 4 states) torch_ans/rans_cpu.cpp:79-182
 *   - per-stream pop loop (1 / 4 states)  torch_ans/rans_cpu.cpp:221-316
 *   - stream initialisation              torch_ans/rans_cpu.cpp:22-41
 *
 * The three coder variants differ only in state width and word width:
 *   rans64    : 64-bit state, 32-bit words (rans.hpp:297-301)
 *   rans32    : 32-bit state,  8-bit words (rans.hpp:305-313)
 *   rans32_16 : 32-bit state, 16-bit words (rans.hpp:314-322)
 * One generic implementation carries the state in a uint64_t and reduces it modulo 2^state_bits
 * after every operation that would wrap in the reference's native type, so the arithmetic is the
 * same as the reference's uint32_t / uint64_t templates (including C's conversions of the signed
 * int32 table values to the unsigned state type).
 *
 * Where the reference has undefined behaviour on invalid input (table index out of range, symbol
 * outside the table without escape coding, zero frequency, reading below the start of a stream,
 * writing past the end of the row), this restatement does not read or write out of bounds: it
 * skips the step and sets an error bit (the same bits the CUDA kernels report), so both sides can
 * be compared on such inputs too.  On valid input it matches the reference byte for byte.
 *
 * Stream row layout (an int32 tensor of shape (B, W)), rans_cpu.cpp:81-84,181:
 *   row[0]            payload length in bytes
 *   row[1..]          payload: I little-endian states, then words appended upward.
 */
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#define ORC_ERR_BAD_INDEX 1u   /* table index outside [0, num_tables) */
#define ORC_ERR_BAD_VALUE 2u   /* symbol outside the table and no escape coding */
#define ORC_ERR_OVERFLOW 4u    /* push would write past the row */
#define ORC_ERR_UNDERFLOW 8u   /* pop would read below the first data word */
#define ORC_ERR_BAD_FREQ 16u   /* zero (or negative) frequency met on the coding path */
#define ORC_ERR_BAD_ESCAPE 32u /* escape value longer than 32 bits */

typedef struct {
  int32_t cut_cdf;
  int32_t other_symbol;
  int32_t self_alias_offset;
  int32_t other_alias_offset;
} orc_alias_elem; /* rans_utils.hpp:75-82 */

typedef struct {
  int state_bits, word_bits, word_bytes, state_bytes;
  uint64_t state_mask, word_mask;
  uint64_t lower_bound; /* RANS_STATE_LOWER_BOUND = 1 << (state_bits - 1 - word_bits) */
  int renorm_while;     /* (USED - WB) >= WB selects the `while` renorm (rans_utils.hpp:45-61) */
} orc_variant;

static orc_variant orc_make_variant(int variant) {
  orc_variant v;
  if (variant == 0) { v.state_bits = 64; v.word_bits = 32; }
  else if (variant == 1) { v.state_bits = 32; v.word_bits = 8; }
  else { v.state_bits = 32; v.word_bits = 16; }
  v.word_bytes = v.word_bits / 8;
  v.state_bytes = v.state_bits / 8;
  v.state_mask = v.state_bits == 64 ? ~0ull : ((1ull << v.state_bits) - 1);
  v.word_mask = (1ull << v.word_bits) - 1;
  v.lower_bound = 1ull << (v.state_bits - 1 - v.word_bits);
  v.renorm_while = (v.state_bits - 1 - v.word_bits) >= v.word_bits;
  return v;
}

/* C conversion of a signed int32 to the state type: sign extension to 64 bits, then reduction. */
static inline uint64_t orc_to_state(const orc_variant* v, int32_t a) {
  return ((uint64_t)(int64_t)a) & v->state_mask;
}

typedef struct {
  const orc_variant* v;
  uint8_t* payload;   /* row + 1 */
  int64_t p;          /* word index of the last written word (the reference's stream_ptr) */
  int64_t cap_words;  /* words that fit in the row's payload */
  int64_t first_word; /* first word index after the state slots */
  uint32_t err;
  int last_ok;        /* whether the last orc_pop_step decoded a symbol (0 when it was skipped) */
} orc_cursor;

static inline uint64_t orc_read_word(const orc_cursor* c, int64_t j) {
  uint64_t w = 0;
  memcpy(&w, c->payload + j * c->v->word_bytes, (size_t)c->v->word_bytes); /* little endian */
  return w;
}

static inline void orc_write_word(orc_cursor* c, int64_t j, uint64_t w) {
  memcpy(c->payload + j * c->v->word_bytes, &w, (size_t)c->v->word_bytes);
}

/* APPEND_STATE_TO_STREAM, rans_utils.hpp:40-41 */
static inline void orc_emit(orc_cursor* c, uint64_t* x) {
  c->p += 1;
  if (c->p < c->cap_words) orc_write_word(c, c->p, *x & c->v->word_mask);
  else c->err |= ORC_ERR_OVERFLOW;
  *x >>= c->v->word_bits;
}

/* POP_STATE_FROM_STREAM inside RANS_POP_STATE_RENORM, rans_utils.hpp:42-43,57-61 */
static inline void orc_pop_renorm(orc_cursor* c, uint64_t* x) {
  while (*x < c->v->lower_bound) {
    uint64_t w = 0;
    if (c->p >= c->first_word) w = orc_read_word(c, c->p);
    else c->err |= ORC_ERR_UNDERFLOW;
    *x = ((*x << c->v->word_bits) | w) & c->v->state_mask;
    c->p -= 1;
    if (!c->v->renorm_while) break;
  }
}

/* RANS_APPEND_BITS, rans_utils.hpp:63-68 */
static inline void orc_append_bits(orc_cursor* c, uint64_t* x, int32_t value, int nbits) {
  const uint64_t bound = (c->v->lower_bound >> nbits) << c->v->word_bits;
  while (*x >= bound) {
    orc_emit(c, x);
    if (!c->v->renorm_while) break;
  }
  *x = ((*x << nbits) | orc_to_state(c->v, value)) & c->v->state_mask;
}

/* int32 right shift that is defined for counts >= 32 (the reference only reaches those for
 * escape values >= 2^28 at precision 4, where its own loop is undefined). */
static inline int32_t orc_shr(int32_t a, int64_t n) { return n >= 32 ? (a < 0 ? -1 : 0) : (a >> n); }

/* rans_push_raw_value_step, rans_utils.hpp:106-164 */
static void orc_push_raw(orc_cursor* c, uint64_t* xs, int32_t raw, int bp) {
  const int32_t maxb = (int32_t)((1u << bp) - 1);
  int32_t nb = 0;
  while (orc_shr(raw, (int64_t)nb * bp) != 0) ++nb;
  int32_t val = nb, ncodes = 0;
  while (val >= maxb) { ncodes += 1; val -= maxb; }
  uint64_t x = *xs;
  for (int64_t j = nb - 1; j >= 0; j--) orc_append_bits(c, &x, orc_shr(raw, j * bp) & maxb, bp);
  orc_append_bits(c, &x, val, bp);
  for (int64_t j = ncodes - 1; j >= 0; j--) orc_append_bits(c, &x, maxb, bp);
  *xs = x;
}

/* rans_push_step, rans_utils.hpp:168-323 (cdf != nullptr branch; the nullptr branch is not
 * reachable from the bound ops).  `remap` is the alias remap row or NULL. */
static void orc_push_step(orc_cursor* c, uint64_t* xs, int32_t symbol, const int32_t* cdf,
                          int32_t cdf_size, int32_t offset, int fp, int bypass, int bp,
                          const int32_t* remap) {
  const orc_variant* v = c->v;
  int32_t value = (int32_t)((uint32_t)symbol - (uint32_t)offset);
  const int32_t maxv = cdf_size - 2;
  int32_t raw = 0;
  if (bypass) {
    if (value < 0) { raw = -2 * value - 1; value = maxv; }
    else if (value >= maxv) { raw = 2 * (value - maxv); value = maxv; }
  }
  if (value < 0 || value >= cdf_size - 1) { c->err |= ORC_ERR_BAD_VALUE; return; }
  if (bypass && value == maxv) orc_push_raw(c, xs, raw, bp);
  const int32_t start = cdf[value];
  const int32_t freq = cdf[value + 1] - start;
  if (freq <= 0) { c->err |= ORC_ERR_BAD_FREQ; return; }
  uint64_t x = *xs;
  const uint64_t bound = ((v->lower_bound >> fp) << v->word_bits) * (uint64_t)(int64_t)freq;
  while (x >= bound) {
    orc_emit(c, &x);
    if (!v->renorm_while) break;
  }
  const uint64_t f = orc_to_state(v, freq);
  const uint64_t q = x / f, r = x % f;
  if (remap) {
    const uint64_t ri = (r + orc_to_state(v, start)) & v->state_mask;
    x = ((q << fp) + orc_to_state(v, remap[ri])) & v->state_mask;
  } else {
    x = ((q << fp) + r + orc_to_state(v, start)) & v->state_mask;
  }
  *xs = x;
}

/* rans_pop_raw_value_step, rans_utils.hpp:327-375 */
static int32_t orc_pop_raw(orc_cursor* c, uint64_t* xs, int bp) {
  const int32_t maxb = (int32_t)((1u << bp) - 1);
  uint64_t x = *xs;
  int32_t val = (int32_t)(x & (uint64_t)((1u << bp) - 1));
  x >>= bp;
  orc_pop_renorm(c, &x);
  int32_t n = val;
  /* a valid escape has at most 32 chunks; longer counts only come from corrupt streams */
  while (val == maxb && n <= 32) {
    val = (int32_t)(x & (uint64_t)((1u << bp) - 1));
    x >>= bp;
    orc_pop_renorm(c, &x);
    n += val;
  }
  int32_t raw = 0;
  if (n > 32) { c->err |= ORC_ERR_BAD_ESCAPE; n = 0; }
  for (int j = 0; j < n; ++j) {
    val = (int32_t)(x & (uint64_t)((1u << bp) - 1));
    x >>= bp;
    orc_pop_renorm(c, &x);
    if (j * bp < 32) raw |= (int32_t)((uint32_t)val << (j * bp));
  }
  *xs = x;
  return raw;
}

/* rans_pop_step, rans_utils.hpp:379-532.  lookup: 0 = bisection on the cdf, 1 = inverse cdf
 * table at cdf_row + cdf_size, 2 = alias table at cdf_row + cdf_size. */
static int32_t orc_pop_step(orc_cursor* c, uint64_t* xs, const int32_t* cdf, int32_t cdf_size,
                            int32_t offset, int fp, int bypass, int bp, int lookup) {
  const orc_variant* v = c->v;
  const int32_t maxv = cdf_size - 2;
  c->last_ok = 0;
  uint64_t x = *xs;
  const int32_t cum = (int32_t)(x & ((1ull << fp) - 1));
  int64_t s;
  int32_t cum_off = cum;
  if (lookup == 2) {
    const orc_alias_elem* tab = (const orc_alias_elem*)(cdf + cdf_size);
    const int32_t cut = (int32_t)((1 << fp) / (cdf_size - 1));
    const int32_t id = cum / cut;
    const int32_t cut_cdf = tab[id].cut_cdf;
    s = (cum >= cut_cdf) ? tab[id].other_symbol : id;
    cum_off -= (cum >= cut_cdf) ? tab[id].other_alias_offset : tab[id].self_alias_offset;
  } else if (lookup == 1) {
    s = cdf[cdf_size + cum];
    if (s < 0 || s >= cdf_size - 1) { c->err |= ORC_ERR_BAD_VALUE; return 0; }
    cum_off -= cdf[s];
  } else {
    /* rans_utils.hpp:427-449: probe (cdf_size*cum)>>fp, then bisection over [0, cdf_size-1] */
    uint64_t idx = (uint64_t)(int64_t)((int32_t)((uint32_t)cdf_size * (uint32_t)cum) >> fp);
    idx &= v->state_mask;
    uint32_t low = 0, high = (uint32_t)(cdf_size - 1);
    while (high > low) {
      if (idx >= (uint64_t)cdf_size) { c->err |= ORC_ERR_BAD_VALUE; return 0; }
      if (cum >= cdf[idx]) low = (uint32_t)idx + 1;
      else high = (uint32_t)idx;
      idx = (low + high) / 2;
    }
    s = (int64_t)((idx - 1) & v->state_mask);
    if (s < 0 || s >= cdf_size - 1) { c->err |= ORC_ERR_BAD_VALUE; return 0; }
    cum_off -= cdf[s];
  }
  if (s < 0 || s >= cdf_size - 1) { c->err |= ORC_ERR_BAD_VALUE; return 0; }
  int32_t value = (int32_t)s;
  const int32_t freq = cdf[s + 1] - cdf[s];
  x = (((x >> fp) * orc_to_state(v, freq)) + orc_to_state(v, cum_off)) & v->state_mask;
  orc_pop_renorm(c, &x);
  *xs = x;
  c->last_ok = 1;
  if (bypass && value == maxv) {
    const int32_t raw = orc_pop_raw(c, xs, bp);
    value = raw >> 1;
    if (raw & 1) value = -value - 1;
    else value += maxv;
  }
  return (int32_t)((uint32_t)value + (uint32_t)offset);
}

static inline uint64_t orc_load_state(const orc_cursor* c, int k) {
  uint64_t s = 0;
  memcpy(&s, c->payload + (size_t)k * c->v->state_bytes, (size_t)c->v->state_bytes);
  return s;
}

static inline void orc_store_state(orc_cursor* c, int k, uint64_t s) {
  memcpy(c->payload + (size_t)k * c->v->state_bytes, &s, (size_t)c->v->state_bytes);
}

typedef struct {
  const int32_t *cdfs, *sizes, *offsets;
  int64_t num_tables, cdf_width;
} orc_tables;

static inline int orc_table(const orc_tables* t, int32_t k, const int32_t** row, int32_t* size,
                            int32_t* off) {
  if (k < 0 || k >= t->num_tables) return 0;
  *row = t->cdfs + (int64_t)k * t->cdf_width;
  *size = t->sizes[k];
  *off = t->offsets[k];
  return 1;
}

/* rans_init_stream, rans_cpu.cpp:22-41 */
void orc_init_stream(int variant, int32_t* stream, int64_t batch, int64_t width, int interleave) {
  const orc_variant v = orc_make_variant(variant);
  memset(stream, 0, sizeof(int32_t) * (size_t)(batch * width));
  for (int64_t b = 0; b < batch; b++) {
    int32_t* row = stream + b * width;
    row[0] = v.state_bytes * interleave;
    for (int k = 0; k < interleave; k++)
      memcpy((uint8_t*)(row + 1) + (size_t)k * v.state_bytes, &v.lower_bound, (size_t)v.state_bytes);
  }
}

/* rans_push_indexed_cpu, rans_cpu.cpp:44-189.  Returns the OR of the per-stream error bits. */
uint32_t orc_push(int variant, int alias, int interleave, int32_t* stream, int64_t batch,
                  int64_t width, const int32_t* symbols, const int32_t* indexes, int64_t nsym,
                  const int32_t* cdfs, int64_t num_tables, int64_t cdf_width, const int32_t* sizes,
                  const int32_t* offsets, int fp, int bypass, int bp, int threads) {
  const orc_variant v = orc_make_variant(variant);
  const orc_tables t = {cdfs, sizes, offsets, num_tables, cdf_width};
  uint32_t err_all = 0;
  const int I = interleave;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads) reduction(| : err_all)
  for (int64_t b = 0; b < batch; b++) {
    int32_t* row = stream + b * width;
    orc_cursor c;
    c.v = &v;
    c.payload = (uint8_t*)(row + 1);
    c.p = row[0] / v.word_bytes - 1;
    c.cap_words = (width - 1) * 4 / v.word_bytes;
    c.first_word = (int64_t)I * v.state_bytes / v.word_bytes;
    c.err = 0;
    uint64_t st[4];
    for (int k = 0; k < I; k++) st[k] = orc_load_state(&c, k);
    const int32_t* sym = symbols + b * nsym;
    const int32_t* idx = indexes + b * nsym;
    const int64_t first = nsym % I;
    int64_t i = nsym - 1;
    for (; i >= nsym - first; i--) { /* rans_cpu.cpp:89-104 */
      const int32_t* row_c; int32_t sz, off;
      if (!orc_table(&t, idx[i], &row_c, &sz, &off)) { c.err |= ORC_ERR_BAD_INDEX; continue; }
      orc_push_step(&c, &st[i % I], sym[i], row_c, sz, off, fp, bypass, bp, alias ? row_c + sz : NULL);
    }
    for (; i >= 0; i -= I) {
      if (I == 1) { /* rans_cpu.cpp:162-175 */
        const int32_t* row_c; int32_t sz, off;
        if (!orc_table(&t, idx[i], &row_c, &sz, &off)) { c.err |= ORC_ERR_BAD_INDEX; continue; }
        orc_push_step(&c, &st[0], sym[i], row_c, sz, off, fp, bypass, bp, alias ? row_c + sz : NULL);
        continue;
      }
      /* rans_cpu.cpp:108-160: escapes of the block first (j = 0..3 -> state 3-j), then symbols */
      int32_t vals[4];
      int ok[4];
      for (int j = 0; j < I; j++) {
        const int32_t* row_c; int32_t sz, off;
        ok[j] = orc_table(&t, idx[i - j], &row_c, &sz, &off);
        if (!ok[j]) { c.err |= ORC_ERR_BAD_INDEX; continue; }
        if (bypass) {
          const int32_t maxv = sz - 2;
          int32_t value = (int32_t)((uint32_t)sym[i - j] - (uint32_t)off);
          int32_t raw = 0;
          if (value < 0) { raw = -2 * value - 1; value = maxv; }
          else if (value >= maxv) { raw = 2 * (value - maxv); value = maxv; }
          vals[j] = value;
          if (value == maxv) orc_push_raw(&c, &st[I - 1 - j], raw, bp);
        }
      }
      for (int j = 0; j < I; j++) {
        if (!ok[j]) continue;
        const int32_t* row_c; int32_t sz, off;
        orc_table(&t, idx[i - j], &row_c, &sz, &off);
        if (bypass)
          orc_push_step(&c, &st[I - 1 - j], vals[j], row_c, sz, 0, fp, 0, bp, alias ? row_c + sz : NULL);
        else
          orc_push_step(&c, &st[I - 1 - j], sym[i - j], row_c, sz, off, fp, 0, bp, alias ? row_c + sz : NULL);
      }
    }
    for (int k = 0; k < I; k++) orc_store_state(&c, k, st[k]);
    row[0] = (int32_t)((c.p + 1) * v.word_bytes); /* rans_cpu.cpp:181 */
    err_all |= c.err;
  }
  return err_all;
}

/* rans_pop_indexed_cpu, rans_cpu.cpp:191-322.  lookup: 0 search, 1 inverse cdf, 2 alias. */
uint32_t orc_pop(int variant, int lookup, int interleave, int32_t* stream, int64_t batch,
                 int64_t width, int32_t* out, const int32_t* indexes, int64_t nsym,
                 const int32_t* cdfs, int64_t num_tables, int64_t cdf_width, const int32_t* sizes,
                 const int32_t* offsets, int fp, int bypass, int bp, int threads) {
  const orc_variant v = orc_make_variant(variant);
  const orc_tables t = {cdfs, sizes, offsets, num_tables, cdf_width};
  uint32_t err_all = 0;
  const int I = interleave;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads) reduction(| : err_all)
  for (int64_t b = 0; b < batch; b++) {
    int32_t* row = stream + b * width;
    orc_cursor c;
    c.v = &v;
    c.payload = (uint8_t*)(row + 1);
    c.p = row[0] / v.word_bytes - 1;
    c.cap_words = (width - 1) * 4 / v.word_bytes;
    c.first_word = (int64_t)I * v.state_bytes / v.word_bytes;
    c.err = 0;
    uint64_t st[4];
    for (int k = 0; k < I; k++) st[k] = orc_load_state(&c, k);
    const int32_t* idx = indexes + b * nsym;
    int32_t* o = out + b * nsym;
    const int64_t last = nsym - (I - 1);
    int64_t i = 0;
    for (; i < last; i += I) {
      if (I == 1) { /* rans_cpu.cpp:280-294 */
        const int32_t* row_c; int32_t sz, off;
        if (!orc_table(&t, idx[i], &row_c, &sz, &off)) { c.err |= ORC_ERR_BAD_INDEX; o[i] = 0; continue; }
        o[i] = orc_pop_step(&c, &st[0], row_c, sz, off, fp, bypass, bp, lookup);
        continue;
      }
      /* rans_cpu.cpp:236-278: four symbol pops (state j), then the escapes of the block */
      int okj[4];
      for (int j = 0; j < I; j++) {
        const int32_t* row_c; int32_t sz, off;
        okj[j] = 0;
        if (!orc_table(&t, idx[i + j], &row_c, &sz, &off)) { c.err |= ORC_ERR_BAD_INDEX; o[i + j] = 0; continue; }
        o[i + j] = orc_pop_step(&c, &st[j], row_c, sz, off, fp, 0, bp, lookup);
        okj[j] = c.last_ok;
      }
      if (bypass) {
        for (int j = 0; j < I; j++) {
          const int32_t* row_c; int32_t sz, off;
          if (!okj[j] || !orc_table(&t, idx[i + j], &row_c, &sz, &off)) continue;
          const int32_t maxv = sz - 2;
          int32_t value = (int32_t)((uint32_t)o[i + j] - (uint32_t)off);
          if (value == maxv) {
            const int32_t raw = orc_pop_raw(&c, &st[j], bp);
            value = raw >> 1;
            if (raw & 1) value = -value - 1;
            else value += maxv;
            o[i + j] = (int32_t)((uint32_t)value + (uint32_t)off);
          }
        }
      }
    }
    for (; i < nsym; i++) { /* rans_cpu.cpp:298-312 */
      const int32_t* row_c; int32_t sz, off;
      if (!orc_table(&t, idx[i], &row_c, &sz, &off)) { c.err |= ORC_ERR_BAD_INDEX; o[i] = 0; continue; }
      o[i] = orc_pop_step(&c, &st[i % I], row_c, sz, off, fp, bypass, bp, lookup);
    }
    for (int k = 0; k < I; k++) orc_store_state(&c, k, st[k]);
    row[0] = (int32_t)((c.p + 1) * v.word_bytes); /* rans_cpu.cpp:314 */
    err_all |= c.err;
  }
  return err_all;
}

/* build_alias_mapping, rans_utils.hpp:537-651 (one cdf row).  Returns 1 on success and 0 where
 * the reference returns false (it then leaves the zero-initialised rows untouched). */
static int orc_build_alias_row(const int32_t* cdf, int32_t cdf_size, orc_alias_elem* tab,
                               int32_t* remap, int sp, int fp, int64_t tab_cap, int64_t remap_cap) {
  const int32_t max_symbols = cdf_size - 1;
  const int32_t max_table = 1 << fp;
  if (max_symbols <= 0) return 0;
  const int32_t cut = max_table / max_symbols;
  const int32_t num_cuts = 1 << sp;
  if (num_cuts * cut != max_table) return 0;
  if (num_cuts < max_symbols || num_cuts * cut < max_table) return 0;
  if ((int64_t)num_cuts > tab_cap || (int64_t)max_table > remap_cap) return 0;
  int32_t* symbols = (int32_t*)malloc(sizeof(int32_t) * (size_t)num_cuts);
  int32_t* proba = (int32_t*)malloc(sizeof(int32_t) * (size_t)num_cuts);
  int32_t* cnt = (int32_t*)calloc((size_t)num_cuts, sizeof(int32_t));
  int ret = 1;
  int l = num_cuts, s = 0;
  int32_t total = 0;
  for (int i = 0; i < num_cuts; ++i) {
    proba[i] = (i < max_symbols) ? (cdf[i + 1] - cdf[i]) : 0;
    total += proba[i];
    if (proba[i] >= cut) symbols[--l] = i;
    else symbols[s++] = i;
  }
  if (total != max_table) { ret = 0; goto done; }
  while (s > 0) {
    if (l >= num_cuts) { ret = 0; goto done; }
    const int S = symbols[--s];
    const int L = symbols[l++];
    const int32_t cut_cdf = proba[S] + S * cut;
    tab[S].cut_cdf = (cut_cdf >= max_table) ? max_table : cut_cdf;
    tab[S].other_symbol = L;
    proba[L] -= cut - proba[S];
    if (proba[L] >= cut) --l;
    else symbols[s++] = L;
    if (l == num_cuts) { ret = 0; goto done; }
  }
  while (l < num_cuts) {
    const int L = symbols[l++];
    tab[L].other_symbol = L;
    const int32_t cut_cdf = cut + L * cut;
    tab[L].cut_cdf = (cut_cdf >= max_table) ? max_table : cut_cdf;
  }
  for (s = 0; s < num_cuts; ++s) {
    if (s * cut >= max_table) break;
    const int other = tab[s].other_symbol;
    const int32_t cut_cdf = tab[s].cut_cdf;
    const int32_t count_s = cut_cdf - s * cut;
    const int32_t count_other = ((s + 1) * cut >= max_table) ? (max_table - cut_cdf) : (cut - count_s);
    tab[s].self_alias_offset = s * cut - cnt[s];
    tab[s].other_alias_offset = s * cut + count_s - cnt[other];
    cnt[s] += count_s;
    cnt[other] += count_other;
  }
  for (int32_t r = 0; r < max_table; ++r) {
    const int32_t id = r / cut;
    const int32_t cut_cdf = tab[id].cut_cdf;
    const int32_t s_idx = (r >= cut_cdf) ? tab[id].other_symbol : id;
    const int32_t a_start = (r >= cut_cdf) ? tab[id].other_alias_offset : tab[id].self_alias_offset;
    const int64_t at = (int64_t)r - a_start + cdf[s_idx];
    if (at >= 0 && at < remap_cap) remap[at] = r;
  }
done:
  free(symbols);
  free(proba);
  free(cnt);
  return ret;
}

/* rans_alias_build_table, rans.cpp:56-95: remap rows (K, W + 2^fp) and table rows (K, 5W), both
 * starting with the cdf row (cdf_size entries) and zero elsewhere.  Returns the number of rows
 * for which the build succeeded. */
int64_t orc_alias_build(const int32_t* cdfs, const int32_t* sizes, int64_t num_tables,
                        int64_t cdf_width, int sp, int fp, int32_t* remap_out, int32_t* table_out) {
  const int64_t rw = cdf_width + ((int64_t)1 << fp);
  const int64_t tw = cdf_width * 5;
  int64_t ok = 0;
  memset(remap_out, 0, sizeof(int32_t) * (size_t)(num_tables * rw));
  memset(table_out, 0, sizeof(int32_t) * (size_t)(num_tables * tw));
  for (int64_t k = 0; k < num_tables; k++) {
    const int32_t* cdf = cdfs + k * cdf_width;
    const int32_t sz = sizes[k];
    int32_t* rrow = remap_out + k * rw;
    int32_t* trow = table_out + k * tw;
    memcpy(rrow, cdf, sizeof(int32_t) * (size_t)sz);
    memcpy(trow, cdf, sizeof(int32_t) * (size_t)sz);
    ok += orc_build_alias_row(cdf, sz, (orc_alias_elem*)(trow + sz), rrow + sz, sp, fp,
                              (tw - sz) / 4, rw - sz);
  }
  return ok;
}
