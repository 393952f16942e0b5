/* chpe_synth.c -- deterministic synthetic .chpe archives; see chpe_synth.h.
 *
 * Tile roles come from the same tensor maps the engine uses (chpe_maps.c).
 * Where the reference reads past a tile (D = 4096/8192 embeddings and 72B
 * norms/biases, which read more bytes than a 16 KiB tile holds), the bytes it
 * reads instead are filled so that the reference's own rules keep them benign:
 * scales read from a neighbour are small positive FP16 values, a 72B q-bias
 * over-read lands on small finite f32 values, and a 72B norm over-read meets a
 * NaN so the reference's "non-finite -> all gains 1.0" rule applies.
 */
#include "chpe_synth.h"

#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "chpe_maps.h"

/* ---- random streams ------------------------------------------------------ */
typedef struct { uint64_t s; } Rng;
static inline uint64_t rng_next(Rng *r) { /* SplitMix64 */
  uint64_t z = (r->s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline Rng rng_for(uint64_t seed, uint64_t tile, uint64_t stream) {
  Rng r = {seed * 0xD1B54A32D192ED03ull ^ (tile + 1) * 0x9E3779B97F4A7C15ull ^
           (stream + 1) * 0xA0761D6478BD642Full};
  rng_next(&r);
  return r;
}
/* Irwin-Hall(4) of 16-bit uniforms: mean 0, unit variance (std 37837.22). */
static inline float rng_normal(Rng *r) {
  uint64_t u = rng_next(r);
  int32_t s = (int32_t)(u & 0xFFFF) + (int32_t)((u >> 16) & 0xFFFF) +
              (int32_t)((u >> 32) & 0xFFFF) + (int32_t)(u >> 48) - 131070;
  return (float)s * (1.0f / 37837.22f);
}

static uint16_t f32_to_f16(float f) { /* round to nearest even */
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  int32_t e = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
  uint32_t m = x & 0x7FFFFFu;
  if (((x >> 23) & 0xFF) == 0xFF) return (uint16_t)(sign | 0x7C00u | (m ? 0x200u : 0));
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    m |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t half = 1u << (shift - 1);
    uint32_t r = m >> shift, rem = m & ((1u << shift) - 1);
    if (rem > half || (rem == half && (r & 1))) r++;
    return (uint16_t)(sign | r);
  }
  uint32_t r = m >> 13, rem = m & 0x1FFFu;
  uint32_t h = sign | ((uint32_t)e << 10) | r;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) h++;
  return (uint16_t)h;
}
static uint16_t f32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t lsb = (x >> 16) & 1u;
  return (uint16_t)((x + 0x7FFFu + lsb) >> 16);
}
static inline void wr16(uint8_t *p, uint16_t v) { memcpy(p, &v, 2); }
static inline void wr32(uint8_t *p, uint32_t v) { memcpy(p, &v, 4); }
static inline void wr64(uint8_t *p, uint64_t v) { memcpy(p, &v, 8); }
static inline void wrf32(uint8_t *p, float v) { memcpy(p, &v, 4); }

/* ---- roles --------------------------------------------------------------- */
enum {
  R_ZERO = 0, R_NORM, R_BIAS, R_RAW_W, R_ROWTILE, R_FLAT, R_EMBED_CELL, R_BIAS_NEIGHBOUR
};
/* cell formats */
enum { F_W4G = 0, F_W4SB, F_W2G, F_W2SB, F_W8, F_F16, F_BF16, F_F32, F_ZEROFLAT };

typedef struct {
  uint8_t role, fmt;
  uint16_t rows; /* row-tiled rows per cell */
} Role;

typedef struct {
  int config, arch, is_raw, bits;
  uint32_t flags;
  uint64_t n_tiles, stride, total;
  Role *roles;
} Plan;

static void set_span(Plan *p, int64_t start, int64_t count, int64_t used, uint8_t role,
                     uint8_t fmt, uint16_t rows) {
  for (int64_t i = 0; i < count; i++) {
    Role r = {i < used ? role : (uint8_t)R_ZERO, fmt, rows};
    p->roles[start + i] = r;
  }
}

static uint8_t mixed_fmt(size_t layer, int tensor, int flat) {
  uint64_t h = (layer * 31 + (uint64_t)tensor * 7 + 3) * 0x9E3779B97F4A7C15ull;
  h ^= h >> 29;
  if (flat) {
    static const uint8_t F[5] = {F_W4G, F_W4SB, F_W2G, F_W2SB, F_ZEROFLAT};
    return F[h % 5];
  }
  static const uint8_t R[8] = {F_W4G, F_W4SB, F_W2G, F_W2SB, F_W8, F_F16, F_BF16, F_F32};
  return R[h % 8];
}
static uint16_t rows_for(uint8_t fmt) {
  switch (fmt) {
    case F_W8: return 8;
    case F_F16: case F_BF16: return 4;
    case F_F32: return 2;
    default: return 16;
  }
}

static int make_plan(int config, uint32_t flags, Plan *p) {
  memset(p, 0, sizeof(*p));
  p->config = config;
  p->flags = flags;
  switch (config) {
    case CHPE_SYNTH_3B_FP16_RAW: case CHPE_SYNTH_3B_BF16_RAW:
      p->arch = CHPE_ARCH_3B; p->is_raw = 1; p->bits = 16; break;
    case CHPE_SYNTH_3B_W4: p->arch = CHPE_ARCH_3B; p->bits = 4; break;
    case CHPE_SYNTH_3B_W2: p->arch = CHPE_ARCH_3B; p->bits = 2; break;
    case CHPE_SYNTH_9B_W4: p->arch = CHPE_ARCH_9B; p->bits = 4; break;
    case CHPE_SYNTH_72B_W4: p->arch = CHPE_ARCH_72B; p->bits = 4; break;
    case CHPE_SYNTH_72B_FP16_RAW: p->arch = CHPE_ARCH_72B; p->is_raw = 1; p->bits = 16; break;
    case CHPE_SYNTH_9B_I8_RAW: p->arch = CHPE_ARCH_9B; p->is_raw = 1; p->bits = 8; break;
    default: return -1;
  }
  p->n_tiles = (uint64_t)chpe_total_records(p->arch, p->is_raw);
  if (p->is_raw) p->stride = CHPE_TILE_CODE_BYTES;
  else p->stride = (flags & CHPE_SYNTH_STANDARD) ? CHPE_RECORD_BYTES : CHPE_CELL_BYTES;
  p->total = CHPE_HEADER_BYTES + p->n_tiles * p->stride;
  return 0;
}

static int fill_roles(Plan *p) {
  p->roles = (Role *)calloc(p->n_tiles, sizeof(Role));
  if (!p->roles) return -1;
  const ChpeArch *A = chpe_arch_preset(p->arch);
  uint8_t wf = p->bits == 2 ? ((p->flags & CHPE_SYNTH_NONGROUP) ? F_W2SB : F_W2G)
                            : ((p->flags & CHPE_SYNTH_NONGROUP) ? F_W4SB : F_W4G);
  int mixed = (p->flags & CHPE_SYNTH_MIXED) != 0;
  const uint64_t wpt = p->is_raw ? (p->bits == 8 ? 16384 : 8192) : 32768;
  /* embeddings */
  int64_t emb_tiles = p->arch == CHPE_ARCH_3B ? (p->is_raw ? 37984 : 9496)
                     : p->arch == CHPE_ARCH_9B ? 62080 : 38016;
  if (p->is_raw) set_span(p, 0, emb_tiles, emb_tiles, R_RAW_W, 0, 0);
  else if (p->arch == CHPE_ARCH_3B) set_span(p, 0, emb_tiles, emb_tiles, R_ROWTILE, wf, 16);
  else set_span(p, 0, emb_tiles, emb_tiles, R_EMBED_CELL, wf, 16);

  for (size_t l = 0; l < A->L; l++) {
    ChpeLayerInfo li;
    chpe_layer_info(p->arch, p->is_raw, l, &li);
    p->roles[li.input_norm].role = R_NORM;
    p->roles[li.post_norm].role = R_NORM;
    int64_t qd = (int64_t)A->H * A->HD, kvd = (int64_t)A->KV * A->HD;
    struct { int64_t start, tiles, rows, cols; } T[7] = {
        {li.q_proj, li.q_tiles, qd, A->D},   {li.k_proj, li.k_tiles, kvd, A->D},
        {li.v_proj, li.v_tiles, kvd, A->D},  {li.o_proj, li.o_tiles, A->D, qd},
        {li.gate_proj, li.gate_tiles, A->F, A->D}, {li.up_proj, li.up_tiles, A->F, A->D},
        {li.down_proj, li.down_tiles, A->D, A->F}};
    for (int t = 0; t < 7; t++) {
      int64_t used = (int64_t)(((uint64_t)T[t].rows * (uint64_t)T[t].cols + wpt - 1) / wpt);
      if (p->is_raw) {
        set_span(p, T[t].start, T[t].tiles, T[t].tiles, R_RAW_W, 0, 0);
      } else if (T[t].cols <= 2048) {
        uint8_t f = mixed ? mixed_fmt(l, t, 0) : wf;
        set_span(p, T[t].start, T[t].tiles, T[t].tiles, R_ROWTILE, f, rows_for(f));
      } else {
        uint8_t f = mixed ? mixed_fmt(l, t, 1) : wf;
        if (used > T[t].tiles) used = T[t].tiles;
        set_span(p, T[t].start, T[t].tiles, used, R_FLAT, f, 0);
      }
    }
    if (li.q_bias >= 0) {
      p->roles[li.q_bias].role = R_BIAS;
      p->roles[li.k_bias].role = R_BIAS;
      p->roles[li.v_bias].role = R_BIAS;
      /* 72B q-bias reads 32 KiB: the first cell of k_proj is its neighbour. */
      if (p->arch == CHPE_ARCH_72B && !p->is_raw)
        p->roles[li.k_proj].role = R_BIAS_NEIGHBOUR;
    }
  }
  p->roles[chpe_final_norm_index(p->arch, p->is_raw)].role = R_NORM;
  int64_t lhs, lht;
  chpe_lm_head_span(p->arch, &lhs, &lht);
  if (lhs >= 0) {
    int64_t used = (int64_t)(((uint64_t)A->V * A->D + wpt - 1) / wpt);
    if (used > lht) used = lht;
    set_span(p, lhs, lht, used, p->is_raw ? R_RAW_W : R_FLAT, wf, 0);
  }
  return 0;
}

/* ---- tile writers -------------------------------------------------------- */
static uint16_t benign_scale16(Rng *r) { /* f16 in [2^-7, 2^-4): as u16 >= 8192 */
  return (uint16_t)(0x2000u + (uint32_t)(rng_next(r) % 0x0C00u));
}

static void write_cell_meta(uint8_t *cell, uint8_t qbits, uint64_t cflags, float scale,
                            float bias, uint32_t rows, uint32_t cols) {
  uint8_t *pl = cell + CHPE_PAYLOAD_OFF;
  pl[20] = qbits;
  wr64(pl + 24, cflags);
  wrf32(pl + 32, scale);
  wrf32(pl + 36, bias);
  wr32(pl + 40, rows);
  wr32(pl + 44, cols);
}

static void write_group_scales(uint8_t *pl, Rng *r) {
  for (int i = 0; i < 256; i++) {
    float s = rng_normal(r) * 0.01f;
    wr16(pl + 48 + 2 * i, f32_to_f16(s < 0 ? -s : s));
  }
}

static void write_codes(uint8_t *codes, size_t n, Rng *r) {
  size_t i = 0;
  for (; i + 8 <= n; i += 8) {
    uint64_t v = rng_next(r);
    memcpy(codes + i, &v, 8);
  }
  if (i < n) {
    uint64_t v = rng_next(r);
    memcpy(codes + i, &v, n - i);
  }
}

static void write_row_outliers(uint8_t *pl, Rng *r, uint32_t cols) {
  for (int i = 0; i < 128; i++) wr16(pl + 560 + 2 * i, f32_to_f16(rng_normal(r) * 0.02f));
  for (int k = 0; k < 8; k++) wr16(pl + 816 + 2 * k, (uint16_t)(rng_next(r) % cols));
}

static void write_down_aux(uint8_t *pl, Rng *r) {
  const int n = 8;
  wr16(pl + 560, (uint16_t)n);
  for (int m = 0; m < n; m++) {
    wr16(pl + 560 + 2 + 2 * m, f32_to_f16(rng_normal(r) * 0.05f));
    wr16(pl + 560 + 130 + 2 * m, (uint16_t)(rng_next(r) % 32768));
  }
}

/* A row-tiled cell of `rows` x 2048 (chpe_engine.zig:223-581 layouts). */
static void write_rowtile(uint8_t *cell, const Plan *p, uint8_t fmt, uint16_t rows, Rng *r) {
  uint8_t *codes = cell + CHPE_CELL_HEADER_BYTES, *pl = cell + CHPE_PAYLOAD_OFF;
  const uint32_t cols = 2048;
  int outl = (p->flags & CHPE_SYNTH_OUTLIERS) != 0;
  switch (fmt) {
    case F_W4G: case F_W2G: {
      int b = fmt == F_W4G ? 4 : 2;
      write_codes(codes, (size_t)rows * cols * b / 8, r);
      write_cell_meta(cell, (uint8_t)b, CHPE_FLAG_GROUP128_OUTLIERS, 0, 0, rows, cols);
      write_group_scales(pl, r);
      if (outl) write_row_outliers(pl, r, cols);
      break;
    }
    case F_W4SB: case F_W2SB: {
      int b = fmt == F_W4SB ? 4 : 2;
      write_codes(codes, (size_t)rows * cols * b / 8, r);
      float s = rng_normal(r) * 0.01f;
      write_cell_meta(cell, (uint8_t)b, 0, s < 0 ? -s : s, rng_normal(r) * 0.001f, rows, cols);
      /* the reference's embedding path reads group scales for every 4/2-bit
       * cell whatever the flag says (unpackEmbedRowCell), so they are filled */
      write_group_scales(pl, r);
      break;
    }
    case F_W8: {
      for (size_t i = 0; i < (size_t)rows * cols; i++) {
        float v = rng_normal(r) * 40.0f;
        int q = (int)(v < 0 ? v - 0.5f : v + 0.5f);
        codes[i] = (uint8_t)(int8_t)(q > 127 ? 127 : q < -127 ? -127 : q);
      }
      write_cell_meta(cell, 8, 0, 0.0005f, 0.0f, rows, cols);
      break;
    }
    case F_F16: case F_BF16:
      for (size_t i = 0; i < (size_t)rows * cols; i++) {
        float w = rng_normal(r) * 0.02f;
        wr16(codes + 2 * i, fmt == F_F16 ? f32_to_f16(w) : f32_to_bf16(w));
      }
      write_cell_meta(cell, 16, fmt == F_F16 ? CHPE_FLAG_RAW_FP16 : 0, 0, 0, rows, cols);
      break;
    case F_F32:
      for (size_t i = 0; i < (size_t)rows * cols; i++) wrf32(codes + 4 * i, rng_normal(r) * 0.02f);
      write_cell_meta(cell, 32, 0, 0, 0, rows, cols);
      break;
  }
}

/* A flat 32768-weight cell (chpe_engine.zig:584-729). */
static void write_flat(uint8_t *cell, const Plan *p, uint8_t fmt, Rng *r) {
  uint8_t *codes = cell + CHPE_CELL_HEADER_BYTES, *pl = cell + CHPE_PAYLOAD_OFF;
  int outl = (p->flags & CHPE_SYNTH_OUTLIERS) != 0;
  switch (fmt) {
    case F_W4G: case F_W2G: {
      int b = fmt == F_W4G ? 4 : 2;
      write_codes(codes, 32768u * b / 8, r);
      write_cell_meta(cell, (uint8_t)b, CHPE_FLAG_GROUP128_OUTLIERS, 0, 0, 0, 0);
      write_group_scales(pl, r);
      break;
    }
    case F_W4SB: case F_W2SB: {
      int b = fmt == F_W4SB ? 4 : 2;
      write_codes(codes, 32768u * b / 8, r);
      float s = rng_normal(r) * 0.01f;
      write_cell_meta(cell, (uint8_t)b, 0, s < 0 ? -s : s, rng_normal(r) * 0.001f, 0, 0);
      break;
    }
    default: /* an 8-bit flat cell: the reference reads it as zeros */
      write_codes(codes, 16384, r);
      write_cell_meta(cell, 8, 0, 0.01f, 0, 0, 0);
      return;
  }
  if (outl) write_down_aux(pl, r);
}

/* Embedding cells of the 9B/72B archives: random codes and group scales, with
 * every FP16 a row >= 16384/(D/2) would read as a scale kept benign (the rest
 * of the payload, this cell's header, the first bytes of its codes). */
static void write_embed_cell(uint8_t *cell, const Plan *p, uint8_t fmt, Rng *r) {
  uint8_t *codes = cell + CHPE_CELL_HEADER_BYTES, *pl = cell + CHPE_PAYLOAD_OFF;
  int b = (fmt == F_W2G || fmt == F_W2SB) ? 2 : 4;
  write_codes(codes, 16384, r);
  write_cell_meta(cell, (uint8_t)b, CHPE_FLAG_GROUP128_OUTLIERS, 0, 0, 16, chpe_arch_preset(p->arch)->D);
  write_group_scales(pl, r);
  for (int off = 560; off < 960; off += 2) wr16(pl + off, benign_scale16(r));
  for (int off = 0; off < 64; off += 2) wr16(cell + off, benign_scale16(r));
  for (int off = 0; off < 1088; off += 2) wr16(codes + off, benign_scale16(r));
}

static void write_tile(const Plan *p, uint64_t seed, uint64_t t, uint8_t *rec) {
  memset(rec, 0, p->stride);
  Role ro = p->roles[t];
  Rng r = rng_for(seed, t, 0);
  const ChpeArch *A = chpe_arch_preset(p->arch);
  uint8_t *cell = p->is_raw ? rec : (p->stride == CHPE_RECORD_BYTES ? rec + CHPE_PREFETCH_BYTES : rec);
  uint8_t *codes = p->is_raw ? rec : cell + CHPE_CELL_HEADER_BYTES;
  switch (ro.role) {
    case R_ZERO: break;
    case R_NORM:
      if (p->is_raw && p->arch == CHPE_ARCH_9B) {
        for (uint32_t i = 0; i < A->D; i++) wr16(codes + 2 * i, 0x3F80u); /* bf16 1.0 */
      } else {
        for (uint32_t i = 0; i < A->D && 4 * i < CHPE_TILE_CODE_BYTES; i++) wrf32(codes + 4 * i, 1.0f);
      }
      if (!p->is_raw) {
        write_cell_meta(cell, 32, 0, 0, 0, 0, 0);
        /* a 72B norm reads 32 KiB; the non-finite value in this cell's payload
         * makes the reference fall back to gains of 1.0 */
        if (p->arch == CHPE_ARCH_72B) wr32(cell + CHPE_PAYLOAD_OFF + 900, 0x7FC00000u);
      }
      break;
    case R_BIAS:
      if (p->flags & CHPE_SYNTH_BIAS)
        for (uint32_t i = 0; i < A->H * A->HD && 4 * i < CHPE_TILE_CODE_BYTES; i++)
          wrf32(codes + 4 * i, rng_normal(&r) * 0.02f);
      if (!p->is_raw) write_cell_meta(cell, 32, 0, 0, 0, 0, 0);
      break;
    case R_RAW_W:
      if (p->bits == 8) {
        for (int i = 0; i < 16384; i++) {
          float v = rng_normal(&r) * 5.35f;
          int q = (int)(v < 0 ? v - 0.5f : v + 0.5f);
          codes[i] = (uint8_t)(int8_t)(q > 127 ? 127 : q < -127 ? -127 : q);
        }
      } else {
        int bf = p->config == CHPE_SYNTH_3B_BF16_RAW;
        for (int i = 0; i < 8192; i++) {
          float w = rng_normal(&r) * 0.02f;
          wr16(codes + 2 * i, bf ? f32_to_bf16(w) : f32_to_f16(w));
        }
      }
      break;
    case R_ROWTILE: write_rowtile(cell, p, ro.fmt, ro.rows, &r); break;
    case R_FLAT: write_flat(cell, p, ro.fmt, &r); break;
    case R_EMBED_CELL: write_embed_cell(cell, p, ro.fmt, &r); break;
    case R_BIAS_NEIGHBOUR: {
      write_flat(cell, p, ro.fmt, &r);
      /* small finite f32 values where a 72B q-bias read overruns its tile */
      for (int i = 0; i < 15360; i += 4) {
        uint32_t v = (uint32_t)rng_next(&r);
        v = (v & 0x80FFFFFFu) | 0x3A000000u;
        wr32(codes + i, v);
      }
      break;
    }
  }
}

static void write_header(const Plan *p, uint8_t *h) {
  memset(h, 0, CHPE_HEADER_BYTES);
  int standard = !p->is_raw && p->stride == CHPE_RECORD_BYTES;
  wr32(h + 0, standard ? CHPE_ARCHIVE_MAGIC : CHPE_CHPE_MAGIC);
  wr32(h + 4, 1);
  wr64(h + 8, CHPE_HEADER_BYTES);
  wr64(h + 16, p->n_tiles);
  wr64(h + 24, p->n_tiles);
  wr64(h + 32, p->stride);
  wr64(h + 40, p->is_raw ? CHPE_TILE_CODE_BYTES : CHPE_CELL_BYTES);
  wr64(h + 48, standard ? CHPE_PREFETCH_BYTES : 0);
  uint64_t fl = 0;
  if (p->is_raw && p->bits == 16 && p->config != CHPE_SYNTH_3B_BF16_RAW) fl |= CHPE_FLAG_RAW_FP16;
  if (p->is_raw && p->bits == 8) fl |= CHPE_FLAG_RAW_INT8;
  wr64(h + 56, fl);
}

uint64_t chpe_synth_bytes(int config, uint32_t flags) {
  Plan p;
  if (make_plan(config, flags, &p)) return 0;
  return p.total;
}

typedef struct {
  const Plan *p;
  uint64_t seed, t0, t1;
  uint8_t *base; /* archive byte 0 */
  uint64_t base_tile; /* tile held at base + HEADER (streaming writes) */
} Work;

static void *work_fn(void *arg) {
  Work *w = (Work *)arg;
  for (uint64_t t = w->t0; t < w->t1; t++)
    write_tile(w->p, w->seed, t, w->base + CHPE_HEADER_BYTES + (t - w->base_tile) * w->p->stride);
  return NULL;
}

static void run_tiles(const Plan *p, uint64_t seed, uint8_t *base, uint64_t base_tile,
                      uint64_t t0, uint64_t t1, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 128) threads = 128;
  pthread_t th[128];
  Work w[128];
  uint64_t n = t1 - t0;
  for (int i = 0; i < threads; i++) {
    w[i].p = p; w[i].seed = seed; w[i].base = base; w[i].base_tile = base_tile;
    w[i].t0 = t0 + n * (uint64_t)i / (uint64_t)threads;
    w[i].t1 = t0 + n * (uint64_t)(i + 1) / (uint64_t)threads;
    pthread_create(&th[i], NULL, work_fn, &w[i]);
  }
  for (int i = 0; i < threads; i++) pthread_join(th[i], NULL);
}

int chpe_synth_fill(int config, uint32_t flags, uint64_t seed, uint8_t *out, uint64_t len,
                    int threads) {
  Plan p;
  if (make_plan(config, flags, &p) || len < p.total) return -1;
  if (fill_roles(&p)) return -2;
  write_header(&p, out);
  run_tiles(&p, seed, out, 0, 0, p.n_tiles, threads);
  free(p.roles);
  return 0;
}

int chpe_synth_write(int config, uint32_t flags, uint64_t seed, const char *path, int threads) {
  Plan p;
  if (make_plan(config, flags, &p)) return -1;
  if (fill_roles(&p)) return -2;
  FILE *f = fopen(path, "wb");
  if (!f) { free(p.roles); return -3; }
  uint8_t *buf = (uint8_t *)malloc(CHPE_HEADER_BYTES + 4096 * p.stride);
  write_header(&p, buf);
  int rc = fwrite(buf, 1, CHPE_HEADER_BYTES, f) == CHPE_HEADER_BYTES ? 0 : -4;
  for (uint64_t t = 0; t < p.n_tiles && rc == 0; t += 4096) {
    uint64_t t1 = t + 4096 < p.n_tiles ? t + 4096 : p.n_tiles;
    run_tiles(&p, seed, buf, t, t, t1, threads);
    size_t n = (size_t)((t1 - t) * p.stride);
    if (fwrite(buf + CHPE_HEADER_BYTES, 1, n, f) != n) rc = -4;
  }
  free(buf);
  free(p.roles);
  if (fclose(f)) rc = -4;
  return rc;
}
