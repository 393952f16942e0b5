/* chpe_maps.c -- see chpe_maps.h for the reference sources restated here. */
#include "chpe_maps.h"

#include <stdlib.h>

static const ChpeArch PRESETS[3] = {
    /* chpe_engine.zig:110-145 */
    {"Qwen2.5-3B", 2048, 11008, 36, 16, 2, 128, 151936, 0, 1000000.0f, 1e-6f},
    {"Qwen3.5-9B", 4096, 12288, 32, 16, 4, 256, 248320, 1, 1000000.0f, 1e-6f},
    {"Qwen2.5-72B", 8192, 29568, 80, 64, 8, 128, 152064, 0, 1000000.0f, 1e-6f},
};

const ChpeArch *chpe_arch_preset(int arch) {
  return (arch >= 0 && arch < 3) ? &PRESETS[arch] : 0;
}

/* The reference's table for the 3B cell archive, carried as data. */
static const int64_t MAP3B_CELL[36][12] = {
#include "qwen3b_cell_map.inc"
};

/* 9B: embed 62080 tiles, then 32 layers in order; a full-attention layer
 * (l % 4 == 3) spans 12804 tiles, a linear-attention layer 13337. */
static int64_t map9b_base(size_t l) {
  int64_t b = 62080;
  for (size_t i = 0; i < l; i++) b += (i % 4 == 3) ? 12804 : 13337;
  return b;
}

void chpe_9b_extra(size_t l, Chpe9bExtra *o) {
  int64_t b = map9b_base(l);
  o->is_full = (l % 4 == 3);
  if (o->is_full) {
    o->in_proj_qkv = o->in_proj_z = o->in_proj_a = o->in_proj_b = -1;
    o->conv1d = o->a_log = o->dt_bias = o->linear_norm = o->out_proj = -1;
    o->q_norm = b + 3585;
    o->k_norm = b + 3586;
  } else {
    o->in_proj_qkv = b + 1;
    o->in_proj_z = b + 2049;
    o->in_proj_a = b + 3073;
    o->in_proj_b = b + 3081;
    o->conv1d = b + 3089;
    o->a_log = b + 3093;
    o->dt_bias = b + 3094;
    o->linear_norm = b + 3095;
    o->out_proj = b + 3096;
    o->q_norm = o->k_norm = -1;
  }
}

void chpe_layer_info(int arch, int is_raw, size_t l, ChpeLayerInfo *o) {
  if (arch == CHPE_ARCH_3B) {
    if (is_raw) {
      int64_t b = 37984 + (int64_t)l * 9413;
      ChpeLayerInfo r = {b, b + 1, 512, b + 513, b + 514, 64, b + 578, b + 579, 64,
                         b + 643, b + 644, 512, b + 1156, b + 1157, 2752, b + 3909,
                         2752, b + 6661, 2752};
      *o = r;
    } else {
      const int64_t *m = MAP3B_CELL[l];
      ChpeLayerInfo r = {m[0], m[1], 128, m[2], m[3], 16, m[4], m[5], 16, m[6],
                         m[7], 128, m[8], m[9], 688, m[10], 688, m[11], 688};
      *o = r;
    }
  } else if (arch == CHPE_ARCH_72B) {
    int64_t b = 38016 + (int64_t)l * 26789;
    ChpeLayerInfo r = {b, b + 1, 2048, b + 2049, b + 2050, 256, b + 2306, b + 2307,
                       256, b + 2563, b + 2564, 2048, b + 4612, b + 4613, 7392,
                       b + 12005, 7392, b + 19397, 7392};
    *o = r;
  } else {
    int64_t b = map9b_base(l);
    if (l % 4 == 3) {
      ChpeLayerInfo r = {b, b + 1, 2048, -1, b + 2049, 256, -1, b + 2305, 256, -1,
                         b + 2561, 1024, b + 3587, b + 3588, 3072, b + 6660, 3072,
                         b + 9732, 3072};
      *o = r;
    } else { /* linear layers run as GQA in the reference (qkv->q, z->k, a->v) */
      ChpeLayerInfo r = {b, b + 1, 2048, -1, b + 2049, 1024, -1, b + 3073, 1, -1,
                         b + 3096, 1024, b + 4120, b + 4121, 3072, b + 7193, 3072,
                         b + 10265, 3072};
      *o = r;
    }
  }
}

int64_t chpe_final_norm_index(int arch, int is_raw) {
  if (arch == CHPE_ARCH_3B) return is_raw ? 376852 : 94348;
  if (arch == CHPE_ARCH_72B) return 2181136;
  return 484600;
}

void chpe_lm_head_span(int arch, int64_t *start, int64_t *tiles) {
  if (arch == CHPE_ARCH_72B) { *start = 2181137; *tiles = 38016; }
  else if (arch == CHPE_ARCH_9B) { *start = 484601; *tiles = 62080; }
  else { *start = -1; *tiles = 0; }
}

int64_t chpe_total_records(int arch, int is_raw) {
  if (arch == CHPE_ARCH_3B) return is_raw ? 376853 : 94349;
  if (arch == CHPE_ARCH_72B) return 2219153;
  return 546681;
}

int chpe_tp_slice_of(int arch, int rank, int world, ChpeTpSlice *out) {
  const ChpeArch *A = chpe_arch_preset(arch);
  if (!A || !out || world < 1 || rank < 0 || rank >= world) return -1;
  const uint32_t N = (uint32_t)world, R = (uint32_t)rank;
  if (A->H % N || A->D % N || A->F % N || A->V % N) return -1;
  const uint32_t G = A->H / A->KV, hq = A->H / N;
  ChpeTpSlice s;
  s.hq = hq;
  s.h0 = R * hq;
  s.kv0 = s.h0 / G;
  if (hq >= G) {
    if (hq % G) return -1;
    s.kvl = hq / G;
  } else {
    if (G % hq) return -1;
    s.kvl = 1;
  }
  s.dl = A->D / N;
  s.d0 = R * s.dl;
  s.fl = A->F / N;
  s.f0 = R * s.fl;
  s.vl = A->V / N;
  s.v0 = R * s.vl;
  *out = s;
  return 0;
}

/* Tile runs of a tensor-parallel rank.  A flat GEMV over rows [r0, r0+n) of
 * a tensor with C columns starting at tile `start` reads the weights
 * [r0*C, (r0+n)*C) of its flat index, i.e. the tiles
 * start + floor(r0*C/wpt) .. start + ceil((r0+n)*C/wpt) - 1, never past the
 * tensor's own tile count (codes and their group scales live in the same
 * record).  The embedding lookup reads record tok/rows_per_tile and up to two
 * records past the table (the reference's over-reads), so the embedding
 * records and two more are taken whole.  Norms and biases are read on the
 * host and take no device tiles. */
typedef struct {
  uint64_t lo, hi;
} TileSpan;

static int span_cmp(const void *a, const void *b) {
  const TileSpan *x = (const TileSpan *)a, *y = (const TileSpan *)b;
  if (x->lo != y->lo) return x->lo < y->lo ? -1 : 1;
  if (x->hi != y->hi) return x->hi < y->hi ? -1 : 1;
  return 0;
}

typedef struct {
  TileSpan *v;
  size_t n;
  uint64_t rc;
} SpanList;

static void span_add(SpanList *s, uint64_t lo, uint64_t hi) {
  if (lo >= s->rc) return;
  if (hi > s->rc) hi = s->rc;
  if (hi > lo) {
    s->v[s->n].lo = lo;
    s->v[s->n].hi = hi;
    s->n++;
  }
}

static void span_rows(SpanList *s, int64_t start, int64_t tiles, uint64_t r0, uint64_t n,
                      uint64_t C, uint64_t wpt) {
  if (start < 0) return;
  const uint64_t lo = (uint64_t)start + r0 * C / wpt;
  const uint64_t hi = (uint64_t)start + ((r0 + n) * C + wpt - 1) / wpt;
  const uint64_t end = (uint64_t)start + (uint64_t)tiles;
  span_add(s, lo, hi < end ? hi : end);
}

int64_t chpe_tp_tile_runs(int arch, int is_raw, uint64_t wpt, uint64_t record_count, int rank,
                          int world, uint64_t *runs, size_t cap) {
  const ChpeArch *A = chpe_arch_preset(arch);
  ChpeTpSlice sl;
  if (!A || wpt == 0 || chpe_tp_slice_of(arch, rank, world, &sl) != 0) return -1;
  SpanList s;
  s.n = 0;
  s.rc = record_count;
  s.v = (TileSpan *)malloc(sizeof(TileSpan) * (2 + 7 * (size_t)A->L));
  if (!s.v) return -1;
  {
    const uint64_t rows_per_tile = is_raw ? (wpt / A->D ? wpt / A->D : 1) : 16;
    span_add(&s, 0, (A->V + rows_per_tile - 1) / rows_per_tile + 2);
  }
  for (uint32_t l = 0; l < A->L; l++) {
    ChpeLayerInfo li;
    chpe_layer_info(arch, is_raw, l, &li);
    span_rows(&s, li.q_proj, li.q_tiles, (uint64_t)sl.h0 * A->HD, (uint64_t)sl.hq * A->HD, A->D, wpt);
    span_rows(&s, li.k_proj, li.k_tiles, (uint64_t)sl.kv0 * A->HD, (uint64_t)sl.kvl * A->HD, A->D, wpt);
    span_rows(&s, li.v_proj, li.v_tiles, (uint64_t)sl.kv0 * A->HD, (uint64_t)sl.kvl * A->HD, A->D, wpt);
    span_rows(&s, li.o_proj, li.o_tiles, sl.d0, sl.dl, A->D, wpt);
    span_rows(&s, li.gate_proj, li.gate_tiles, sl.f0, sl.fl, A->D, wpt);
    span_rows(&s, li.up_proj, li.up_tiles, sl.f0, sl.fl, A->D, wpt);
    span_rows(&s, li.down_proj, li.down_tiles, sl.d0, sl.dl, A->F, wpt);
  }
  {
    int64_t lhs, lht;
    chpe_lm_head_span(arch, &lhs, &lht);
    span_rows(&s, lhs, lht, sl.v0, sl.vl, A->D, wpt);
  }
  qsort(s.v, s.n, sizeof(TileSpan), span_cmp);
  /* merge overlapping and touching spans into runs */
  size_t nr = 0;
  for (size_t i = 0; i < s.n; i++) {
    if (nr > 0 && s.v[i].lo <= s.v[nr - 1].hi) {
      if (s.v[i].hi > s.v[nr - 1].hi) s.v[nr - 1].hi = s.v[i].hi;
    } else {
      s.v[nr++] = s.v[i];
    }
  }
  for (size_t i = 0; i < nr && i < cap && runs; i++) {
    runs[2 * i] = s.v[i].lo;
    runs[2 * i + 1] = s.v[i].hi;
  }
  free(s.v);
  return (int64_t)nr;
}
