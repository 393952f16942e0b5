/* chpe_maps.c -- see chpe_maps.h for the reference sources restated here. */
#include "chpe_maps.h"

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
