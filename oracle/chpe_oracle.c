/*
 * chpe_oracle.c -- TEST INFRASTRUCTURE, NOT PART OF THE PRODUCT.
 *
 * CPU restatement of chpe-qwen-engine's per-token decode path.  Every function
 * cites the reference file:line it restates.  See chpe_oracle.h for the parity
 * status and numeric conventions.  Build: oracle/Makefile (gcc, -O2
 * -ffp-contract=off, pthreads).
 */
#include "chpe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <pthread.h>
#include <stdio.h>

/* ---- geometry (geometry.zig:24-62, weight_archive.zig:20-34) ------------- */
#define HEADER_BYTES 4096u
#define CELL_BYTES 17408u
#define RECORD_BYTES 20480u
#define PREFETCH_LABEL_BYTES 3072u
#define BYTECODE_HEADER_BYTES 64u
#define TILE_CODE_BYTES 16384u
#define PAYLOAD_OFF 16448u /* Cell.semantic_payload offset, geometry.zig:254 */
#define ARCHIVE_MAGIC 0x57415243u
#define CHPE_MAGIC 0x45504843u
#define FLAG_GROUP128_OUTLIERS 0x01u
#define FLAG_RAW_FP16 0x04u
#define INT8_RAW_SCALE 0.00373708f /* chpe_engine.zig:1236,1521 */

typedef float v8f __attribute__((vector_size(32)));

static inline uint16_t rd16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }
static inline uint32_t rd32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }
static inline uint64_t rd64(const uint8_t *p) { uint64_t v; memcpy(&v, p, 8); return v; }
static inline float rdf32(const uint8_t *p) { float v; memcpy(&v, p, 4); return v; }

/* IEEE binary16 -> binary32, exact (Zig @floatCast(f16 -> f32)). */
static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do { man <<= 1; e++; } while ((man & 0x400u) == 0);
      man &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
static inline float bf16_to_f32(uint16_t b) {
  uint32_t bits = (uint32_t)b << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
static inline float rdf16(const uint8_t *p) { return f16_to_f32(rd16(p)); }

/* @reduce(.Add, v) with preserved associativity: ordered lane sum. */
static inline float vreduce(v8f v) {
  float s = v[0];
  for (int i = 1; i < 8; i++) s += v[i];
  return s;
}
static inline v8f vfma(v8f a, v8f b, v8f c) {
  v8f r;
  for (int i = 0; i < 8; i++) r[i] = fmaf(a[i], b[i], c[i]);
  return r;
}
static inline v8f vload(const float *p) { v8f v; memcpy(&v, p, 32); return v; }

/* ---- parallel-for (pthreads; work items claimed in ascending order) ------ */
typedef void (*item_fn)(void *ctx, size_t i);
typedef struct { item_fn fn; void *ctx; size_t n; size_t next; pthread_mutex_t mu; } ParJob;
static void *par_worker(void *arg) {
  ParJob *j = (ParJob *)arg;
  for (;;) {
    pthread_mutex_lock(&j->mu);
    size_t i = j->next++;
    pthread_mutex_unlock(&j->mu);
    if (i >= j->n) return NULL;
    j->fn(j->ctx, i);
  }
}
static void par_for(size_t n, int nt, item_fn fn, void *ctx) {
  if (nt <= 1 || n <= 1) {
    for (size_t i = 0; i < n; i++) fn(ctx, i);
    return;
  }
  ParJob j = {fn, ctx, n, 0, PTHREAD_MUTEX_INITIALIZER};
  pthread_t th[256];
  if (nt > 256) nt = 256;
  for (int t = 0; t < nt; t++) pthread_create(&th[t], NULL, par_worker, &j);
  for (int t = 0; t < nt; t++) pthread_join(th[t], NULL);
}

static const float CODEBOOK_W2[4] = {0.0f, 1.0f, -2.0f, -1.0f}; /* chpe_engine.zig:220 */

/* ---- archive header (weight_archive.zig:53-86,152-172) ------------------- */
int oracle_validate(const uint8_t *b, size_t len, OracleHeader *h) {
  if (len < HEADER_BYTES) return ORACLE_ERR_FILE_TOO_SMALL;
  OracleHeader x;
  x.magic = rd32(b + 0); x.version = rd32(b + 4);
  x.header_bytes = rd64(b + 8); x.record_count = rd64(b + 16);
  x.tile_count = rd64(b + 24); x.record_bytes = rd64(b + 32);
  x.cell_bytes = rd64(b + 40); x.prefetch_bytes = rd64(b + 48);
  x.flags = rd64(b + 56);
  if (h) *h = x;
  if (x.magic != ARCHIVE_MAGIC && x.magic != CHPE_MAGIC) return ORACLE_ERR_INVALID_MAGIC;
  if (x.version != 1) return ORACLE_ERR_UNSUPPORTED_VERSION;
  if (x.header_bytes != HEADER_BYTES) return ORACLE_ERR_MISALIGNED_HEADER;
  int is_standard = x.record_bytes == RECORD_BYTES && x.prefetch_bytes == PREFETCH_LABEL_BYTES;
  int is_dense = x.record_bytes == CELL_BYTES && x.prefetch_bytes == 0;
  int is_raw = x.record_bytes == TILE_CODE_BYTES && x.prefetch_bytes == 0;
  if (!is_standard && !is_dense && !is_raw) return ORACLE_ERR_BAD_GEOMETRY;
  if (!is_raw && x.cell_bytes != CELL_BYTES) return ORACLE_ERR_BAD_GEOMETRY;
  if (is_raw && x.cell_bytes != TILE_CODE_BYTES) return ORACLE_ERR_BAD_GEOMETRY;
  /* header_bytes + record_count * stride, u64 arithmetic as in the reference */
  uint64_t required = x.header_bytes + x.record_count * x.record_bytes;
  if (required > len) return ORACLE_ERR_TRUNCATED;
  return ORACLE_OK;
}

/* ---- model presets (chpe_engine.zig:96-146) ------------------------------ */
typedef struct {
  const char *name;
  size_t D, F, L, H, KV, HD, V;
  int hybrid;
  float theta, eps;
} Arch;
static const Arch ARCHES[3] = {
    {"Qwen2.5-3B", 2048, 11008, 36, 16, 2, 128, 151936, 0, 1000000.0f, 1e-6f},
    {"Qwen3.5-9B", 4096, 12288, 32, 16, 4, 256, 248320, 1, 1000000.0f, 1e-6f},
    {"Qwen2.5-72B", 8192, 29568, 80, 64, 8, 128, 152064, 0, 1000000.0f, 1e-6f},
};

struct OracleEngine {
  Arch arch;
  int arch_id;
  const uint8_t *rec;
  size_t len;
  int is_dense, is_raw, is_raw_fp16, archive_valid;
  size_t stride, record_count, wpt;
  uint8_t quant_bits;
  int threads;
  float *hidden, *norm_buf, *norm_gamma, *bias_buf, *q, *k, *v, *attn_out,
      *gate, *up, *mlp, *logits, *lm_row;
  float *k_cache, *v_cache; /* [L][max_seq][KV*HD] f32, zeroed (chpe_engine.zig:755-801) */
  size_t max_seq;
  int kv_fp16; /* test option: round cached K/V to FP16 as a half-precision cache does */
};

static float round_f16(float f) { return (float)(_Float16)f; }

/* chpe_engine.zig:854-974 CHPEEngine.init format sniffing and sizing. */
OracleEngine *oracle_engine_new(const uint8_t *a, size_t len, int arch_id, size_t max_seq) {
  if (arch_id < 0 || arch_id > 2) return NULL;
  OracleEngine *e = (OracleEngine *)calloc(1, sizeof(*e));
  e->arch = ARCHES[arch_id];
  e->arch_id = arch_id;
  e->rec = a;
  e->len = len;
  e->threads = 1;
  e->quant_bits = 2;
  if (len >= 4096) {
    uint32_t magic = rd32(a);
    if (magic == CHPE_MAGIC || magic == ARCHIVE_MAGIC) {
      e->archive_valid = 1;
      e->record_count = (size_t)rd64(a + 16);
      uint64_t rec_b = rd64(a + 32), cell_b = rd64(a + 40), pre_b = rd64(a + 48),
               flags = rd64(a + 56);
      e->is_dense = pre_b == 0 && rec_b == cell_b && rec_b == CELL_BYTES;
      e->is_raw = rec_b == TILE_CODE_BYTES;
      e->is_raw_fp16 = e->is_raw && (flags & FLAG_RAW_FP16) != 0;
      if (e->is_raw_fp16) {
        e->quant_bits = 16;
      } else if (e->is_raw) {
        /* Q7: INT8 iff the arch name contains "9B" and (flag 0x08 or a
         * 7..10 GiB file) -- chpe_engine.zig:886-890 */
        int name9b = strstr(e->arch.name, "9B") != NULL;
        int sized = len < (size_t)10 * 1024 * 1024 * 1024 && len > (size_t)7 * 1024 * 1024 * 1024;
        e->quant_bits = (name9b && ((flags & 0x08) != 0 || sized)) ? 8 : 16;
      } else if (e->record_count > 0 &&
                 len >= 4096 + (e->is_dense ? CELL_BYTES : RECORD_BYTES)) {
        size_t cell_off = 4096 + (e->is_dense ? 0 : PREFETCH_LABEL_BYTES);
        e->quant_bits = a[cell_off + PAYLOAD_OFF + 20];
        if (e->quant_bits == 0) e->quant_bits = 2;
      }
    }
  }
  e->stride = e->is_raw ? TILE_CODE_BYTES : (e->is_dense ? CELL_BYTES : RECORD_BYTES);
  if (e->is_raw_fp16 || (e->is_raw && e->quant_bits == 16)) e->wpt = 8192;
  else if (e->is_raw && e->quant_bits == 8) e->wpt = 16384;
  else if (e->quant_bits == 8) e->wpt = 16384;
  else if (e->quant_bits == 4 || e->quant_bits == 2) e->wpt = 32768;
  else e->wpt = 8192;

  const Arch *A = &e->arch;
  size_t maxproj = A->D;
  if (A->H * A->HD > maxproj) maxproj = A->H * A->HD;
  if (A->F > maxproj) maxproj = A->F;
  e->hidden = calloc(A->D, 4);
  e->norm_buf = calloc(A->D, 4);
  e->norm_gamma = calloc(A->D, 4);
  e->bias_buf = calloc(maxproj, 4);
  e->q = calloc(A->H * A->HD, 4);
  e->k = calloc(A->KV * A->HD, 4);
  e->v = calloc(A->KV * A->HD, 4);
  e->attn_out = calloc(A->D, 4);
  e->gate = calloc(A->F, 4);
  e->up = calloc(A->F, 4);
  e->mlp = calloc(A->F, 4);
  e->logits = calloc(A->V, 4);
  e->lm_row = calloc(8192, 4);
  e->max_seq = max_seq;
  e->k_cache = calloc(A->L * max_seq * A->KV * A->HD, 4);
  e->v_cache = calloc(A->L * max_seq * A->KV * A->HD, 4);
  return e;
}

void oracle_engine_free(OracleEngine *e) {
  if (!e) return;
  free(e->hidden); free(e->norm_buf); free(e->norm_gamma); free(e->bias_buf);
  free(e->q); free(e->k); free(e->v); free(e->attn_out); free(e->gate);
  free(e->up); free(e->mlp); free(e->logits); free(e->lm_row);
  free(e->k_cache); free(e->v_cache);
  free(e);
}
void oracle_set_threads(OracleEngine *e, int n) { e->threads = n < 1 ? 1 : n; }
void oracle_set_kv_fp16(OracleEngine *e, int on) { e->kv_fp16 = on != 0; }

/* Writes K/V rows [n][KV*HD] at positions pos0.. of one layer of the cache
 * (chpe_engine.zig:755-801 holds them as f32 [L][max_seq][KV*HD]); a test
 * harness for prefilled long contexts, not a reference function.  Returns 0,
 * or -1 when the rows do not fit. */
int oracle_kv_load(OracleEngine *e, size_t layer, size_t pos0, size_t n, const float *k,
                   const float *v) {
  const Arch *A = &e->arch;
  size_t kvd = A->KV * A->HD;
  if (layer >= A->L || pos0 + n > e->max_seq) return -1;
  memcpy(e->k_cache + (layer * e->max_seq + pos0) * kvd, k, n * kvd * 4);
  memcpy(e->v_cache + (layer * e->max_seq + pos0) * kvd, v, n * kvd * 4);
  return 0;
}
const float *oracle_logits(const OracleEngine *e) { return e->logits; }
const float *oracle_hidden(const OracleEngine *e) { return e->hidden; }
size_t oracle_vocab(const OracleEngine *e) { return e->arch.V; }
size_t oracle_hidden_dim(const OracleEngine *e) { return e->arch.D; }
void oracle_engine_facts(const OracleEngine *e, int64_t o[7]) {
  o[0] = e->is_raw; o[1] = e->is_raw_fp16; o[2] = e->is_dense; o[3] = e->quant_bits;
  o[4] = (int64_t)e->wpt; o[5] = e->archive_valid; o[6] = (int64_t)e->record_count;
}

/* chpe_engine.zig:994-1011 getTileCodedPtr / getCellPointer */
static const uint8_t *tile_code_ptr(const OracleEngine *e, size_t idx) {
  if (e->is_raw) return e->rec + 4096 + idx * (size_t)TILE_CODE_BYTES;
  if (e->is_dense) return e->rec + 4096 + idx * (size_t)CELL_BYTES + BYTECODE_HEADER_BYTES;
  return e->rec + 4096 + idx * (size_t)RECORD_BYTES + PREFETCH_LABEL_BYTES + BYTECODE_HEADER_BYTES;
}
static const uint8_t *cell_ptr(const OracleEngine *e, size_t idx) {
  size_t off = 4096 + idx * e->stride;
  return e->rec + (e->is_dense ? off : off + PREFETCH_LABEL_BYTES);
}

/* ---- tensor maps -------------------------------------------------------- */
/* qwen3b_tensor_map.zig:27-531 LAYERS: the reference table, carried as data
 * (it is irregular: layer 21's down_proj follows layer 9).  Columns:
 * input_norm q_proj q_bias k_proj k_bias v_proj v_bias o_proj post_norm gate up down */
static const int64_t MAP3B_CELL[36][12] = {
#include "../chpe_qwen_engine_b200/csrc/qwen3b_cell_map.inc"
};
void oracle_map_3b_cell_layer(size_t l, int64_t o[12]) {
  for (int i = 0; i < 12; i++) o[i] = MAP3B_CELL[l][i];
}
/* qwen72b_tensor_map.zig:24-79 makeLayer */
void oracle_map_72b_layer(size_t l, int64_t o[12]) {
  int64_t base = 38016 + (int64_t)l * 26789;
  o[0] = base; o[1] = base + 1; o[2] = base + 1 + 2048; o[3] = base + 2 + 2048;
  o[4] = base + 2 + 2048 + 256; o[5] = base + 3 + 2048 + 256;
  o[6] = base + 3 + 2048 + 512; o[7] = base + 4 + 2048 + 512;
  o[8] = base + 4 + 4096 + 512; o[9] = base + 5 + 4096 + 512;
  o[10] = base + 5 + 4096 + 512 + 7392; o[11] = base + 5 + 4096 + 512 + 2 * 7392;
}
/* qwen35_tensor_map.zig:53-1015: embed 62080 tiles, then 32 layers in order;
 * full attention at l % 4 == 3 (12804 tiles), linear otherwise (13337). */
static int64_t map9b_base(size_t l) {
  int64_t b = 62080;
  for (size_t i = 0; i < l; i++) b += (i % 4 == 3) ? 12804 : 13337;
  return b;
}

/* chpe_engine.zig:1035-1132 getLayerInfo */
void oracle_layer_info(const OracleEngine *e, size_t l, OracleLayerInfo *o) {
  if (e->arch.D == 2048) {
    if (e->is_raw) {
      int64_t base = 37984 + (int64_t)l * 9413; /* qwen3b_geometry.zig:48-79 */
      *o = (OracleLayerInfo){base + 0, base + 1, 512, base + 513, base + 514, 64, base + 578,
                             base + 579, 64, base + 643, base + 644, 512, base + 1156,
                             base + 1157, 2752, base + 3909, 2752, base + 6661, 2752};
    } else {
      int64_t m[12];
      oracle_map_3b_cell_layer(l, m);
      *o = (OracleLayerInfo){m[0], m[1], 128, m[2], m[3], 16, m[4], m[5], 16, m[6],
                             m[7], 128, m[8], m[9], 688, m[10], 688, m[11], 688};
    }
  } else if (e->arch.D == 8192) {
    int64_t m[12];
    oracle_map_72b_layer(l, m);
    *o = (OracleLayerInfo){m[0], m[1], 2048, m[2], m[3], 256, m[4], m[5], 256, m[6],
                           m[7], 2048, m[8], m[9], 7392, m[10], 7392, m[11], 7392};
  } else {
    int64_t b = map9b_base(l);
    if (l % 4 == 3) { /* full attention */
      *o = (OracleLayerInfo){b, b + 1, 2048, -1, b + 2049, 256, -1, b + 2305, 256, -1,
                             b + 2561, 1024, b + 3587, b + 3588, 3072, b + 6660, 3072,
                             b + 9732, 3072};
    } else { /* Q8: linear layers run as GQA: qkv->q, z->k, a(1 tile)->v, out->o */
      *o = (OracleLayerInfo){b, b + 1, 2048, -1, b + 2049, 1024, -1, b + 3073, 1, -1,
                             b + 3096, 1024, b + 4120, b + 4121, 3072, b + 7193, 3072,
                             b + 10265, 3072};
    }
  }
}
/* chpe_engine.zig:1134-1142 */
int64_t oracle_final_norm_index(const OracleEngine *e) {
  if (e->arch.D == 2048) return e->is_raw ? 376852 : 94348;
  if (e->arch.D == 8192) return 2181136;
  return 484600;
}

/* ---- norm / bias (chpe_engine.zig:1144-1192) ------------------------------ */
void oracle_unpack_norm(const OracleEngine *e, size_t tile, float *out, size_t n) {
  if (!e->archive_valid || tile >= e->record_count) {
    for (size_t i = 0; i < n; i++) out[i] = 1.0f;
    return;
  }
  const uint8_t *t = tile_code_ptr(e, tile);
  if (e->arch.D == 4096 && e->is_raw) {
    for (size_t i = 0; i < n; i++) out[i] = bf16_to_f32(rd16(t + 2 * i));
  } else {
    memcpy(out, t, n * 4);
  }
  int all_zero = 1;
  for (size_t i = 0; i < n; i++) {
    if (!isfinite(out[i])) {
      for (size_t j = 0; j < n; j++) out[j] = 1.0f;
      return;
    }
    if (out[i] != 0.0f) all_zero = 0;
  }
  if (all_zero)
    for (size_t i = 0; i < n; i++) out[i] = 1.0f;
}
void oracle_unpack_bias(const OracleEngine *e, size_t tile, float *out, size_t n) {
  if (!e->archive_valid || tile >= e->record_count) {
    memset(out, 0, n * 4);
    return;
  }
  const uint8_t *t = tile_code_ptr(e, tile);
  if (e->arch.D == 4096 && e->is_raw) {
    for (size_t i = 0; i < n; i++) out[i] = bf16_to_f32(rd16(t + 2 * i));
  } else {
    memcpy(out, t, n * 4);
  }
  for (size_t i = 0; i < n; i++)
    if (!isfinite(out[i])) out[i] = 0.0f;
}

/* ---- raw segment dot (chpe_engine.zig:1194-1286) ------------------------ */
static float dot_segment(const OracleEngine *e, const uint8_t *tile, size_t j, size_t seg,
                         const float *x) {
  size_t k = 0;
  v8f acc = {0};
  if (e->is_raw_fp16) {
    const uint8_t *s = tile + 2 * j;
    for (; k + 8 <= seg; k += 8) {
      v8f w = {0};
      for (int i = 0; i < 8; i++) w[i] = rdf16(s + 2 * (k + i));
      acc = vfma(w, vload(x + k), acc);
    }
    float sum = vreduce(acc);
    for (; k < seg; k++) sum += rdf16(s + 2 * k) * x[k];
    return sum;
  } else if (e->is_raw) {
    if (e->quant_bits == 8) {
      const int8_t *s = (const int8_t *)tile + j;
      for (; k + 8 <= seg; k += 8) {
        v8f w = {0};
        for (int i = 0; i < 8; i++) w[i] = (float)s[k + i];
        acc = vfma(w, vload(x + k), acc);
      }
      float sum = vreduce(acc);
      for (; k < seg; k++) sum += (float)s[k] * x[k];
      return sum * INT8_RAW_SCALE;
    } else {
      const uint8_t *s = tile + 2 * j;
      for (; k + 8 <= seg; k += 8) {
        v8f w = {0};
        for (int i = 0; i < 8; i++) w[i] = bf16_to_f32(rd16(s + 2 * (k + i)));
        acc = vfma(w, vload(x + k), acc);
      }
      float sum = vreduce(acc);
      for (; k < seg; k++) sum += bf16_to_f32(rd16(s + 2 * k)) * x[k];
      return sum;
    }
  }
  /* The non-raw branch (:1255-1285) is unreachable: gemvLinear only calls
   * dotSegment for raw archives. */
  return 0.0f;
}

/* ---- cell GEMV kernels (chpe_engine.zig:223-581) ------------------------ */
typedef struct { float scale, bias; uint32_t rows, cols; } TileDims;
static TileDims tile_dims(const uint8_t *cell) {
  const uint8_t *p = cell + PAYLOAD_OFF + 32;
  TileDims d = {rdf32(p), rdf32(p + 4), rd32(p + 8), rd32(p + 12)};
  return d;
}
static inline uint8_t cell_qbits(const uint8_t *cell) { return cell[PAYLOAD_OFF + 20]; }
static inline uint64_t cell_flags(const uint8_t *cell) { return rd64(cell + PAYLOAD_OFF + 24); }

static void outlier_x(const uint8_t *payload, const float *x, size_t x_len, v8f *xo) {
  v8f z = {0};
  *xo = z;
  for (int k = 0; k < 8; k++) {
    uint16_t col = rd16(payload + 816 + 2 * k);
    if (col < x_len) (*xo)[k] = x[col];
  }
}
static float outlier_term(const uint8_t *payload, size_t r, v8f xo) {
  v8f w;
  for (int k = 0; k < 8; k++) w[k] = rdf16(payload + 560 + 2 * (r * 8 + k));
  return vreduce(w * xo);
}

static void gemv_w2(const uint8_t *cell, const float *x, size_t x_len, float *y, size_t y_len,
                    size_t row_base, int acc) {
  const uint8_t *pl = cell + PAYLOAD_OFF;
  const uint8_t *coded = cell + BYTECODE_HEADER_BYTES;
  TileDims d = tile_dims(cell);
  size_t rows = d.rows, cols = d.cols;
  int g128 = (cell_flags(cell) & FLAG_GROUP128_OUTLIERS) != 0;
  int has_out = g128 && rows == 16;
  v8f xo = {0};
  if (has_out) outlier_x(pl, x, x_len, &xo);
  size_t max_rows = row_base >= y_len ? 0 : (rows < y_len - row_base ? rows : y_len - row_base);
  size_t n_groups = cols / 128 < x_len / 128 ? cols / 128 : x_len / 128;
  size_t total_groups = cols / 128;
  for (size_t r = 0; r < max_rows; r++) {
    float row_sum = 0.0f;
    size_t rbo = r * (cols / 4);
    if (g128) {
      for (size_t g = 0; g < n_groups; g++) {
        float scale = rdf16(pl + 48 + 2 * (r * total_groups + g));
        const uint8_t *gb = coded + rbo + g * 32;
        const float *xs = x + g * 128;
        v8f dv = {0};
        for (size_t j = 0; j < 32; j += 2) {
          uint8_t b0 = gb[j], b1 = gb[j + 1];
          v8f qv = {CODEBOOK_W2[b0 & 3], CODEBOOK_W2[(b0 >> 2) & 3], CODEBOOK_W2[(b0 >> 4) & 3],
                    CODEBOOK_W2[(b0 >> 6) & 3], CODEBOOK_W2[b1 & 3], CODEBOOK_W2[(b1 >> 2) & 3],
                    CODEBOOK_W2[(b1 >> 4) & 3], CODEBOOK_W2[(b1 >> 6) & 3]};
          dv += qv * vload(xs + 4 * j);
        }
        row_sum += vreduce(dv) * scale;
      }
    } else {
      float scale = d.scale, bias = d.bias;
      size_t max_quads = cols / 4 < x_len / 4 ? cols / 4 : x_len / 4;
      const uint8_t *rb = coded + rbo;
      for (size_t b = 0; b < max_quads; b++) {
        uint8_t v = rb[b];
        float w0 = CODEBOOK_W2[v & 3] * scale + bias;
        float w1 = CODEBOOK_W2[(v >> 2) & 3] * scale + bias;
        float w2 = CODEBOOK_W2[(v >> 4) & 3] * scale + bias;
        float w3 = CODEBOOK_W2[(v >> 6) & 3] * scale + bias;
        size_t base = b * 4;
        row_sum += w0 * x[base] + w1 * x[base + 1] + w2 * x[base + 2] + w3 * x[base + 3];
      }
    }
    if (has_out) row_sum += outlier_term(pl, r, xo);
    if (acc) y[row_base + r] += row_sum; else y[row_base + r] = row_sum;
  }
}

static void gemv_w4(const uint8_t *cell, const float *x, size_t x_len, float *y, size_t y_len,
                    size_t row_base, int acc) {
  const uint8_t *pl = cell + PAYLOAD_OFF;
  const uint8_t *coded = cell + BYTECODE_HEADER_BYTES;
  TileDims d = tile_dims(cell);
  size_t rows = d.rows, cols = d.cols;
  int g128 = (cell_flags(cell) & FLAG_GROUP128_OUTLIERS) != 0;
  int has_out = g128 && rows == 16;
  v8f xo = {0};
  if (has_out) outlier_x(pl, x, x_len, &xo);
  size_t max_rows = row_base >= y_len ? 0 : (rows < y_len - row_base ? rows : y_len - row_base);
  for (size_t r = 0; r < max_rows; r++) {
    float row_sum = 0.0f;
    size_t rbo = r * (cols / 2);
    if (g128) {
      size_t n_groups = cols / 128 < x_len / 128 ? cols / 128 : x_len / 128;
      size_t total_groups = cols / 128;
      for (size_t g = 0; g < n_groups; g++) {
        float scale = rdf16(pl + 48 + 2 * (r * total_groups + g));
        const uint8_t *gb = coded + rbo + g * 64;
        const float *xs = x + g * 128;
        float gacc = 0.0f;
        for (size_t j = 0; j < 64; j += 4) {
          for (size_t idx = 0; idx < 4; idx++) {
            uint8_t v = gb[j + idx];
            float q0 = (float)(v & 0x0F) - 8.0f;
            float q1 = (float)((v >> 4) & 0x0F) - 8.0f;
            size_t base = (j + idx) * 2;
            gacc += q0 * xs[base] + q1 * xs[base + 1];
          }
        }
        row_sum += gacc * scale;
      }
    } else {
      float scale = d.scale, bias = d.bias;
      size_t max_pairs = cols / 2 < x_len / 2 ? cols / 2 : x_len / 2;
      const uint8_t *rb = coded + rbo;
      for (size_t b = 0; b < max_pairs; b++) {
        uint8_t v = rb[b];
        int n0 = (int)(v & 0x0F) - 8, n1 = (int)((v >> 4) & 0x0F) - 8;
        float w0 = (float)n0 * scale + bias, w1 = (float)n1 * scale + bias;
        size_t base = b * 2;
        row_sum += w0 * x[base] + w1 * x[base + 1];
      }
    }
    if (has_out) row_sum += outlier_term(pl, r, xo);
    if (acc) y[row_base + r] += row_sum; else y[row_base + r] = row_sum;
  }
}

static void gemv_w8(const uint8_t *cell, const float *x, size_t x_len, float *y, size_t y_len,
                    size_t row_base, int acc) {
  const int8_t *coded = (const int8_t *)(cell + BYTECODE_HEADER_BYTES);
  TileDims d = tile_dims(cell);
  size_t rows = d.rows, cols = d.cols;
  size_t max_rows = row_base >= y_len ? 0 : (rows < y_len - row_base ? rows : y_len - row_base);
  size_t max_cols = cols < x_len ? cols : x_len;
  for (size_t r = 0; r < max_rows; r++) {
    const int8_t *rw = coded + r * cols;
    v8f av = {0};
    size_t i = 0;
    for (; i + 8 <= max_cols; i += 8) {
      v8f w = {0};
      for (int k = 0; k < 8; k++) w[k] = (float)rw[i + k];
      av += w * vload(x + i);
    }
    float rs = vreduce(av);
    for (; i < max_cols; i++) rs += (float)rw[i] * x[i];
    float fv = rs * d.scale + d.bias;
    if (acc) y[row_base + r] += fv; else y[row_base + r] = fv;
  }
}

static void gemv_f16(const uint8_t *cell, const float *x, size_t x_len, float *y, size_t y_len,
                     size_t row_base, int acc) {
  const uint8_t *coded = cell + BYTECODE_HEADER_BYTES;
  TileDims d = tile_dims(cell);
  size_t rows = d.rows, cols = d.cols;
  int ieee = (cell_flags(cell) & FLAG_RAW_FP16) != 0;
  size_t max_rows = row_base >= y_len ? 0 : (rows < y_len - row_base ? rows : y_len - row_base);
  size_t max_cols = cols < x_len ? cols : x_len;
  for (size_t r = 0; r < max_rows; r++) {
    const uint8_t *rw = coded + 2 * r * cols;
    v8f av = {0};
    size_t c = 0;
    for (; c + 8 <= max_cols; c += 8) {
      v8f w = {0};
      for (int k = 0; k < 8; k++)
        w[k] = ieee ? rdf16(rw + 2 * (c + k)) : bf16_to_f32(rd16(rw + 2 * (c + k)));
      av = vfma(w, vload(x + c), av);
    }
    float sum = vreduce(av);
    for (; c < max_cols; c++)
      sum += (ieee ? rdf16(rw + 2 * c) : bf16_to_f32(rd16(rw + 2 * c))) * x[c];
    if (acc) y[row_base + r] += sum; else y[row_base + r] = sum;
  }
}

static void gemv_f32(const uint8_t *cell, const float *x, size_t x_len, float *y, size_t y_len,
                     size_t row_base, int acc) {
  const uint8_t *coded = cell + BYTECODE_HEADER_BYTES;
  TileDims d = tile_dims(cell);
  size_t rows = d.rows, cols = d.cols;
  size_t max_rows = row_base >= y_len ? 0 : (rows < y_len - row_base ? rows : y_len - row_base);
  size_t max_cols = cols < x_len ? cols : x_len;
  for (size_t r = 0; r < max_rows; r++) {
    const uint8_t *rw = coded + 4 * r * cols;
    v8f av = {0};
    size_t c = 0;
    for (; c + 8 <= max_cols; c += 8) {
      v8f w = {0};
      for (int k = 0; k < 8; k++) w[k] = rdf32(rw + 4 * (c + k));
      av = vfma(w, vload(x + c), av);
    }
    float sum = vreduce(av);
    for (; c < max_cols; c++) sum += rdf32(rw + 4 * c) * x[c];
    if (acc) y[row_base + r] += sum; else y[row_base + r] = sum;
  }
}

/* chpe_engine.zig:732-751 gemvTilePolymorphic */
void oracle_gemv_tile_polymorphic(const uint8_t *cell, const float *x, size_t x_len, float *y,
                                  size_t y_len, size_t row_base, int acc) {
  switch (cell_qbits(cell)) {
    case 4: gemv_w4(cell, x, x_len, y, y_len, row_base, acc); break;
    case 8: gemv_w8(cell, x, x_len, y, y_len, row_base, acc); break;
    case 16: gemv_f16(cell, x, x_len, y, y_len, row_base, acc); break;
    case 32: gemv_f32(cell, x, x_len, y, y_len, row_base, acc); break;
    default: gemv_w2(cell, x, x_len, y, y_len, row_base, acc); break; /* 2 and fallback */
  }
}

/* gemvCellFlat's tile_weights materialisation (chpe_engine.zig:598-696). */
static void flat_dequant(const uint8_t *cell, size_t wpt, float *tw) {
  const uint8_t *pl = cell + PAYLOAD_OFF;
  const uint8_t *coded = cell + BYTECODE_HEADER_BYTES;
  uint8_t qb = cell_qbits(cell);
  int g128 = (cell_flags(cell) & FLAG_GROUP128_OUTLIERS) != 0;
  if (qb == 4 || qb == 2) {
    if (qb == 4) {
      if (g128) {
        for (size_t g = 0; g < 256; g++) {
          float s = rdf16(pl + 48 + 2 * g);
          for (size_t k = 0; k < 64; k++) {
            uint8_t b = coded[g * 64 + k];
            tw[g * 128 + 2 * k] = ((float)(b & 0x0F) - 8.0f) * s;
            tw[g * 128 + 2 * k + 1] = ((float)((b >> 4) & 0x0F) - 8.0f) * s;
          }
        }
      } else {
        TileDims d = tile_dims(cell);
        for (size_t k = 0; k < wpt / 2; k++) {
          uint8_t b = coded[k];
          tw[2 * k] = ((float)(b & 0x0F) - 8.0f) * d.scale + d.bias;
          tw[2 * k + 1] = ((float)((b >> 4) & 0x0F) - 8.0f) * d.scale + d.bias;
        }
      }
    } else {
      if (g128) {
        for (size_t g = 0; g < 256; g++) {
          float s = rdf16(pl + 48 + 2 * g);
          for (size_t k = 0; k < 32; k++) {
            uint8_t b = coded[g * 32 + k];
            tw[g * 128 + 4 * k + 0] = CODEBOOK_W2[b & 3] * s;
            tw[g * 128 + 4 * k + 1] = CODEBOOK_W2[(b >> 2) & 3] * s;
            tw[g * 128 + 4 * k + 2] = CODEBOOK_W2[(b >> 4) & 3] * s;
            tw[g * 128 + 4 * k + 3] = CODEBOOK_W2[(b >> 6) & 3] * s;
          }
        }
      } else {
        TileDims d = tile_dims(cell);
        for (size_t k = 0; k < wpt / 4; k++) {
          uint8_t b = coded[k];
          tw[4 * k + 0] = CODEBOOK_W2[b & 3] * d.scale + d.bias;
          tw[4 * k + 1] = CODEBOOK_W2[(b >> 2) & 3] * d.scale + d.bias;
          tw[4 * k + 2] = CODEBOOK_W2[(b >> 4) & 3] * d.scale + d.bias;
          tw[4 * k + 3] = CODEBOOK_W2[(b >> 6) & 3] * d.scale + d.bias;
        }
      }
    }
    /* down_aux replace-outliers (:632-646, :679-693) */
    uint16_t n = rd16(pl + 560);
    if (n > 0 && n <= 64) {
      for (size_t m = 0; m < n; m++) {
        uint16_t off = rd16(pl + 560 + 130 + 2 * m);
        if (off < wpt) tw[off] = rdf16(pl + 560 + 2 + 2 * m);
      }
    }
  } else {
    memset(tw, 0, 32768 * sizeof(float));
  }
}

/* Segment dots of one flat tile restricted to rows [r_lo, r_hi). */
static void flat_segments(const float *tw, size_t t, size_t wpt, size_t r_total, size_t c_total,
                          const float *x, float *y, size_t r_lo, size_t r_hi) {
  size_t j = 0;
  size_t gs = t * wpt;
  size_t r = gs / c_total, c = gs % c_total;
  while (j < wpt && r < r_total) {
    size_t seg = wpt - j < c_total - c ? wpt - j : c_total - c;
    if (r >= r_lo && r < r_hi) {
      const float *ws = tw + j, *xs = x + c;
      v8f av = {0};
      size_t k = 0;
      for (; k + 8 <= seg; k += 8) av = vfma(vload(ws + k), vload(xs + k), av);
      float dot = vreduce(av);
      for (; k < seg; k++) dot += ws[k] * xs[k];
      y[r] += dot;
    }
    j += seg;
    c += seg;
    if (c == c_total) { c = 0; r++; }
  }
}

/* chpe_engine.zig:584-729 gemvCellFlat */
void oracle_gemv_cell_flat(const uint8_t *cell, size_t t, size_t wpt, size_t r_total,
                           size_t c_total, const float *x, float *y) {
  float *tw = (float *)malloc(32768 * sizeof(float));
  flat_dequant(cell, wpt, tw);
  flat_segments(tw, t, wpt, r_total, c_total, x, y, 0, (size_t)-1);
  free(tw);
}

size_t oracle_dequant_cell(const uint8_t *cell, int flat, float *out, size_t cap) {
  if (flat) {
    if (cap < 32768) return 0;
    flat_dequant(cell, 32768, out);
    return 32768;
  }
  TileDims d = tile_dims(cell);
  uint8_t qb = cell_qbits(cell);
  const uint8_t *pl = cell + PAYLOAD_OFF;
  const uint8_t *coded = cell + BYTECODE_HEADER_BYTES;
  int g128 = (cell_flags(cell) & FLAG_GROUP128_OUTLIERS) != 0;
  size_t rows = d.rows, cols = d.cols, n = 0;
  size_t tg = cols / 128;
  for (size_t r = 0; r < rows && n < cap; r++) {
    for (size_t c = 0; c < cols && n < cap; c++) {
      float w;
      if (qb == 4) {
        uint8_t b = coded[r * (cols / 2) + c / 2];
        uint8_t nib = (c & 1) ? (b >> 4) & 0xF : b & 0xF;
        if (g128) w = ((float)nib - 8.0f) * rdf16(pl + 48 + 2 * (r * tg + c / 128));
        else w = (float)((int)nib - 8) * d.scale + d.bias;
      } else if (qb == 8) {
        w = (float)(int8_t)coded[r * cols + c];
      } else if (qb == 16) {
        uint16_t h = rd16(coded + 2 * (r * cols + c));
        w = (cell_flags(cell) & FLAG_RAW_FP16) ? f16_to_f32(h) : bf16_to_f32(h);
      } else if (qb == 32) {
        w = rdf32(coded + 4 * (r * cols + c));
      } else {
        uint8_t b = coded[r * (cols / 4) + c / 4];
        float cb = CODEBOOK_W2[(b >> (2 * (c & 3))) & 3];
        if (g128) w = cb * rdf16(pl + 48 + 2 * (r * tg + c / 128));
        else w = cb * d.scale + d.bias;
      }
      out[n++] = w;
    }
  }
  return n;
}

/* ---- gemvLinear (chpe_engine.zig:1396-1489) ------------------------------ */
static int nthreads(const OracleEngine *e) { return e->threads; }

typedef struct {
  OracleEngine *e; size_t tile_start, avail, r_total, c_total; const float *x; float *y;
  size_t nchunks;
} FlatCtx;
static void flat_item(void *p, size_t ch) {
  FlatCtx *c = (FlatCtx *)p;
  const size_t wpt = 32768;
  size_t r_lo = c->r_total * ch / c->nchunks, r_hi = c->r_total * (ch + 1) / c->nchunks;
  if (r_lo >= r_hi) return;
  float *tw = (float *)malloc(32768 * sizeof(float));
  size_t t_lo = (r_lo * c->c_total) / wpt, t_hi = (r_hi * c->c_total + wpt - 1) / wpt;
  if (t_hi > c->avail) t_hi = c->avail;
  for (size_t t = t_lo; t < t_hi; t++) {
    flat_dequant(cell_ptr(c->e, c->tile_start + t), wpt, tw);
    flat_segments(tw, t, wpt, c->r_total, c->c_total, c->x, c->y, r_lo, r_hi);
  }
  free(tw);
}
typedef struct {
  OracleEngine *e; size_t tile_start; const size_t *rb; const float *x; size_t x_len;
  float *y; size_t r_total; int acc;
} RowTileCtx;
static void rowtile_item(void *p, size_t t) {
  RowTileCtx *c = (RowTileCtx *)p;
  oracle_gemv_tile_polymorphic(cell_ptr(c->e, c->tile_start + t), c->x, c->x_len, c->y,
                               c->r_total, c->rb[t], c->acc);
}
typedef struct {
  OracleEngine *e; size_t tile_start, limit, wpt, c_total; const float *x; float *y;
  size_t r_total;
} RawCtx;
static void raw_item(void *p, size_t blk) {
  RawCtx *c = (RawCtx *)p;
  for (size_t r = blk * 64; r < (blk + 1) * 64 && r < c->r_total; r++) {
    size_t f = r * c->c_total, end = f + c->c_total;
    if (end > c->limit) end = c->limit;
    while (f < end) {
      size_t t = f / c->wpt, j = f % c->wpt;
      size_t seg = c->wpt - j < end - f ? c->wpt - j : end - f;
      c->y[r] += dot_segment(c->e, tile_code_ptr(c->e, c->tile_start + t), j, seg,
                             c->x + (f - r * c->c_total));
      f += seg;
    }
  }
}

void oracle_gemv_linear(OracleEngine *e, size_t tile_start, size_t num_tiles, const float *x,
                        size_t x_len, float *y, size_t r_total, size_t c_total, int acc,
                        int64_t bias_tile) {
  if (!acc) memset(y, 0, r_total * 4);
  if (!e->archive_valid || tile_start >= e->record_count) {
    if (!acc)
      for (size_t r = 0; r < r_total; r++) y[r] = 0.01f * (float)((int)(r % 13) - 6);
    return;
  }
  size_t avail = num_tiles < e->record_count - tile_start ? num_tiles : e->record_count - tile_start;
  int nt = nthreads(e);
  if (!e->is_raw) {
    if (c_total > 2048) {
      FlatCtx fc = {e, tile_start, avail, r_total, c_total, x, y, (size_t)nt * 4};
      par_for(fc.nchunks, nt, flat_item, &fc);
    } else {
      /* row_base prefix with the reference's break conditions */
      size_t *rb = (size_t *)malloc((avail + 1) * sizeof(size_t));
      size_t ncell = 0, row_base = 0;
      for (size_t t = 0; t < avail; t++) {
        if (row_base >= r_total) break;
        TileDims d = tile_dims(cell_ptr(e, tile_start + t));
        if (d.rows == 0) break;
        rb[ncell++] = row_base;
        row_base += d.rows;
      }
      RowTileCtx rc = {e, tile_start, rb, x, x_len, y, r_total, acc};
      par_for(ncell, nt, rowtile_item, &rc);
      free(rb);
    }
    if (bias_tile >= 0 && (size_t)bias_tile < e->record_count) {
      oracle_unpack_bias(e, (size_t)bias_tile, e->bias_buf, r_total);
      for (size_t r = 0; r < r_total; r++) y[r] += e->bias_buf[r];
    }
    return;
  }
  size_t wpt = e->wpt;
  /* Raw: each row's segments in tile order; rows are independent. */
  size_t limit = avail * wpt;
  RawCtx wc = {e, tile_start, limit, wpt, c_total, x, y, r_total};
  par_for((r_total + 63) / 64, nt, raw_item, &wc);
  if (bias_tile >= 0 && (size_t)bias_tile < e->record_count) {
    oracle_unpack_bias(e, (size_t)bias_tile, e->bias_buf, r_total);
    for (size_t r = 0; r < r_total; r++) y[r] += e->bias_buf[r];
  }
}

/* ---- embedding (chpe_engine.zig:1288-1394, 1491-1552) -------------------- */
void oracle_unpack_embed_row_cell(const uint8_t *cell, size_t row, float *out, size_t D) {
  const uint8_t *pl = cell + PAYLOAD_OFF;
  const uint8_t *coded = cell + BYTECODE_HEADER_BYTES;
  uint8_t qb = cell_qbits(cell);
  uint64_t fl = cell_flags(cell);
  if (qb == 8) {
    if (row >= 8) return; /* Q3: output left unchanged */
    size_t ng = D / 128;
    for (size_t g = 0; g < ng; g++) {
      float s = rdf16(pl + 48 + 2 * (row * ng + g));
      for (size_t j = 0; j < 128; j++)
        out[g * 128 + j] = (float)(int8_t)coded[row * D + g * 128 + j] * s;
    }
    return;
  }
  if (qb == 2) {
    if (row >= 16) return;
    size_t ng = D / 128;
    const uint8_t *rbytes = coded + row * (D / 4);
    for (size_t g = 0; g < ng; g++) {
      float s = rdf16(pl + 48 + 2 * (row * ng + g));
      for (size_t j = 0; j < 32; j++) {
        uint8_t b = rbytes[g * 32 + j];
        out[g * 128 + 4 * j + 0] = CODEBOOK_W2[b & 3] * s;
        out[g * 128 + 4 * j + 1] = CODEBOOK_W2[(b >> 2) & 3] * s;
        out[g * 128 + 4 * j + 2] = CODEBOOK_W2[(b >> 4) & 3] * s;
        out[g * 128 + 4 * j + 3] = CODEBOOK_W2[(b >> 6) & 3] * s;
      }
    }
    if (fl & FLAG_GROUP128_OUTLIERS)
      for (int k = 0; k < 8; k++) {
        uint16_t col = rd16(pl + 816 + 2 * k);
        if (col < D) out[col] = rdf16(pl + 560 + 2 * (row * 8 + k));
      }
    return;
  }
  if ((fl & FLAG_GROUP128_OUTLIERS) || qb == 4) {
    if (row >= 16) return;
    size_t ng = D / 128;
    const uint8_t *rbytes = coded + row * (D / 2);
    for (size_t g = 0; g < ng; g++) {
      float s = rdf16(pl + 48 + 2 * (row * ng + g));
      for (size_t j = 0; j < 64; j++) {
        uint8_t b = rbytes[g * 64 + j];
        out[g * 128 + 2 * j] = ((float)(b & 0x0F) - 8.0f) * s;
        out[g * 128 + 2 * j + 1] = ((float)((b >> 4) & 0x0F) - 8.0f) * s;
      }
    }
    if (fl & FLAG_GROUP128_OUTLIERS)
      for (int k = 0; k < 8; k++) {
        uint16_t col = rd16(pl + 816 + 2 * k);
        if (col < D) out[col] = rdf16(pl + 560 + 2 * (row * 8 + k));
      }
    return;
  }
  TileDims d = tile_dims(cell);
  size_t bo = row * (D / 2);
  for (size_t j = 0; j < D / 2; j++) {
    uint8_t b = coded[bo + j];
    out[2 * j] = ((float)(b & 0x0F) - 8.0f) * d.scale + d.bias;
    out[2 * j + 1] = ((float)((b >> 4) & 0x0F) - 8.0f) * d.scale + d.bias;
  }
}

static void embed_fallback(uint32_t tok, float *out, size_t D) {
  for (size_t i = 0; i < D; i++) out[i] = 0.05f * (float)((int)((i + tok) % 17) - 8);
}

void oracle_unpack_embed_row(const OracleEngine *e, uint32_t tok, float *out) {
  size_t D = e->arch.D;
  if (!e->archive_valid || e->record_count == 0) { embed_fallback(tok, out, D); return; }
  if (e->is_raw_fp16) {
    size_t rpt = 8192 / D;
    if (rpt > 0 && tok / rpt < e->record_count) {
      const uint8_t *row = tile_code_ptr(e, tok / rpt) + 2 * (tok % rpt) * D;
      for (size_t i = 0; i < D; i++) out[i] = rdf16(row + 2 * i);
      return;
    }
  } else if (e->is_raw) {
    if (e->quant_bits == 8) {
      size_t rpt = 16384 / D;
      if (rpt > 0 && tok / rpt < e->record_count) {
        const int8_t *row = (const int8_t *)tile_code_ptr(e, tok / rpt) + (tok % rpt) * D;
        for (size_t i = 0; i < D; i++) out[i] = (float)row[i] * INT8_RAW_SCALE;
        return;
      }
    } else {
      size_t rpt = 8192 / D;
      if (rpt > 0 && tok / rpt < e->record_count) {
        const uint8_t *row = tile_code_ptr(e, tok / rpt) + 2 * (tok % rpt) * D;
        for (size_t i = 0; i < D; i++) out[i] = bf16_to_f32(rd16(row + 2 * i));
        return;
      }
    }
  } else {
    size_t ti = tok / 16, ri = tok % 16; /* Q2: tok/16 for every D */
    if (ti < e->record_count) {
      oracle_unpack_embed_row_cell(cell_ptr(e, ti), ri, out, D);
      return;
    }
  }
  embed_fallback(tok, out, D);
}

/* ---- LM head (chpe_engine.zig:1554-1660) -------------------------------- */
static float dot8(const float *a, const float *b, size_t n) {
  v8f av = {0};
  size_t k = 0;
  for (; k + 8 <= n; k += 8) av = vfma(vload(a + k), vload(b + k), av);
  float s = vreduce(av);
  for (; k < n; k++) s += a[k] * b[k];
  return s;
}

typedef struct { OracleEngine *e; const size_t *vstart; const float *xn; float *logits; int nt; } TiedCellCtx;
static void tied_cell_item(void *p, size_t t) {
  TiedCellCtx *c = (TiedCellCtx *)p;
  OracleEngine *e = c->e;
  size_t D = e->arch.D, V = e->arch.V;
  float *row = (float *)malloc(8192 * sizeof(float));
  if (c->nt == 1) memcpy(row, e->lm_row, 8192 * 4);
  const uint8_t *cp = cell_ptr(e, t);
  TileDims d = tile_dims(cp);
  size_t rpt = d.rows == 0 ? 16 : d.rows;
  for (size_t r = 0; r < rpt; r++) {
    size_t vv = c->vstart[t] + r;
    if (vv >= V) break;
    oracle_unpack_embed_row_cell(cp, r, row, D);
    c->logits[vv] = dot8(c->xn, row, D);
  }
  if (c->nt == 1) memcpy(e->lm_row, row, 8192 * 4);
  free(row);
}
typedef struct { OracleEngine *e; const float *xn; float *logits; size_t rpt; } TiedRawCtx;
static void tied_raw_item(void *p, size_t t);

void oracle_compute_lm_head(OracleEngine *e, const float *xn, float *logits) {
  size_t D = e->arch.D, V = e->arch.V;
  if (!e->archive_valid || e->record_count == 0) {
    for (size_t v = 0; v < V; v++) logits[v] = 0.001f * (float)((int)(v % 13) - 6);
    return;
  }
  int64_t lhs = -1;
  size_t lht = 0;
  if (D == 8192) { lhs = 2181137; lht = 38016; }
  else if (D == 4096) { lhs = 484601; lht = 62080; }
  if (lhs >= 0 && (size_t)lhs < e->record_count) {
    oracle_gemv_linear(e, (size_t)lhs, lht, xn, D, logits, V, D, 0, -1);
    return;
  }
  int nt = nthreads(e);
  if (!e->is_raw) {
    /* Tied embeddings in a cell archive.  Rows beyond a format's decodable
     * range leave the scratch row stale (Q3); such archives run serially so
     * the stale contents match. */
    size_t ncell = 0, v = 0, stale = 0;
    size_t *vstart = (size_t *)malloc((e->record_count + 1) * sizeof(size_t));
    for (size_t t = 0; t < e->record_count && v < V; t++) {
      const uint8_t *c = cell_ptr(e, t);
      TileDims d = tile_dims(c);
      size_t rpt = d.rows == 0 ? 16 : d.rows;
      uint8_t qb = cell_qbits(c);
      if ((qb == 8 && rpt > 8) || rpt > 16) stale = 1;
      vstart[ncell++] = v;
      v += rpt;
    }
    if (stale) nt = 1;
    TiedCellCtx tc = {e, vstart, xn, logits, nt};
    par_for(ncell, nt, tied_cell_item, &tc);
    free(vstart);
    return;
  }
  size_t rpt = 8192 / D;
  if (rpt == 0) rpt = 1;
  size_t tiles = (V + rpt - 1) / rpt;
  if (tiles > e->record_count) tiles = e->record_count;
  TiedRawCtx rc = {e, xn, logits, rpt};
  par_for(tiles, nt, tied_raw_item, &rc);
}

static void tied_raw_item(void *p, size_t t) {
  TiedRawCtx *c = (TiedRawCtx *)p;
  OracleEngine *e = c->e;
  size_t D = e->arch.D, V = e->arch.V, rpt = c->rpt;
  const float *xn = c->xn;
  float *logits = c->logits;
  {
    const uint8_t *tp = tile_code_ptr(e, t);
    for (size_t r = 0; r < rpt; r++) {
      size_t v = t * rpt + r;
      if (v >= V) break;
      const uint8_t *row = tp + 2 * r * D;
      v8f av = {0};
      size_t k = 0;
      for (; k + 8 <= D; k += 8) {
        v8f w = {0};
        for (int i = 0; i < 8; i++)
          w[i] = e->is_raw_fp16 ? rdf16(row + 2 * (k + i)) : bf16_to_f32(rd16(row + 2 * (k + i)));
        av = vfma(w, vload(xn + k), av);
      }
      float s = vreduce(av);
      for (; k < D; k++)
        s += (e->is_raw_fp16 ? rdf16(row + 2 * k) : bf16_to_f32(rd16(row + 2 * k))) * xn[k];
      logits[v] = s;
    }
  }
}

/* ---- primitives (chpe_engine.zig:159-216) ------------------------------- */
float oracle_silu(float z) { return z / (1.0f + expf(-z)); }

void oracle_rms_norm(const float *x, const float *g, float *y, size_t n, float eps) {
  v8f av = {0};
  size_t i = 0;
  for (; i + 8 <= n; i += 8) {
    v8f v = vload(x + i);
    av += v * v;
  }
  float ss = vreduce(av);
  for (; i < n; i++) ss += x[i] * x[i];
  float mean = ss / (float)n;
  float inv = 1.0f / sqrtf(mean + eps);
  for (i = 0; i < n; i++) y[i] = x[i] * inv * g[i];
}

void oracle_apply_rope(float *vec, size_t pos, size_t nh, size_t hd, float theta) {
  float pf = (float)pos;
  for (size_t h = 0; h < nh; h++) {
    size_t hb = h * hd;
    for (size_t i = 0; i < hd / 2; i++) {
      float fe = 2.0f * (float)i / (float)hd;
      float freq = 1.0f / powf(theta, fe);
      float th = pf * freq;
      float c = cosf(th), s = sinf(th);
      float x0 = vec[hb + i], x1 = vec[hb + i + hd / 2];
      vec[hb + i] = x0 * c - x1 * s;
      vec[hb + i + hd / 2] = x0 * s + x1 * c;
    }
  }
}

static void attention_head(const float *q, const float *kc, const float *vc, size_t pos,
                           size_t kvd, size_t kv_h, size_t hd, float scale, float *scores,
                           float *out) {
  float mx = -1e30f;
  for (size_t t = 0; t <= pos; t++) {
    const float *ks = kc + t * kvd + kv_h * hd;
    float dot = 0.0f;
    for (size_t d = 0; d < hd; d++) dot += q[d] * ks[d];
    float s = dot * scale;
    scores[t] = s;
    if (s > mx) mx = s;
  }
  float se = 0.0f;
  for (size_t t = 0; t <= pos; t++) {
    float ev = expf(scores[t] - mx);
    scores[t] = ev;
    se += ev;
  }
  float inv = 1.0f / se;
  for (size_t d = 0; d < hd; d++) out[d] = 0.0f;
  for (size_t t = 0; t <= pos; t++) {
    float a = scores[t] * inv;
    const float *vs = vc + t * kvd + kv_h * hd;
    for (size_t d = 0; d < hd; d++) out[d] += a * vs[d];
  }
}

void oracle_gqa_attention(const float *q, const float *kc, const float *vc, size_t pos,
                          size_t H, size_t KV, size_t hd, float *out) {
  float scale = 1.0f / sqrtf((float)hd);
  float *scores = (float *)malloc((pos + 1) * sizeof(float));
  for (size_t h = 0; h < H; h++)
    attention_head(q + h * hd, kc, vc, pos, KV * hd, h / (H / KV), hd, scale, scores, out + h * hd);
  free(scores);
}

/* ---- forwardDecode (chpe_engine.zig:1663-1803) --------------------------- */
static uint64_t now_ns(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

typedef struct {
  const float *q, *kc, *vc; size_t pos, kvd, gqa, hd; float scale; float *out;
} AttnCtx;
static void attn_item(void *p, size_t qh) {
  AttnCtx *c = (AttnCtx *)p;
  float *scores = (float *)malloc((c->pos + 1) * sizeof(float));
  attention_head(c->q + qh * c->hd, c->kc, c->vc, c->pos, c->kvd, qh / c->gqa, c->hd, c->scale,
                 scores, c->out + qh * c->hd);
  free(scores);
}

void oracle_forward_decode(OracleEngine *e, uint32_t tok, size_t pos, OracleForwardResult *res) {
  uint64_t t0 = now_ns();
  const Arch *A = &e->arch;
  oracle_unpack_embed_row(e, tok, e->hidden);
  size_t gqa = A->H / A->KV, kvd = A->KV * A->HD;
  int nt = nthreads(e);
  for (size_t l = 0; l < A->L; l++) {
    OracleLayerInfo li;
    oracle_layer_info(e, l, &li);
    oracle_unpack_norm(e, (size_t)li.input_norm, e->norm_gamma, A->D);
    oracle_rms_norm(e->hidden, e->norm_gamma, e->norm_buf, A->D, A->eps);
    oracle_gemv_linear(e, li.q_proj, li.q_tiles, e->norm_buf, A->D, e->q, A->H * A->HD, A->D, 0, li.q_bias);
    oracle_gemv_linear(e, li.k_proj, li.k_tiles, e->norm_buf, A->D, e->k, kvd, A->D, 0, li.k_bias);
    oracle_gemv_linear(e, li.v_proj, li.v_tiles, e->norm_buf, A->D, e->v, kvd, A->D, 0, li.v_bias);
    oracle_apply_rope(e->q, pos, A->H, A->HD, A->theta);
    oracle_apply_rope(e->k, pos, A->KV, A->HD, A->theta);
    float *kc = e->k_cache + l * e->max_seq * kvd, *vc = e->v_cache + l * e->max_seq * kvd;
    if (pos * kvd + kvd <= e->max_seq * kvd) {
      memcpy(kc + pos * kvd, e->k, kvd * 4);
      memcpy(vc + pos * kvd, e->v, kvd * 4);
      if (e->kv_fp16)
        for (size_t i = 0; i < kvd; i++) {
          kc[pos * kvd + i] = round_f16(kc[pos * kvd + i]);
          vc[pos * kvd + i] = round_f16(vc[pos * kvd + i]);
        }
    }
    float scale = 1.0f / sqrtf((float)A->HD);
    AttnCtx ac = {e->q, kc, vc, pos, kvd, gqa, A->HD, scale, e->attn_out};
    par_for(A->H, nt, attn_item, &ac);
    oracle_gemv_linear(e, li.o_proj, li.o_tiles, e->attn_out, A->D, e->hidden, A->D, A->D, 1, -1);
    oracle_unpack_norm(e, (size_t)li.post_norm, e->norm_gamma, A->D);
    oracle_rms_norm(e->hidden, e->norm_gamma, e->norm_buf, A->D, A->eps);
    oracle_gemv_linear(e, li.gate_proj, li.gate_tiles, e->norm_buf, A->D, e->gate, A->F, A->D, 0, -1);
    oracle_gemv_linear(e, li.up_proj, li.up_tiles, e->norm_buf, A->D, e->up, A->F, A->D, 0, -1);
    for (size_t i = 0; i < A->F; i++) e->mlp[i] = oracle_silu(e->gate[i]) * e->up[i];
    oracle_gemv_linear(e, li.down_proj, li.down_tiles, e->mlp, A->F, e->hidden, A->D, A->F, 1, -1);
    /* Q5: debug-norm block with early exit (:1753-1764) */
    if (l < 3 || (l >= 8 && l <= 16) || !isfinite(e->hidden[0])) {
      float hs = 0.0f;
      for (size_t i = 0; i < A->D; i++) hs += e->hidden[i] * e->hidden[i];
      if (!isfinite(hs)) break;
    }
  }
  oracle_unpack_norm(e, (size_t)oracle_final_norm_index(e), e->norm_gamma, A->D);
  oracle_rms_norm(e->hidden, e->norm_gamma, e->norm_buf, A->D, A->eps);
  oracle_compute_lm_head(e, e->norm_buf, e->logits);
  float mx = -1e30f;
  uint32_t am = 0;
  int fin = 1;
  for (size_t v = 0; v < A->V; v++) {
    float val = e->logits[v];
    if (!isfinite(val)) fin = 0;
    if (val > mx) { mx = val; am = (uint32_t)v; }
  }
  float hs = 0.0f;
  for (size_t i = 0; i < A->D; i++) hs += e->hidden[i] * e->hidden[i];
  res->argmax_token = am;
  res->max_logit = mx;
  res->token0_logit = e->logits[0];
  res->elapsed_ns = now_ns() - t0;
  res->hidden_norm = sqrtf(hs);
  res->all_finite = fin;
}


/* ---- archive converters (weight_archive.zig:617-776) -------------------- */

/* f32 -> f16 as Zig's @floatCast rounds it (nearest, ties to even); a NaN
 * keeps its sign, gets the quiet bit and the top payload bits. */
static uint16_t f32_to_f16_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if (((u >> 23) & 0xFF) == 0xFF && (u & 0x7FFFFF))
    return (uint16_t)(((u >> 16) & 0x8000) | 0x7E00 | ((u & 0x7FFFFF) >> 13));
  _Float16 h = (_Float16)f;
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}

/* Output header (4096 bytes) of a conversion (`mode` 0 dense, 1 raw, 2 raw FP16). */
void oracle_convert_header(const uint8_t *src, int mode, uint8_t *out) {
  memset(out, 0, 4096);
  memcpy(out, src, 64);
  uint64_t v;
  if (mode == 0) {
    v = CELL_BYTES; memcpy(out + 32, &v, 8);
    v = 0; memcpy(out + 48, &v, 8);
  } else {
    v = TILE_CODE_BYTES; memcpy(out + 32, &v, 8); memcpy(out + 40, &v, 8);
    v = 0; memcpy(out + 48, &v, 8);
    if (mode == 2) { v = rd64(src + 56) | FLAG_RAW_FP16; memcpy(out + 56, &v, 8); }
  }
}

/* Output record `i` of a conversion: a 17408-byte cell (mode 0) or a 16384-byte
 * tile (modes 1, 2).  Returns the bytes written. */
size_t oracle_convert_record(const uint8_t *src, int mode, size_t i, uint8_t *out) {
  uint64_t count = rd64(src + 16), rb = rd64(src + 32), pb = rd64(src + 48);
  int raw = rb == TILE_CODE_BYTES && pb == 0, dense = pb == 0;
  const uint8_t *cell = src + 4096 + i * rb + pb; /* getCellDirect */
  const uint8_t *tile = raw ? src + 4096 + i * TILE_CODE_BYTES
                        : dense ? src + 4096 + i * CELL_BYTES + 64
                                : src + 4096 + i * RECORD_BYTES + PREFETCH_LABEL_BYTES + 64;
  if (mode == 0) { memcpy(out, cell, CELL_BYTES); return CELL_BYTES; }
  if (mode == 1) { memcpy(out, tile, TILE_CODE_BYTES); return TILE_CODE_BYTES; }
  int one_d = 0, decided = 0;
  if (count == 376853) {
    if (i == 376852) { one_d = 1; decided = 1; }
    else if (i < 37984) { one_d = 0; decided = 1; }
    else {
      size_t rel = (i - 37984) % 9413;
      if (rel == 0 || rel == 513 || rel == 578 || rel == 643 || rel == 1156) { one_d = 1; decided = 1; }
    }
  }
  if (!decided && !raw) one_d = cell[PAYLOAD_OFF + 20] == 32;
  if (one_d) { memcpy(out, tile, TILE_CODE_BYTES); return TILE_CODE_BYTES; }
  for (size_t k = 0; k < 8192; k++) {
    uint32_t b = (uint32_t)rd16(tile + 2 * k) << 16;
    float f;
    memcpy(&f, &b, 4);
    uint16_t h = f32_to_f16_bits(f);
    memcpy(out + 2 * k, &h, 2);
  }
  return TILE_CODE_BYTES;
}
