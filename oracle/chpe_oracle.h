/*
 * chpe_oracle.h -- TEST INFRASTRUCTURE, NOT PART OF THE PRODUCT.
 *
 * CPU restatement of the reference engine's per-token decode path
 * (src/chpe_engine.zig, src/weight_archive.zig, src/chpe_c_api.zig of
 * chpe-qwen-engine).  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load this library, and only as the checker.  The product
 * (libchpe.so) never links it.
 *
 * Parity status: the reference is Zig 0.17-dev and no Zig toolchain exists
 * in this build environment, so the reference itself cannot be run.  This
 * restatement is pinned by the known-answer tests found in the reference's
 * own unit tests (RoPE, SiLU, SwiGLU, RMSNorm, attention pass-through, the
 * 2/4/8-bit cell GEMV tests, the zero-byte mock archive forward pass, the
 * tensor-map index tests, the archive layout, create/reopen and corruption
 * tests); see tests/test_oracle_kats.py.  Beyond those constant cases, three
 * independent float64 restatements check it on random hand-built archives:
 * every tile format of gemvLinear (tests/test_oracle_formats_cpu.py), the
 * embedding lookup, tied LM head and norm/bias unpacking
 * (tests/test_oracle_embed_cpu.py), and the composition of forwardDecode
 * around its weight readers (tests/test_oracle_forward_cpu.py).
 *
 * Numerics follow the reference: f32 everywhere, 8-lane accumulators where
 * the reference uses @Vector(8, f32), fmaf() where it uses @mulAdd, ordered
 * lane reductions for @reduce(.Add) (Zig keeps float associativity outside
 * Optimized float mode), no contraction of a*b+c elsewhere
 * (compile with -ffp-contract=off).
 */
#ifndef CHPE_ORACLE_H
#define CHPE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Architecture ids (chpe_engine.zig:110-145). */
enum { ORACLE_ARCH_3B = 0, ORACLE_ARCH_9B = 1, ORACLE_ARCH_72B = 2 };

/* WeightArchiveError codes (weight_archive.zig:128-139); 0 = ok. */
enum {
  ORACLE_OK = 0,
  ORACLE_ERR_INVALID_MAGIC = 1,
  ORACLE_ERR_UNSUPPORTED_VERSION = 2,
  ORACLE_ERR_BAD_GEOMETRY = 3,
  ORACLE_ERR_TRUNCATED = 4,
  ORACLE_ERR_FILE_TOO_SMALL = 6,
  ORACLE_ERR_MISALIGNED_HEADER = 10,
};

typedef struct {
  uint32_t magic, version;
  uint64_t header_bytes, record_count, tile_count, record_bytes, cell_bytes,
      prefetch_bytes, flags;
} OracleHeader;

typedef struct {
  uint32_t argmax_token;
  float max_logit;
  float token0_logit;
  uint64_t elapsed_ns;
  float hidden_norm;
  int32_t all_finite;
} OracleForwardResult;

typedef struct {
  int64_t input_norm, q_proj, q_tiles, q_bias, k_proj, k_tiles, k_bias, v_proj,
      v_tiles, v_bias, o_proj, o_tiles, post_norm, gate_proj, gate_tiles,
      up_proj, up_tiles, down_proj, down_tiles; /* bias = -1 when absent */
} OracleLayerInfo;

typedef struct OracleEngine OracleEngine;

/* weight_archive.zig:152 WeightArchive.validate */
int oracle_validate(const uint8_t *bytes, size_t len, OracleHeader *out);

/* chpe_engine.zig:854 CHPEEngine.init (archive bytes are borrowed). */
OracleEngine *oracle_engine_new(const uint8_t *archive, size_t len, int arch,
                                size_t max_seq_len);
void oracle_engine_free(OracleEngine *e);
/* Worker threads for the GEMV / LM head / attention loops.  Results do not
 * depend on the thread count: every output element keeps the reference's
 * accumulation order. */
void oracle_set_threads(OracleEngine *e, int n);
/* Test option, not reference behaviour (the reference caches f32): round each
 * cached K/V row to FP16 when a step stores it, as a half-precision KV cache
 * does, so a comparison can separate the cache's rounding from the rest. */
void oracle_set_kv_fp16(OracleEngine *e, int on);

/* Test harness (no reference function): K/V rows [n][kv_heads*head_dim] at
 * positions pos0.. of one layer's cache, for prefilled long contexts.  0, or
 * -1 when they do not fit. */
int oracle_kv_load(OracleEngine *e, size_t layer, size_t pos0, size_t n, const float *k,
                   const float *v);

/* chpe_engine.zig:1663 forwardDecode */
void oracle_forward_decode(OracleEngine *e, uint32_t token, size_t pos,
                           OracleForwardResult *out);
const float *oracle_logits(const OracleEngine *e);
const float *oracle_hidden(const OracleEngine *e);
size_t oracle_vocab(const OracleEngine *e);
size_t oracle_hidden_dim(const OracleEngine *e);
/* engine facts after init sniffing: is_raw, is_raw_fp16, is_dense, quant_bits,
 * weights_per_tile, archive_valid, record_count */
void oracle_engine_facts(const OracleEngine *e, int64_t out[7]);
void oracle_layer_info(const OracleEngine *e, size_t l, OracleLayerInfo *out);
int64_t oracle_final_norm_index(const OracleEngine *e);

/* chpe_engine.zig:1396 gemvLinear; bias_tile < 0 means none. */
void oracle_gemv_linear(OracleEngine *e, size_t tile_start, size_t num_tiles,
                        const float *x, size_t x_len, float *y, size_t r_total,
                        size_t c_total, int accumulate, int64_t bias_tile);
/* chpe_engine.zig:1144 unpackNorm / :1172 unpackBias / :1491 unpackEmbedRow */
void oracle_unpack_norm(const OracleEngine *e, size_t tile, float *out, size_t n);
void oracle_unpack_bias(const OracleEngine *e, size_t tile, float *out, size_t n);
void oracle_unpack_embed_row(const OracleEngine *e, uint32_t token, float *out);
/* chpe_engine.zig:1554 computeLmHead over a caller-supplied normed hidden */
void oracle_compute_lm_head(OracleEngine *e, const float *normed, float *logits);

/* Single-cell kernels (chpe_engine.zig:223-751); `cell` points at a 17408-byte
 * Cell (64 B header, 16384 B codes, 960 B payload). */
void oracle_gemv_tile_polymorphic(const uint8_t *cell, const float *x, size_t x_len,
                                  float *y, size_t y_len, size_t row_base,
                                  int accumulate);
void oracle_gemv_cell_flat(const uint8_t *cell, size_t t, size_t wpt,
                           size_t r_total, size_t c_total, const float *x,
                           float *y);
/* Dequantised f32 weights of one cell exactly as the reference materialises
 * them: flat cells (gemvCellFlat's tile_weights, 32768 values) when flat != 0,
 * otherwise the row-tiled weight w[r][c] for r < rows, c < cols (scale/bias
 * affine forms; group-scaled forms give q*scale).  Returns the count written. */
size_t oracle_dequant_cell(const uint8_t *cell, int flat, float *out, size_t cap);
/* unpackEmbedRowCell (chpe_engine.zig:1288) for one cell row. */
void oracle_unpack_embed_row_cell(const uint8_t *cell, size_t row, float *out,
                                  size_t d);

/* Primitive ops (chpe_engine.zig:159-216). */
float oracle_silu(float z);
void oracle_rms_norm(const float *x, const float *gamma, float *y, size_t n,
                     float eps);
void oracle_apply_rope(float *vec, size_t pos, size_t num_heads, size_t head_dim,
                       float theta);
/* One GQA attention step over a caller KV (the forwardDecode inner loops,
 * chpe_engine.zig:1699-1734): k/v are [t][kv_heads*head_dim]. */
void oracle_gqa_attention(const float *q, const float *k_cache,
                          const float *v_cache, size_t pos, size_t num_heads,
                          size_t num_kv_heads, size_t head_dim, float *out);

/* Mock-archive path used by the reference's own engine tests
 * (chpe_engine.zig:1893-1933): the engine over `len` zero bytes. */

/* One decode step of a Qwen3.5 Gated DeltaNet layer after its input
 * projections (deltanet_oracle.c; no reference function exists). */
void oracle_deltanet_step(const float *mixed_qkv, const float *z, const float *a, const float *b,
                          const float *conv_w, float *conv_hist, uint32_t t, const float *a_log,
                          const float *dt_bias, const float *norm_w, float *state, float *out,
                          uint32_t nk, uint32_t nv, uint32_t dk, uint32_t dv, float eps);

/* Archive converters (weight_archive.zig:617-776): the output header of a
 * conversion (mode 0 dense, 1 raw, 2 raw FP16; 4096 bytes) and output record
 * i (returns its size).  `src` is a validated archive. */
void oracle_convert_header(const uint8_t *src, int mode, uint8_t *out);
size_t oracle_convert_record(const uint8_t *src, int mode, size_t i, uint8_t *out);

/* Tensor maps (as the reference tables give them). */
void oracle_map_3b_cell_layer(size_t l, int64_t out[12]);
void oracle_map_72b_layer(size_t l, int64_t out[12]);

#ifdef __cplusplus
}
#endif
#endif
