/* chpe_maps.h -- archive geometry, model presets and tensor maps.
 *
 * Restates the layout facts of chpe-qwen-engine that any reader of a .chpe
 * archive must agree on bit for bit:
 *   geometry.zig:24-62, 243-270          cell / record byte layout
 *   weight_archive.zig:20-34, 53-112     header, tile metadata, flags
 *   chpe_engine.zig:96-155               model presets, TileDims
 *   qwen3b_geometry.zig:48-79            3B raw archive offsets
 *   qwen3b_tensor_map.zig:27-531         3B cell archive table (data)
 *   qwen35_tensor_map.zig:53-1015        9B archive (formula, checked vs table)
 *   qwen72b_tensor_map.zig:24-87         72B archive
 *   chpe_engine.zig:1035-1142            getLayerInfo / getFinalNormIndex
 */
#ifndef CHPE_MAPS_H
#define CHPE_MAPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CHPE_HEADER_BYTES 4096u
#define CHPE_CELL_BYTES 17408u
#define CHPE_RECORD_BYTES 20480u
#define CHPE_PREFETCH_BYTES 3072u
#define CHPE_CELL_HEADER_BYTES 64u
#define CHPE_TILE_CODE_BYTES 16384u
#define CHPE_PAYLOAD_OFF 16448u /* payload offset inside a cell */
#define CHPE_PAYLOAD_FROM_CODES 16384u /* payload offset from the code area */
#define CHPE_ARCHIVE_MAGIC 0x57415243u /* "WARC" */
#define CHPE_CHPE_MAGIC 0x45504843u /* "CHPE" */
#define CHPE_FLAG_GROUP128_OUTLIERS 0x01u
#define CHPE_FLAG_HYBRID 0x02u
#define CHPE_FLAG_RAW_FP16 0x04u
#define CHPE_FLAG_RAW_INT8 0x08u
#define CHPE_INT8_RAW_SCALE 0.00373708f

enum { CHPE_ARCH_3B = 0, CHPE_ARCH_9B = 1, CHPE_ARCH_72B = 2 };

typedef struct {
  const char *name;
  uint32_t D, F, L, H, KV, HD, V;
  int hybrid;
  float theta, eps;
} ChpeArch;

typedef struct {
  int64_t input_norm, q_proj, q_tiles, q_bias, k_proj, k_tiles, k_bias, v_proj,
      v_tiles, v_bias, o_proj, o_tiles, post_norm, gate_proj, gate_tiles, up_proj,
      up_tiles, down_proj, down_tiles; /* a bias is -1 when absent */
} ChpeLayerInfo;

/* Extra tensors of a 9B layer (qwen35_tensor_map.zig LayerTensorMap); -1 when
 * the layer kind has none. */
typedef struct {
  int is_full;
  int64_t in_proj_qkv, in_proj_z, in_proj_a, in_proj_b, conv1d, a_log, dt_bias,
      linear_norm, out_proj, q_norm, k_norm;
} Chpe9bExtra;

/* One tensor-parallel rank's slices (rows of every projection): query heads
 * [h0, h0+hq), kv heads [kv0, kv0+kvl), hidden rows [d0, d0+dl) of O and
 * down, FFN rows [f0, f0+fl) of gate/up, vocabulary rows [v0, v0+vl). */
typedef struct {
  uint32_t hq, h0, kv0, kvl, dl, d0, fl, f0, vl, v0;
} ChpeTpSlice;

const ChpeArch *chpe_arch_preset(int arch);
/* 0, or -1 when the architecture does not split over `world` ranks. */
int chpe_tp_slice_of(int arch, int rank, int world, ChpeTpSlice *out);
/* The archive tiles a tensor-parallel rank's kernels read, merged into
 * disjoint runs [lo, hi) in ascending order (runs[2i], runs[2i+1]; at most
 * `cap` written).  wpt = weights per tile of the archive's projections,
 * record_count bounds every run.  Returns the number of runs, or -1 when the
 * architecture does not split over `world`. */
int64_t chpe_tp_tile_runs(int arch, int is_raw, uint64_t wpt, uint64_t record_count, int rank,
                          int world, uint64_t *runs, size_t cap);
void chpe_layer_info(int arch, int is_raw, size_t l, ChpeLayerInfo *out);
void chpe_9b_extra(size_t l, Chpe9bExtra *out);
int64_t chpe_final_norm_index(int arch, int is_raw);
/* Untied LM head span (chpe_engine.zig:1565-1580); start = -1 when tied. */
void chpe_lm_head_span(int arch, int64_t *start, int64_t *tiles);
/* Total records of the reference archive for (arch, raw?) -- 3B raw 376853,
 * 3B cell 94349, 9B 546681, 72B 2219153. */
int64_t chpe_total_records(int arch, int is_raw);

#ifdef __cplusplus
}
#endif
#endif
