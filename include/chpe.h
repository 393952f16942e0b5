/*
 * chpe.h -- C ABI of the B200 decode engine (libchpe.so).
 *
 * The first block is exactly the FFI surface of chpe-qwen-engine's
 * src/chpe_c_api.zig: same names, argument meaning, sentinels and
 * ownership.  Each declaration cites the reference interface it replaces.
 * The second block adds entry points the reference lacks; the third holds
 * test probes used by the parity suite.
 *
 * Threading: a context is not thread-safe (one context per thread), calls
 * are synchronous, as in the reference.  Each context owns one CUDA stream on
 * one device.
 */
#ifndef CHPE_H
#define CHPE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference surface (src/chpe_c_api.zig) ------------------------------ */

/* chpe_c_api.zig:25-48.  Opens and validates the archive (mmap, read-only),
 * picks the architecture from the path ("9B"/"9b"/"qwen35" -> Qwen3.5-9B,
 * "72B"/"72b" -> Qwen2.5-72B, else Qwen2.5-3B), uploads it to HBM and builds
 * the engine with max_seq_len 2048 on CUDA device 0.  NULL on any failure. */
void *chpe_init(const char *archive_path);

/* chpe_c_api.zig:50-78.  Runs tokens[0..num_tokens) at positions
 * 0..num_tokens-1 (a fresh sequence on every call), keeps the last step's
 * logits, copies them to out_logits when it is non-NULL (vocab floats,
 * unchecked) and returns the last argmax.  -1 when ctx or tokens is NULL,
 * num_tokens is 0, num_tokens exceeds max_seq_len, or the device failed. */
int chpe_forward_tokens(void *ctx, const uint32_t *tokens, size_t num_tokens,
                        float *out_logits);

/* chpe_c_api.zig:80-87.  Copies the last logits; returns vocab, or 0 when a
 * pointer is NULL or max_len < vocab. */
size_t chpe_get_last_logits(void *ctx, float *out_logits, size_t max_len);

/* chpe_c_api.zig:89-105.  A NULL ctx answers for Qwen2.5-3B. */
size_t chpe_get_vocab_size(void *ctx);
size_t chpe_get_hidden_dim(void *ctx);
size_t chpe_get_num_layers(void *ctx);

/* chpe_c_api.zig:107-135.  Fields of the last ForwardResult
 * (chpe_engine.zig:803-810); a NULL ctx returns 0. */
uint64_t chpe_get_last_elapsed_ns(void *ctx);
uint32_t chpe_get_last_argmax(void *ctx);
float chpe_get_last_max_logit(void *ctx);
float chpe_get_last_token0_logit(void *ctx);
float chpe_get_last_hidden_norm(void *ctx);

/* chpe_c_api.zig:137-143.  NULL-safe. */
void chpe_free(void *ctx);

/* ---- additions (no counterpart in the reference) ------------------------- */

/* Architecture ids for the calls below; CHPE_ARCH_BY_PATH picks from the
 * path as chpe_init does. */
#define CHPE_ARCH_BY_PATH (-1)
#define CHPE_ARCH_QWEN2_5_3B 0
#define CHPE_ARCH_QWEN3_5_9B 1
#define CHPE_ARCH_QWEN2_5_72B 2

/* chpe_init with the architecture, max_seq_len and CUDA device chosen by the
 * caller (chpe_init fixes them to path-derived, 2048 and 0). */
void *chpe_init_ex(const char *archive_path, int arch, uint32_t max_seq_len, int device);

/* The engine over archive bytes held by the caller (CHPEEngine.init,
 * chpe_engine.zig:854, which takes bytes, not a path).  No header validation,
 * exactly as the engine-level reference: an invalid archive runs the
 * reference's synthetic fallbacks.  The bytes are copied to the device and
 * must stay valid until chpe_free (small tensors are read from them at init). */
void *chpe_init_bytes(const void *bytes, uint64_t len, int arch, uint32_t max_seq_len,
                      int device);

/* Tensor parallelism over the GPUs of one node, one process per GPU (an
 * extension: the reference engine is single-threaded CPU code).  Every rank
 * opens the same archive (path: a shared read-only mmap, or bytes) with its
 * rank and the world size (1..8), exports the 64-byte CUDA IPC handle of its
 * exchange region, receives every rank's handles in rank order (any host
 * transport: the Python layer uses torch.distributed), and connects; after
 * that every rank calls the same forward / generate / bench functions in
 * lockstep.  Heads, hidden, FFN rows and vocabulary must divide by world; all
 * projections must be flat cells or raw streams (the 9B and 72B archives).
 * Each rank uploads only the archive tiles it reads.
 * Results equal the single-GPU engine's: each output element is computed
 * whole on one rank.  Returns NULL / -1 on failure (chpe_last_error). */
void *chpe_init_tp(const char *archive_path, int arch, uint32_t max_seq_len, int device, int rank,
                   int world);
void *chpe_init_tp_bytes(const void *bytes, uint64_t len, int arch, uint32_t max_seq_len, int device,
                         int rank, int world);
int chpe_tp_export_handle(void *ctx, uint8_t *handle64);
int chpe_tp_connect(void *ctx, const uint8_t *handles, int world);
/* The rows one rank owns (no GPU needed): ten uint32 values, query heads
 * (count, first), kv heads (first, count), hidden rows (count, first), FFN
 * rows (count, first), vocabulary rows (count, first).  0, or -1 when the
 * architecture does not split evenly over `world`. */
int chpe_tp_slice(int arch, int rank, int world, uint32_t out[10]);
/* The archive tiles (records) one rank uploads and its kernels read, merged
 * into disjoint ascending runs [lo, hi): runs[2i] = lo, runs[2i+1] = hi, at
 * most `cap` runs written (no GPU needed).  wpt = weights per tile (32768 for
 * cell archives, 16384 for int8 raw tiles, 8192 for FP16/BF16 raw tiles),
 * record_count = the archive's record count.  Returns the number of runs, or -1 when the architecture does
 * not split evenly over `world`. */
int64_t chpe_tp_tile_runs(int arch, int is_raw, uint64_t wpt, uint64_t record_count, int rank,
                          int world, uint64_t *runs, size_t cap);

/* WeightArchive.validate (weight_archive.zig:152-172): 0 when valid, else the
 * error: 1 InvalidMagic, 2 UnsupportedVersion, 3 BadGeometry, 4 Truncated,
 * 6 FileTooSmall, 10 MisalignedHeader. */
int chpe_validate_archive(const void *bytes, uint64_t len);

/* Archive converters (weight_archive.zig:617-776: convertToDensePosix,
 * convertToRawContiguousPosix, convertToRawFp16ContiguousPosix), writing
 * dst_path from the archive at src_path (validated first):
 *   CHPE_CONVERT_DENSE     20480-byte records -> 17408-byte cells (the
 *                          prefetch labels dropped; a raw source is refused);
 *   CHPE_CONVERT_RAW       -> raw 16384-byte tiles (the code bytes only);
 *   CHPE_CONVERT_RAW_FP16  -> raw tiles with every 2-D tile's BF16 weights
 *                          rounded to FP16 on CUDA device `device`, 1-D tiles
 *                          (the 3B raw layout's norm/bias positions, cells of
 *                          quant_bits 32) copied verbatim, FLAG_RAW_FP16 set.
 * The header keeps the source's fields with the new geometry.  0, or -1 with
 * the reason in chpe_last_error(NULL). */
#define CHPE_CONVERT_DENSE 0
#define CHPE_CONVERT_RAW 1
#define CHPE_CONVERT_RAW_FP16 2
int chpe_convert_archive(const char *src_path, const char *dst_path, int mode, int device);

/* One forwardDecode(token, pos) step that continues the current sequence
 * (the reference's ABI can only restart at 0).  Returns the argmax or -1. */
int chpe_decode_step(void *ctx, uint32_t token, uint32_t pos, float *out_logits);

/* One decode step of a Qwen3.5 Gated DeltaNet (linear-attention) layer after
 * its input projections, on the caller's device buffers (an extension: the
 * reference runs these layers as GQA).  mixed_qkv [2*nk*128 + nv*128] (q|k|v
 * before the conv), z [nv*128], a and b [nv]; conv_w [conv_dim][4] taps
 * (oldest input first, 16-byte aligned); conv_hist [4][conv_dim] holds the
 * inputs of position p in slot p % 4 (zero it at the start of a sequence);
 * t is this token's position; A_log, dt_bias [nv]; norm_w [128]; state
 * [nv][128][128] f32 per value head as [value j][key i], updated in place
 * (16-byte aligned); out [nv*128] = gated-RMSNorm'ed output (the input of
 * out_proj).  Head dims must be 128 and nv a multiple of nk.  Enqueued on
 * `stream` (a cudaStream_t, or NULL); 0, or -1 for invalid arguments. */
int chpe_deltanet_step(const float *mixed_qkv, const float *z, const float *a, const float *b,
                       const float *conv_w, float *conv_hist, uint32_t t, const float *a_log,
                       const float *dt_bias, const float *norm_w, float *state, float *out,
                       uint32_t num_k_heads, uint32_t num_v_heads, uint32_t k_head_dim,
                       uint32_t v_head_dim, float eps, void *stream);

/* Batch-M speculative verification (an extension; the reference has no such
 * function): scores m candidate tokens at positions pos..pos+m-1 of the
 * current sequence, candidate i seeing the KV entries of candidates < i
 * (causal), which is exactly m forwardDecode steps.  out_logits gets
 * [m][vocab] floats and out_argmax m ids (either may be NULL).  The cache
 * keeps all m entries and the next position is pos+m (roll back by calling
 * chpe_decode_step / chpe_verify at an earlier pos).  0, or -1 on error. */
int chpe_verify(void *ctx, const uint32_t *toks, size_t m, uint32_t pos, float *out_logits,
                uint32_t *out_argmax);
/* How chpe_verify runs: for m <= 8 candidates on an archive whose
 * projections and LM head are 4-bit group-scaled flat cells in whole 128-row
 * blocks (the 9B and 72B archives) it runs one batched step of 4 or 8 tokens
 * whose GEMMs read every weight once for all candidates on the tcgen05 tensor
 * cores (results equal m decode steps up to f32 rounding); otherwise m
 * sequential decode steps (bit-identical to chpe_decode_step).  The
 * environment variable CHPE_VERIFY_BATCHED=0 forces the sequential steps.
 * chpe_last_verify_batched: 1 when the last chpe_verify ran the batched
 * step.  chpe_verify_batched_unavailable: "" when m candidates can take the
 * batched step, else the reason (valid until the next call on ctx). */
int chpe_last_verify_batched(void *ctx);
const char *chpe_verify_batched_unavailable(void *ctx, int m);

/* Greedy generation on the device: runs the prompt from position 0, then
 * n_gen tokens, each the argmax of the step before, without host round
 * trips.  out_tokens receives n_gen ids.  0 on success, -1 on error. */
int chpe_generate(void *ctx, const uint32_t *prompt, size_t n_prompt, size_t n_gen,
                  uint32_t *out_tokens);

/* Speculative greedy generation (an extension; the reference has no
 * speculative decoding): like chpe_generate, but after the prompt each round
 * drafts up to draft_len tokens by prompt lookup (the tokens that followed
 * the latest earlier occurrence of the sequence's last ngram .. 1 tokens),
 * scores the pending token and the draft in one chpe_verify call, keeps the
 * longest draft prefix equal to the model's greedy tokens plus the model's
 * next token, and continues from there (the KV entries of rejected draft
 * tokens are overwritten by the next round).  out_tokens receives exactly
 * the n_gen tokens chpe_generate gives.  stats (may be NULL) receives three
 * counts: verify rounds, draft tokens proposed, draft tokens accepted.
 * 0 on success, -1 on error. */
int chpe_speculative_generate(void *ctx, const uint32_t *prompt, size_t n_prompt, size_t n_gen,
                              uint32_t draft_len, uint32_t ngram, uint32_t *out_tokens,
                              uint64_t *stats);

/* Benchmark helpers.  chpe_bench_greedy: n greedy steps from the current
 * position, device time by CUDA events on the engine stream.
 * chpe_bench_host: n steps with host tokens, each step copying its token in
 * and its logits (to `logits`, vocab floats) and result out; wall time. */
int chpe_bench_greedy(void *ctx, size_t n_steps, float *device_ms);
int chpe_bench_host(void *ctx, const uint32_t *tokens, size_t n_steps, float *logits,
                    double *wall_ms);

/* Per-kernel timing for the roofline: launches every recorded op of one role
 * (1 QKV, 2 attention, 3 O, 4 gate/up, 5 down, 6 LM head, 7 embedding)
 * across all layers, `rounds` times, on the engine stream, so consecutive
 * launches stream different layers' weights from HBM.  Gives the average
 * milliseconds per launch, the algorithmic weight bytes per launch (codes +
 * scales of the rows used) and the launch count.  Needs a prior forward. */
int chpe_bench_kernel(void *ctx, int role, int rounds, float *avg_ms, double *bytes_per_launch,
                      int *launches);

/* chpe_bench_kernel with every launch timed alone from a cold L2: before
 * each launch a 256 MiB buffer (twice the L2) is written, so weights that a
 * role's layers would otherwise keep in L2 between rounds (small tensors)
 * come from HBM.  Same outputs; the average covers the launches only. */
int chpe_bench_kernel_cold(void *ctx, int role, int rounds, float *avg_ms, double *bytes_per_launch,
                           int *launches);

/* Name of the kernel that runs the first op of a role (same role numbers as
 * chpe_bench_kernel), e.g. "gemv_flat_tma_kernel<W4G,FLAT>"; "" when the
 * role has no op or ctx is NULL.  The string lives as long as ctx. */
const char *chpe_role_kernel_name(void *ctx, int role);

/* One greedy decode step launched op by op (not as the graph), with CUDA
 * events between the ops: writes up to `cap` per-op milliseconds and roles
 * (chpe_bench_kernel's numbering, 0 other) and returns the op count, -1 on
 * error.  With tensor parallelism every rank calls it together.  Advances the
 * position by one.  Needs a prior forward. */
int chpe_profile_step(void *ctx, float *op_ms, int *op_roles, int cap);

/* The batched verification step of m (<= 8) scratch candidates at pos,
 * launched op by op with CUDA events between the ops: per role (numbers as
 * chpe_bench_kernel; 0 other) the summed milliseconds and algorithmic weight
 * bytes, `cap` entries each.  The KV entries at pos.. are overwritten.
 * Returns the op count, -1 on error. */
int chpe_profile_verify(void *ctx, size_t m, uint32_t pos, float *role_ms, double *role_bytes, int cap);

/* Algorithmic weight bytes one decode step of this context streams (codes
 * and scales of the rows its projections use; with tensor parallelism, this
 * rank's share).  0 for NULL. */
double chpe_step_weight_bytes(void *ctx);

/* all_finite of the last ForwardResult (1/0; 0 for NULL). */
int chpe_get_last_all_finite(void *ctx);
/* Kernels launched per decode step (graph nodes). */
int chpe_kernels_per_step(void *ctx);
/* Current sequence position (next step's pos). */
uint32_t chpe_get_position(void *ctx);
/* Archive bytes held in this context's device memory: the whole archive on
 * one GPU; with tensor parallelism only the tiles the rank reads (the
 * embedding records and its row slice of every projection), about
 * 1/world of the weights. */
uint64_t chpe_device_archive_bytes(void *ctx);
/* Last error message of ctx, or, when ctx is NULL, of the calling thread's
 * last failed init or chpe_attention_decode_noalloc call; "" when none. */
const char *chpe_last_error(void *ctx);

/* Paged KV cache (an extension; the reference keeps one contiguous f32
 * cache, chpe_engine.zig:755-801).  Every layer's FP16 K and V live in a pool
 * of pages of chpe_kv_page_size() positions; the sequence's page table maps
 * logical page p (positions p*page ..) to a physical page, the same table for
 * every layer.  A step maps the pages it reaches from a free list; a new
 * sequence (any call that runs position 0) returns them all.
 *
 * chpe_kv_load writes K (rotated, as the cache holds it) and V rows
 * k, v [n][kv_heads*head_dim] floats, rounded to FP16, at positions
 * pos0..pos0+n-1 of one layer (restoring a saved prefix, or a test's
 * prefilled context); with tensor parallelism each rank keeps its kv heads.
 * It does not move the sequence position.
 * chpe_kv_set_page_order sets the order free pages are handed out in (a
 * permutation of all n pages) and starts a new sequence.
 * chpe_kv_page_table writes up to cap entries of the mapped page table,
 * stores the pool's page count in *num_pages (when non-NULL) and returns the
 * mapped count.  0 / count on success, -1 on error (chpe_last_error). */
uint32_t chpe_kv_page_size(void);
int chpe_kv_load(void *ctx, uint32_t layer, uint32_t pos0, uint32_t n, const float *k,
                 const float *v);
int chpe_kv_set_page_order(void *ctx, const uint32_t *order, uint32_t n);
int chpe_kv_page_table(void *ctx, uint32_t *out, uint32_t cap, uint32_t *num_pages);

/* Decode attention for callers that cannot allocate device memory: serving
 * runtimes that hand out device memory only from their own pre-sized pools,
 * and plugins inside a host process that owns all allocation on the GPU.  No
 * counterpart in the reference.  It is the attention step of
 * chpe_probe_attention (RoPE on q and k with theta rope_theta, append k/v at
 * pos, GQA softmax over positions 0..pos) on device pointers the caller owns:
 * q [num_heads*head_dim] and k, v [num_kv_heads*head_dim] float; k_cache and
 * v_cache FP16, contiguous [max_seq_len][num_kv_heads][head_dim]; out
 * [num_heads*head_dim] float; stream a cudaStream_t (NULL: default stream).
 * It allocates nothing: its scratch is a fixed 1 MiB static device array per
 * GPU, held until the library unloads.  The first call on a device resolves
 * that array's address (with the device current).  Calls share the array,
 * so calls that overlap on the GPU race; each call clears what it needs.
 * Limits: head_dim 128 or 256, at most 8 query heads per kv head, and
 * 4096 + num_kv_heads * 16 * (num_heads/num_kv_heads) * (head_dim+4) * 4
 * bytes (16 splits of the positions per kv head, one partial record of
 * head_dim+4 floats per split and query head) within 1 MiB.
 * Returns 0, -1 for invalid arguments, -2 when the sizes exceed the scratch
 * limit, -3 for a CUDA error; the reason is in chpe_last_error(NULL). */
int chpe_attention_decode_noalloc(const float *q, const float *k, const float *v, void *k_cache,
                                  void *v_cache, float *out, uint32_t pos, uint32_t max_seq_len,
                                  uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim,
                                  float rope_theta, void *stream);

/* ---- probes for the parity tests ------------------------------------------ */

/* gemvLinear (chpe_engine.zig:1396) on the device over host vectors:
 * y (r_total floats) is read (for accumulate) and written.  bias_tile < 0:
 * none.  0 on success. */
int chpe_probe_gemv_linear(void *ctx, uint64_t tile_start, uint64_t num_tiles, const float *x,
                           uint64_t x_len, float *y, uint64_t r_total, uint64_t c_total,
                           int accumulate, int64_t bias_tile);
/* The decode attention of one layer (chpe_engine.zig:1688-1734: RoPE on q
 * and k, append k/v to the layer's cache at `pos`, GQA softmax over t <= pos)
 * on host vectors q [heads*head_dim], k and v [kv_heads*head_dim]; writes
 * out [heads*head_dim].  Positions 0..pos-1 of the layer's cache are whatever
 * earlier steps or calls left there.  0 on success. */
int chpe_probe_attention(void *ctx, uint32_t layer, uint32_t pos, const float *q, const float *k,
                         const float *v, float *out);
/* Failure detection without a GPU fault: a bounded device wait (the kind
 * the tensor-parallel exchanges use) for an arrival nothing sends, limited to
 * `polls` polls.  Returns -1 with the device-timeout error in
 * chpe_last_error(ctx), exactly as a decode step whose exchange timed out
 * does; the context stays usable.  (The decode path's limit is set with the
 * environment variable CHPE_WAIT_POLLS when a context is created.) */
int chpe_probe_wait_timeout(void *ctx, uint32_t polls);
/* The batched GEMM of chpe_verify on one gemvLinear call site of 4-bit
 * group-scaled flat cells (tcgen05 tensor cores): y[t] (= or +=) W x[t] for
 * nt (4 or 8) tokens; x [nt][c_total], y [nt][r_total] host buffers; rows a
 * multiple of 128, columns of 128.  0, or -1 (chpe_last_error) when the call
 * cannot take that path. */
int chpe_probe_bgemm(void *ctx, uint64_t tile_start, uint64_t num_tiles, const float *x, int nt,
                     float *y, uint64_t r_total, uint64_t c_total, int accumulate);
/* The tensor-core path of the batched GEMMs on its own: D [128][n] (s32) =
 * A [128][64] (unsigned bytes) x B [n][64] (signed bytes)^T through
 * tcgen05.mma kind::i8 with A in tensor memory and B in shared memory
 * (n 16 or 32), on CUDA device `device`, host buffers.  0, or -1 with the
 * reason in chpe_last_error(NULL). */
int chpe_probe_tc_i8(const uint8_t *a, const int8_t *b, int n, int32_t *d, int device);
/* unpackEmbedRow (chpe_engine.zig:1491) for one token into out (hidden_dim
 * floats, read first: rows the reference leaves unwritten keep them). */
int chpe_probe_embed(void *ctx, uint32_t token, float *out);
/* Dequantised weights of one cell as the reference materialises them
 * (flat != 0: gemvCellFlat's 32768 tile weights; else rows*cols row-tiled
 * weights).  *n_out receives the count.  0 on success. */
int chpe_probe_dequant_cell(void *ctx, uint64_t tile, int flat, float *out, uint64_t cap,
                            uint64_t *n_out);

#ifdef __cplusplus
}
#endif
#endif /* CHPE_H */
