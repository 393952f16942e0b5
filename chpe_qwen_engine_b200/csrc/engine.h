// engine.h -- the B200 decode engine behind the chpe C ABI.
//
// Mirrors CHPEEngine (chpe_engine.zig:820-1804): init sniffs the archive
// format and sizes buffers, forwardDecode(token, pos) runs one token through
// every layer.  Here the archive bytes live in HBM verbatim (the reference's
// flat-index addressing, including its over-reads, then reads the same bytes),
// every per-token op is a CUDA kernel, and one decode step is a CUDA graph of
// PDL-chained kernels replayed per token with (token, pos) in device memory.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "chpe_maps.h"
#include "engine_types.h"

namespace chpe {

// Records the calling thread's last error message, which chpe_last_error(NULL)
// returns (failed inits and the context-free entry points).
void set_thread_error(const std::string& msg);

struct Op;         // one recorded kernel launch (engine.cu)
struct BatchStep;  // the batched decode step of NT tokens (engine_verify.cu)

struct EngineFacts {  // CHPEEngine fields after init sniffing (:862-918)
  int archive_valid = 0, is_raw = 0, is_raw_fp16 = 0, is_dense = 0;
  int quant_bits = 2;
  uint64_t record_count = 0, stride = 0, wpt = 8192;
};

class Engine {
 public:
  // Counterpart of CHPEEngine.init over archive bytes the caller keeps alive
  // for the engine's lifetime (`bytes` may be an mmap).  Throws std::runtime_error.
  // With tp_world > 1 the engine is rank tp_rank of a tensor-parallel group
  // (one process per GPU) and is usable after tp_connect().
  Engine(const uint8_t* bytes, uint64_t len, int arch, uint32_t max_seq, int device, int tp_rank = 0,
         int tp_world = 1);
  ~Engine();

  // Tensor parallel set-up: the CUDA IPC handle (64 bytes) of this rank's
  // exchange region, then every rank's handles in rank order; builds the step.
  void tp_export(uint8_t* handle64) const;
  void tp_connect(const uint8_t* handles, int world);
  int tp_world() const { return tp_world_; }
  int tp_rank() const { return tp_rank_; }

  const ChpeArch& arch() const { return *arch_; }
  const EngineFacts& facts() const { return f_; }
  uint32_t max_seq() const { return max_seq_; }

  // forwardDecode over tokens at positions start_pos.. (blocking).
  void forward(const uint32_t* toks, size_t n, uint32_t start_pos);
  // Greedy generation on the device: prompt (n_prompt) then n_gen steps
  // feeding each argmax back as the next token; out_tokens gets n_gen ids.
  void generate(const uint32_t* prompt, size_t n_prompt, size_t n_gen, uint32_t* out_tokens);
  // Batch-M verification: logits of m candidate tokens scored at positions
  // pos..pos+m-1, each seeing the KV entries of the ones before it (causal),
  // i.e. m forwardDecode steps; logits_out [m][vocab], argmax_out [m] (either
  // may be null).  The last step's result becomes last_result().
  void verify(const uint32_t* toks, size_t m, uint32_t pos, float* logits_out, uint32_t* argmax_out);
  // How the last verify() ran: 1 batched tensor-core step, 0 sequential
  // steps; and why the batched step does not apply ("" when it does).
  int last_verify_batched() const { return last_verify_batched_; }
  // The batched step of m candidates at pos launched op by op with CUDA
  // events between the ops (scratch candidates; the KV entries at
  // pos.. are overwritten): per role (chpe_bench_kernel's numbering, 0
  // other) the summed milliseconds and algorithmic weight bytes.  Returns
  // the op count.
  int profile_verify(size_t m, uint32_t pos, float* role_ms, double* role_bytes, int cap);
  std::string batch_unavailable_reason(int nt);
  // Greedy generation with speculative verification: drafts of up to
  // `draft` tokens are proposed by prompt lookup (the tokens that followed the
  // latest earlier occurrence of the last `ngram`.. 1 tokens of the sequence)
  // and scored in one verify() call together with the pending token; the
  // longest prefix matching the target's greedy tokens is kept, plus the
  // target's own next token.  Output equals generate()'s.  stats (may be
  // null): verify rounds, draft tokens proposed, draft tokens accepted.
  void speculative_generate(const uint32_t* prompt, size_t n_prompt, size_t n_gen, uint32_t draft,
                            uint32_t ngram, uint32_t* out_tokens, uint64_t* stats);
  // n greedy steps from the current position, timed with CUDA events on the
  // engine stream; returns milliseconds.
  float timed_greedy_steps(size_t n);
  // Same workload through host round trips: per step a pinned H2D of the
  // token and a D2H of the logits and result (wall time, milliseconds).
  double timed_host_steps(const uint32_t* toks, size_t n, float* logits_host);

  const StepResult& last_result() const { return last_; }
  uint64_t last_elapsed_ns() const { return last_ns_; }
  void copy_logits(float* out) const;  // last step's logits (vocab floats)
  uint32_t current_pos() const { return pos_; }
  // Bytes of archive held in device memory: the whole archive on one GPU, this
  // rank's shards with tensor parallelism.
  uint64_t device_archive_bytes() const { return dev_arc_bytes_; }
  int kernels_per_step() const;

  // Times every recorded op of one role (ROLE_*) across all layers, `rounds`
  // times, with CUDA events on the engine stream; returns the average
  // milliseconds per launch and the algorithmic weight bytes per launch.
  // flush_l2: before every launch a 256 MiB buffer is written (evicting the
  // weights from L2), and each launch is timed alone between its own events.
  void bench_role(int role, int rounds, float* avg_ms, double* bytes_per_launch, int* launches,
                  bool flush_l2 = false);
  std::string role_kernel_name(int role) const;
  // One greedy step launched op by op with CUDA events between the ops (no
  // graph); per-op milliseconds and roles.  With tensor parallelism every rank
  // calls it together.  Advances the position like a decode step.
  int profile_step(float* op_ms, int* op_roles, int cap);
  double step_weight_bytes() const;  // algorithmic weight bytes of one step (this rank)

  // Test entry points that run one kernel family on host vectors.
  void debug_gemv_linear(uint64_t tile_start, uint64_t num_tiles, const float* x, uint64_t x_len,
                         float* y, uint64_t r_total, uint64_t c_total, int accumulate,
                         int64_t bias_tile);
  void debug_embed(uint32_t token, float* out);
  // The decode attention kernel of `layer` at position pos on host vectors:
  // q [H*HD], k/v [KV*HD] (un-rotated), appends k/v to that layer's cache at
  // pos and returns the attention output [H*HD].
  void debug_attention(uint32_t layer, uint32_t pos, const float* q, const float* k, const float* v,
                       float* out);
  void debug_dequant_cell(uint64_t tile, int flat, float* out, uint64_t cap, uint64_t* n_out);
  // The batched tensor-core GEMM of NT (4 or 8) tokens over one gemvLinear
  // call site: x [nt][c_total], y [nt][r_total] (read for accumulate).
  void debug_bgemm(uint64_t tile_start, uint64_t num_tiles, const float* x, int nt, float* y,
                   uint64_t r_total, uint64_t c_total, int accumulate);
  // Runs a bounded device wait for an arrival that never comes, with `polls`
  // polls at most; throws the device-timeout error the decode path raises and
  // leaves the engine usable.
  void debug_wait_timeout(uint32_t polls);

  // ---- paged KV cache ------------------------------------------------------
  // The cache of every layer is a pool of pages of kKvPage positions; the
  // sequence's page table maps logical page p (positions p*kKvPage..) to a
  // physical page, the same for every layer.  Pages are taken from a free
  // list when a step first reaches them and all return to it when a new
  // sequence starts at position 0.
  static constexpr int kKvPageShift = 6;
  static constexpr uint32_t kKvPage = 1u << kKvPageShift;
  // Writes K (already rotated, as the cache holds it) and V rows
  // [n][kv_heads*head_dim] for positions pos0..pos0+n-1 of one layer into the
  // cache as FP16 (round to nearest), mapping pages as needed.  With tensor
  // parallelism the rows hold every kv head; this rank keeps its own.
  void kv_load(uint32_t layer, uint32_t pos0, uint32_t n, const float* k, const float* v);
  // Sets the order in which free pages are handed out (a permutation of
  // 0..n_pages-1); returns every mapped page first (a new sequence).
  void kv_set_page_order(const uint32_t* order, uint32_t n);
  // Mapped logical pages and their physical pages (up to cap entries).
  uint32_t kv_page_table(uint32_t* out, uint32_t cap) const;
  uint32_t kv_pages() const { return n_pages_; }

  cudaStream_t stream() const { return stream_; }

 private:
  GemvSrc plan_linear(uint64_t tile_start, uint64_t num_tiles, uint32_t r_total,
                      uint32_t c_total, uint32_t x_len, int accumulate, int64_t bias_tile);
  void unpack_norm(uint64_t tile, float* out) const;
  void unpack_bias(uint64_t tile, float* out, uint32_t n) const;
  uint64_t code_off(uint64_t tile) const;
  const float* upload_floats(const std::vector<float>& v);
  void build_step();
  void build_step_tp();
  void push_embed(std::vector<Op>& ops);
  GemvSrc plan_lm_head();
  void add_linear_ops(std::vector<Op>& ops, const GemvSrc* src, float* const* out, int nseg,
                      int epi, const float* x, const float* gamma, int check_layer,
                      uint32_t ncols, bool ignore_stop, const TpLink* tp = nullptr);
  void launch(const Op& op, cudaStream_t s) const;
  void record(cudaStream_t s) const;
  void run_steps(size_t n);
  void kv_ensure(uint64_t end_pos);  // map pages for positions < end_pos
  void kv_reset();                   // a new sequence: every page back to the free list
  void sync_result();
  void ensure_graph();

  const ChpeArch* arch_;
  int arch_id_;
  int device_;
  uint32_t max_seq_;
  const uint8_t* host_;  // borrowed archive bytes
  uint64_t len_;
  EngineFacts f_;

  cudaStream_t stream_ = nullptr;
  cudaGraphExec_t graph_ = nullptr;
  uint8_t* d_arc_ = nullptr;
  std::vector<void*> allocs_;
  float *d_hidden_, *d_q_, *d_k_, *d_v_, *d_attn_, *d_mlp_, *d_logits_, *d_xn_, *d_tmp_, *d_tmp2_;
  float *d_part_, *d_invfreq_;
  uint32_t* d_counters_;
  float* d_rb_part_ = nullptr;    // row-block GEMV: [part][rows] row sums
  uint32_t* d_rb_cnt_ = nullptr;  // row-block GEMV: arrival counters and abort flags
  uint64_t rb_part_cap_ = 0;      // floats in d_rb_part_
  __half *d_kc_, *d_vc_;
  StepState* d_st_;
  StepResult* d_res_;
  int32_t* d_gen_;
  uint32_t max_gen_ = 0;
  StepState* h_st_;      // pinned
  StepResult* h_res_;    // pinned
  uint32_t* h_tok_;      // pinned token ring
  size_t h_tok_cap_ = 0;
  std::vector<Op>* ops_ = nullptr;
  StepResult last_{};
  uint64_t last_ns_ = 0;
  uint32_t pos_ = 0;
  int num_sms_ = 148;
  int nsplit_ = 16;  // attention splits of the positions per kv head
  uint32_t wait_polls_ = 0;  // tensor-parallel wait limit (0: the default; CHPE_WAIT_POLLS)
  int last_verify_batched_ = 0;
  // Tensor parallelism uploads only the archive tiles this rank reads: the
  // embedding records and its row slice of every projection, each merged
  // run of tiles in its own allocation.  arc_for(tile) is the base pointer
  // that addresses byte offsets of the original archive inside the run that
  // holds `tile` (the whole archive's allocation without sharding).
  struct Shard {
    uint64_t lo, hi;  // tiles [lo, hi)
    uint8_t* dev;     // bytes of record lo onward (+ zero padding)
  };
  std::vector<Shard> shards_;
  uint64_t dev_arc_bytes_ = 0;
  void upload_archive(const uint8_t* bytes, uint64_t len);
  void upload_shards(const uint8_t* bytes, uint64_t len);
  const uint8_t* arc_for(uint64_t tile) const;
  // paged KV cache
  uint32_t n_pages_ = 0, mapped_ = 0;
  uint32_t kv0_ = 0, kvl_ = 0;         // kv heads this rank holds (all of them on one GPU)
  size_t layer_kv_elems_ = 0;          // halves per layer pool (n_pages * page * kv heads here * hd)
  uint32_t* d_pages_ = nullptr;        // device page table [n_pages]
  uint32_t* h_pages_ = nullptr;        // pinned mirror
  std::vector<uint32_t> free_pages_;   // stack: back() is handed out next

  // tensor parallelism
  int tp_rank_ = 0, tp_world_ = 1;
  uint8_t* d_region_ = nullptr;  // exchange region: step state, counters, hidden, attn, mlp, logits
  size_t region_bytes_ = 0;
  TpShared* d_tpsh_ = nullptr;
  long long tp_delta_[kTpMax] = {};
  std::vector<void*> ipc_open_;
  // The batched step of nt (4 or 8) tokens, built on first use; null when
  // the archive cannot take it (then verify() runs sequential steps).
  BatchStep* batch_step(int nt);
  // verify() through the batched step; false when it does not apply (the
  // caller then runs the sequential steps).
  bool verify_batched(const uint32_t* toks, size_t m, uint32_t pos, float* logits_out, uint32_t* argmax_out);
  void free_batch_steps();
  BatchStep* bsteps_[2] = {nullptr, nullptr};
  int bstep_state_[2] = {0, 0};  // 0 not tried, 1 built, -1 not applicable
  std::string bstep_why_[2];
  // verify(): per-candidate logits and results on the device
  float* d_vlogits_ = nullptr;
  StepResult* d_vres_ = nullptr;
  size_t vcap_ = 0;
};

}  // namespace chpe
