// engine_types.h -- plain structs shared by the host planner and the kernels.
#pragma once
#include <cstdint>

namespace chpe {

// How one gemvLinear call site (chpe_engine.zig:1396) reads its weights.
enum SrcKind : int32_t {
  SRC_NOOP = 0,     // accumulate onto an invalid span: nothing happens
  SRC_PATTERN = 1,  // invalid archive / start past the end: 0.01*((r%13)-6)
  SRC_RAW = 2,      // raw contiguous tiles: row-major stream from tile_start
  SRC_ROWTILE = 3,  // uniform row-tiled cells (c_total <= 2048)
  SRC_FLAT = 4,     // uniform flat 32768-weight cells (c_total > 2048)
  SRC_GEN_ROWTILE = 5,  // any row-tiled cells, per-row table, per-cell format
  SRC_GEN_FLAT = 6,     // any flat cells, per-tile format
};

// Weight formats; each 16-byte chunk of codes covers CW columns.
enum Fmt : int32_t {
  FMT_W4G = 0,   // 4-bit, group-128 FP16 scales (+ outliers)
  FMT_W4SB = 1,  // 4-bit, per-tile scale and bias
  FMT_W2G = 2,   // 2-bit codebook {0,1,-2,-1}, group-128 scales
  FMT_W2SB = 3,  // 2-bit codebook, per-tile scale and bias
  FMT_W8 = 4,    // int8 cell, (sum q*x)*scale + bias
  FMT_F16 = 5,   // IEEE half
  FMT_BF16 = 6,  // bfloat16
  FMT_F32 = 7,   // float
  FMT_I8RAW = 8, // raw int8 stream, (sum q*x) * 0.00373708
  FMT_ZERO = 9,  // flat 8/16/32-bit cells: the reference reads zeros
};

struct GemvSrc {
  int32_t kind;
  int32_t fmt;
  uint32_t r_total;       // output rows (y length the call writes)
  uint32_t c_total;       // columns
  uint32_t x_len;         // length of the x slice the reference passes
  uint32_t rows_covered;  // ROWTILE: rows the cells cover (rest: zero/untouched)
  uint32_t cell_rows;     // ROWTILE uniform rows per cell
  uint32_t cell_cols;     // ROWTILE uniform cols per cell (row stride)
  uint32_t outliers;      // ROWTILE W4G/W2G with rows == 16: additive outliers
  uint32_t has_aux;       // FLAT: some tile carries down_aux replacements
  uint32_t n_tiles;       // available tiles
  uint32_t row0;          // FLAT/RAW: first tensor row of this call (a tensor-parallel slice)
  const uint8_t* arc;     // device archive (byte 0)
  uint64_t tile0;         // byte offset of tile_start's code area
  uint64_t stride;        // bytes between tiles
  uint64_t flat_limit;    // FLAT/RAW: available weights (n_tiles * wpt)
  const float* bias;      // optional bias (r_total floats)
  const uint32_t* row_cell;    // GEN_ROWTILE: cell (relative) per row, ~0u = none
  const uint16_t* row_in_cell; // GEN_ROWTILE: row inside that cell
};

// Per-step state in device memory.
struct StepState {
  int32_t token;       // token for this step (host-written)
  int32_t pos;         // position of this step
  int32_t feed_argmax; // 1: take the token from the previous step's argmax
  int32_t stop;        // early-exit flag of the layer loop (chpe_engine.zig:1763)
  unsigned long long best;  // packed (ordered logit, ~index) for argmax
  uint32_t finite;     // 1 until a non-finite logit is seen
  uint32_t done_ctas;  // LM-head CTAs finished (last one finalises)
  int32_t n_gen;       // generated-token counter (chpe_generate)
  int32_t err;         // non-zero: a kernel gave up a bounded wait (device timeout)
  int32_t gather;      // tensor parallel: 1 = every rank receives the full logits
  int32_t pad_;
};

// ---- tensor parallelism (one process per GPU) ------------------------------
// Every rank owns one exchange region (step state, these counters, hidden,
// attention output, MLP activation, logits) mapped into every other rank
// through CUDA IPC.  A producing kernel writes its output rows into every
// rank's region and then adds 1 to counter `kind` on every rank (release,
// system scope); the consuming kernel waits until its own counter reaches the
// arrivals of all ranks for that (step, layer).
constexpr int kTpMax = 8;
enum TpSig : int32_t { SIG_ATT = 0, SIG_O = 1, SIG_GU = 2, SIG_DOWN = 3, SIG_LM = 4, SIG_KINDS = 5 };

struct TpShared {
  unsigned long long sig[8];  // arrivals per kind since the engine was built
  uint32_t epoch;             // decode steps completed (advanced by the LM head)
  float token0;               // logit of token 0 (from the rank that owns vocab row 0)
  uint32_t pad_[14];
};

struct TpLink {
  int32_t world;               // 1: single GPU, nothing exchanged
  int32_t rank;
  long long delta[kTpMax];     // byte distance from this rank's region to rank r's
  TpShared* sh;                // this rank's counters
  int32_t wait_sig;            // kind to wait for before reading x, -1 none
  int32_t signal_sig;          // kind to signal after the outputs, -1 none
  uint32_t wait_index;         // target = (epoch * wait_per_step + wait_index) * wait_units
  uint32_t wait_per_step;
  unsigned long long wait_units;  // arrivals per (step, layer) of the awaited kind
  unsigned long long lm_units;    // LM head: arrivals per step of all ranks' CTAs
  int32_t bcast;               // 1: outputs lie in the region; write them on every rank
  uint32_t wait_polls;         // polls before a wait gives up (0: the default limit)
  const int32_t* err;          // this rank's StepState::err: once set, waits give up at once
};

// Result of one forward step (chpe_engine.zig:803 ForwardResult).
struct StepResult {
  uint32_t argmax_token;
  float max_logit;
  float token0_logit;
  float hidden_norm;
  int32_t all_finite;
  int32_t pos;
};

}  // namespace chpe
