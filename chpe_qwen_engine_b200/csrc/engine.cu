// engine.cu -- CHPEEngine for B200: archive upload, per-call-site plans,
// one decode step recorded as a chain of PDL kernels and replayed as a graph.
#include "engine.h"

#include <time.h>

#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "attention.cuh"
#include "aux_kernels.cuh"
#include "gemv.cuh"
#include "gemv_tma.cuh"
#include "gemv_flat_tma.cuh"
#include "gemv_rowblk.cuh"

namespace chpe {

#define CK(x)                                                                               \
  do {                                                                                      \
    cudaError_t e_ = (x);                                                                   \
    if (e_ != cudaSuccess)                                                                  \
      throw std::runtime_error(std::string(#x) + ": " + cudaGetErrorString(e_));            \
  } while (0)

enum OpType : int32_t {
  OP_GEMV = 0, OP_GEN_ROW, OP_GEN_FLAT, OP_AUX, OP_ATTN, OP_EMBED, OP_NORM, OP_SWIGLU,
  OP_PATTERN, OP_ARGMAX, OP_TMA, OP_FLAT_TMA
};
constexpr int kTmaStages = 4;
constexpr uint32_t kFlatSmemLimit = 227u * 1024u - 1024u;  // dynamic shared memory of one flat-TMA CTA
constexpr uint32_t kFlatSmemHalf = 112u * 1024u;           // ... when two CTAs share an SM
constexpr uint32_t kFlatStagesWanted = 12;

// Roles of recorded ops (for per-kernel timing).
enum Role : int32_t { ROLE_OTHER = 0, ROLE_QKV = 1, ROLE_ATTN = 2, ROLE_O = 3, ROLE_GATEUP = 4,
                      ROLE_DOWN = 5, ROLE_LMHEAD = 6, ROLE_EMBED = 7 };

struct Op {
  int32_t type = 0, fmt = 0, kind = 0, threads = 256, hd = 128;
  int32_t role = ROLE_OTHER;
  double alg_bytes = 0;  // algorithmic weight bytes this op streams
  dim3 grid{1, 1, 1};
  size_t smem = 0;
  GemvLaunch g{};
  GenLaunch gen{};
  AuxLaunch aux{};
  AttnLaunch at{};
  EmbedLaunch em{};
  NormLaunch nm{};
  SwigluLaunch sw{};
  PatternLaunch pt{};
  ArgmaxLaunch am{};
  TmaLaunch tm{};
  FlatTmaLaunch fl{};
};

// ---- host restatements of small archive reads ------------------------------
static inline uint16_t rd16(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return v; }
static inline uint32_t rd32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }
static inline uint64_t rd64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }

static uint64_t now_ns() {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

static int fmt_bits(int fmt) {
  switch (fmt) {
    case FMT_W4G: case FMT_W4SB: return 4;
    case FMT_W2G: case FMT_W2SB: return 2;
    case FMT_W8: case FMT_I8RAW: return 8;
    case FMT_F16: case FMT_BF16: return 16;
    default: return 32;
  }
}

static int fmt_cw(int fmt) {
  switch (fmt) {
    case FMT_W4G: case FMT_W4SB: return 32;
    case FMT_W2G: case FMT_W2SB: return 64;
    case FMT_W8: case FMT_I8RAW: return 16;
    case FMT_F16: case FMT_BF16: return 8;
    default: return 4;
  }
}

uint64_t Engine::code_off(uint64_t tile) const {
  if (f_.is_raw) return 4096 + tile * 16384ull;
  if (f_.is_dense) return 4096 + tile * 17408ull + 64;
  return 4096 + tile * 20480ull + 3072 + 64;
}

// chpe_engine.zig:1144-1170 unpackNorm, reading past the archive end as zeros.
void Engine::unpack_norm(uint64_t tile, float* out) const {
  const uint32_t D = arch_->D;
  if (!f_.archive_valid || tile >= f_.record_count) {
    for (uint32_t i = 0; i < D; i++) out[i] = 1.0f;
    return;
  }
  uint64_t off = code_off(tile);
  auto byte_at = [&](uint64_t o) -> uint8_t { return o < len_ ? host_[o] : 0; };
  for (uint32_t i = 0; i < D; i++) {
    if (D == 4096 && f_.is_raw) {
      uint32_t b = (uint32_t)byte_at(off + 2 * i) | ((uint32_t)byte_at(off + 2 * i + 1) << 8);
      uint32_t bits = b << 16;
      memcpy(&out[i], &bits, 4);
    } else {
      uint8_t b[4] = {byte_at(off + 4 * i), byte_at(off + 4 * i + 1), byte_at(off + 4 * i + 2),
                      byte_at(off + 4 * i + 3)};
      memcpy(&out[i], b, 4);
    }
  }
  bool all_zero = true;
  for (uint32_t i = 0; i < D; i++) {
    if (!std::isfinite(out[i])) {
      for (uint32_t j = 0; j < D; j++) out[j] = 1.0f;
      return;
    }
    if (out[i] != 0.0f) all_zero = false;
  }
  if (all_zero)
    for (uint32_t i = 0; i < D; i++) out[i] = 1.0f;
}

// chpe_engine.zig:1172-1192 unpackBias.
void Engine::unpack_bias(uint64_t tile, float* out, uint32_t n) const {
  if (!f_.archive_valid || tile >= f_.record_count) {
    for (uint32_t i = 0; i < n; i++) out[i] = 0.f;
    return;
  }
  uint64_t off = code_off(tile);
  auto byte_at = [&](uint64_t o) -> uint8_t { return o < len_ ? host_[o] : 0; };
  for (uint32_t i = 0; i < n; i++) {
    if (arch_->D == 4096 && f_.is_raw) {
      uint32_t b = (uint32_t)byte_at(off + 2 * i) | ((uint32_t)byte_at(off + 2 * i + 1) << 8);
      uint32_t bits = b << 16;
      memcpy(&out[i], &bits, 4);
    } else {
      uint8_t b[4] = {byte_at(off + 4 * i), byte_at(off + 4 * i + 1), byte_at(off + 4 * i + 2),
                      byte_at(off + 4 * i + 3)};
      memcpy(&out[i], b, 4);
    }
    if (!std::isfinite(out[i])) out[i] = 0.f;
  }
}

const float* Engine::upload_floats(const std::vector<float>& v) {
  float* d = nullptr;
  CK(cudaMalloc(&d, v.size() * sizeof(float)));
  allocs_.push_back(d);
  CK(cudaMemcpy(d, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
  return d;
}

// Copies archive bytes [src_off, src_off + n) to device memory at dst
// through two pinned staging buffers.
static void stage_upload(uint8_t* dst, const uint8_t* bytes, uint64_t src_off, uint64_t n, cudaStream_t s) {
  const uint64_t chunk = 64ull << 20;
  uint8_t* stage[2] = {nullptr, nullptr};
  cudaEvent_t ev[2];
  CK(cudaMallocHost(&stage[0], chunk));
  CK(cudaMallocHost(&stage[1], chunk));
  CK(cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming));
  CK(cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming));
  int i = 0;
  for (uint64_t off = 0; off < n; off += chunk, i ^= 1) {
    const uint64_t m = n - off < chunk ? n - off : chunk;
    CK(cudaEventSynchronize(ev[i]));
    memcpy(stage[i], bytes + src_off + off, m);
    CK(cudaMemcpyAsync(dst + off, stage[i], m, cudaMemcpyHostToDevice, s));
    CK(cudaEventRecord(ev[i], s));
  }
  CK(cudaStreamSynchronize(s));
  cudaFreeHost(stage[0]);
  cudaFreeHost(stage[1]);
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
}

// The whole archive verbatim, plus a zeroed tail so reads past the last
// record stay inside the allocation.
void Engine::upload_archive(const uint8_t* bytes, uint64_t len) {
  const uint64_t pad = 1ull << 20;
  CK(cudaMalloc(&d_arc_, len + pad));
  CK(cudaMemsetAsync(d_arc_ + len, 0, pad, stream_));
  stage_upload(d_arc_, bytes, 0, len, stream_);
  dev_arc_bytes_ = len;
}

// Tensor parallelism: the tiles this rank's kernels read (chpe_tp_tile_runs:
// the embedding records and two more, and every projection's row slice),
// one allocation per run.  Norms and biases are read on the host.
void Engine::upload_shards(const uint8_t* bytes, uint64_t len) {
  const uint64_t rc = f_.record_count, wpt = f_.is_raw ? f_.wpt : 32768ull;
  const int64_t nr = chpe_tp_tile_runs(arch_id_, f_.is_raw, wpt, rc, tp_rank_, tp_world_, nullptr, 0);
  if (nr < 0) {
    upload_archive(bytes, len);  // the step builder reports the unsplittable shape
    return;
  }
  std::vector<uint64_t> rv(2 * (size_t)nr);
  chpe_tp_tile_runs(arch_id_, f_.is_raw, wpt, rc, tp_rank_, tp_world_, rv.data(), (size_t)nr);
  std::vector<std::pair<uint64_t, uint64_t>> runs;
  for (int64_t i = 0; i < nr; i++) runs.push_back({rv[2 * i], rv[2 * i + 1]});
  const uint64_t pad = 1ull << 20;
  for (const auto& r : runs) {
    const uint64_t off = 4096 + r.first * f_.stride;
    uint64_t n = (r.second - r.first) * f_.stride;
    if (off + n > len) n = len > off ? len - off : 0;
    Shard sh{r.first, r.second, nullptr};
    CK(cudaMalloc(&sh.dev, n + pad));
    CK(cudaMemsetAsync(sh.dev + n, 0, pad, stream_));
    stage_upload(sh.dev, bytes, off, n, stream_);
    dev_arc_bytes_ += n;
    shards_.push_back(sh);
  }
}

const uint8_t* Engine::arc_for(uint64_t tile) const {
  if (shards_.empty()) return d_arc_;
  for (const Shard& sh : shards_)
    if (tile >= sh.lo && tile < sh.hi) return sh.dev - (4096 + sh.lo * f_.stride);
  throw std::runtime_error("tensor parallel: a kernel would read a tile this rank did not upload");
}

// ---- construction: CHPEEngine.init (chpe_engine.zig:854-974) ---------------
Engine::Engine(const uint8_t* bytes, uint64_t len, int arch, uint32_t max_seq, int device, int tp_rank,
               int tp_world)
    : arch_(chpe_arch_preset(arch)), arch_id_(arch), device_(device), max_seq_(max_seq),
      host_(bytes), len_(len), tp_rank_(tp_rank), tp_world_(tp_world) {
  if (!arch_) throw std::runtime_error("unknown architecture id");
  if (max_seq_ == 0) throw std::runtime_error("max_seq_len must be > 0");
  if (tp_world < 1 || tp_world > kTpMax || tp_rank < 0 || tp_rank >= tp_world)
    throw std::runtime_error("tensor parallel rank/world out of range (world 1..8)");
  // format sniffing, :869-898
  if (len >= 4096) {
    uint32_t magic = rd32(bytes);
    if (magic == CHPE_CHPE_MAGIC || magic == CHPE_ARCHIVE_MAGIC) {
      f_.archive_valid = 1;
      f_.record_count = rd64(bytes + 16);
      uint64_t rec_b = rd64(bytes + 32), cell_b = rd64(bytes + 40), pre_b = rd64(bytes + 48),
               flags = rd64(bytes + 56);
      f_.is_dense = pre_b == 0 && rec_b == cell_b && rec_b == CHPE_CELL_BYTES;
      f_.is_raw = rec_b == CHPE_TILE_CODE_BYTES;
      f_.is_raw_fp16 = f_.is_raw && (flags & CHPE_FLAG_RAW_FP16) != 0;
      if (f_.is_raw_fp16) {
        f_.quant_bits = 16;
      } else if (f_.is_raw) {
        bool name9b = strstr(arch_->name, "9B") != nullptr;
        bool sized = len < 10ull * 1024 * 1024 * 1024 && len > 7ull * 1024 * 1024 * 1024;
        f_.quant_bits = (name9b && ((flags & 0x08) != 0 || sized)) ? 8 : 16;
      } else if (f_.record_count > 0 && len >= 4096 + (f_.is_dense ? CHPE_CELL_BYTES : CHPE_RECORD_BYTES)) {
        uint64_t cell_off = 4096 + (f_.is_dense ? 0 : CHPE_PREFETCH_BYTES);
        f_.quant_bits = bytes[cell_off + CHPE_PAYLOAD_OFF + 20];
        if (f_.quant_bits == 0) f_.quant_bits = 2;
      }
    }
  }
  f_.stride = f_.is_raw ? CHPE_TILE_CODE_BYTES : (f_.is_dense ? CHPE_CELL_BYTES : CHPE_RECORD_BYTES);
  if (f_.is_raw_fp16 || (f_.is_raw && f_.quant_bits == 16)) f_.wpt = 8192;
  else if (f_.quant_bits == 8) f_.wpt = 16384;
  else if (f_.quant_bits == 4 || f_.quant_bits == 2) f_.wpt = 32768;
  else f_.wpt = 8192;
  // Records the header promises but the bytes do not hold are never read:
  // the C ABI validates first; a raw engine over short bytes clamps here.
  if (f_.archive_valid) {
    uint64_t avail = len > 4096 ? (len - 4096) / f_.stride : 0;
    if (f_.record_count > avail) f_.record_count = avail;
  }

  if (const char* wp = getenv("CHPE_WAIT_POLLS")) wait_polls_ = (uint32_t)strtoul(wp, nullptr, 10);
  CK(cudaSetDevice(device_));
  CK(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device_));
  CK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));

  if (tp_world_ > 1 && f_.archive_valid && f_.record_count > 0) upload_shards(bytes, len);
  else upload_archive(bytes, len);

  const ChpeArch& A = *arch_;
  auto dalloc = [&](size_t bytes_) -> void* {
    void* p = nullptr;
    CK(cudaMalloc(&p, bytes_ < 256 ? 256 : bytes_));
    CK(cudaMemset(p, 0, bytes_ < 256 ? 256 : bytes_));
    allocs_.push_back(p);
    return p;
  };
  uint32_t maxproj = A.D;
  if (A.H * A.HD > maxproj) maxproj = A.H * A.HD;
  if (A.F > maxproj) maxproj = A.F;
  // Exchange region: everything another tensor-parallel rank reads or writes
  // (one allocation, so one CUDA IPC handle maps it).
  {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t attn_n = (size_t)(A.H * A.HD > A.D ? A.H * A.HD : A.D);
    size_t off = 0;
    const size_t o_st = off; off += al(sizeof(StepState));
    const size_t o_sh = off; off += al(sizeof(TpShared));
    const size_t o_hid = off; off += al((size_t)A.D * 4);
    const size_t o_attn = off; off += al(attn_n * 4);
    const size_t o_mlp = off; off += al((size_t)A.F * 4);
    const size_t o_log = off; off += al((size_t)A.V * 4);
    region_bytes_ = off;
    CK(cudaMalloc(&d_region_, region_bytes_));
    CK(cudaMemset(d_region_, 0, region_bytes_));
    d_st_ = (StepState*)(d_region_ + o_st);
    d_tpsh_ = (TpShared*)(d_region_ + o_sh);
    d_hidden_ = (float*)(d_region_ + o_hid);
    d_attn_ = (float*)(d_region_ + o_attn);
    d_mlp_ = (float*)(d_region_ + o_mlp);
    d_logits_ = (float*)(d_region_ + o_log);
  }
  d_q_ = (float*)dalloc((size_t)A.H * A.HD * 4);
  d_k_ = (float*)dalloc((size_t)A.KV * A.HD * 4);
  d_v_ = (float*)dalloc((size_t)A.KV * A.HD * 4);
  d_tmp_ = (float*)dalloc(maxproj * 4);
  d_tmp2_ = (float*)dalloc(maxproj * 4);
  d_xn_ = (float*)dalloc(maxproj * 4);
  const int G = A.H / A.KV;
  nsplit_ = attn_splits(num_sms_, (int)A.KV, (int)max_seq_);
  d_part_ = (float*)dalloc((size_t)A.KV * kAttnMaxSplits * G * (A.HD + 4) * 4);
  d_counters_ = (uint32_t*)dalloc(A.KV * 4);
  // row sums of the column parts of the row-block GEMV, and its arrival
  // counters and abort flags (two per row range)
  rb_part_cap_ = (uint64_t)kRbMaxParts * maxproj;
  d_rb_part_ = (float*)dalloc(rb_part_cap_ * 4);
  d_rb_cnt_ = (uint32_t*)dalloc(2u * 1024u * 4u);
  // Paged KV cache: per layer a pool of n_pages pages of kKvPage positions of
  // this rank's kv heads; the page table starts all-zero (page 0) and the
  // free list hands out pages 0, 1, 2, ... unless an order is set.
  kv0_ = 0;
  kvl_ = A.KV;
  if (tp_world_ > 1) {
    ChpeTpSlice sl;
    if (chpe_tp_slice_of(arch_id_, tp_rank_, tp_world_, &sl) == 0) {
      kv0_ = sl.kv0;
      kvl_ = sl.kvl;
    }
  }
  n_pages_ = (max_seq_ + kKvPage - 1) / kKvPage;
  layer_kv_elems_ = (size_t)n_pages_ * kKvPage * kvl_ * A.HD;
  d_kc_ = (__half*)dalloc((size_t)A.L * layer_kv_elems_ * 2);
  d_vc_ = (__half*)dalloc((size_t)A.L * layer_kv_elems_ * 2);
  d_pages_ = (uint32_t*)dalloc((size_t)n_pages_ * 4);
  CK(cudaMallocHost(&h_pages_, (size_t)n_pages_ * 4));
  memset(h_pages_, 0, (size_t)n_pages_ * 4);
  free_pages_.clear();
  for (uint32_t i = n_pages_; i-- > 0;) free_pages_.push_back(i);
  d_res_ = (StepResult*)dalloc(sizeof(StepResult));
  max_gen_ = max_seq_;
  d_gen_ = (int32_t*)dalloc((size_t)max_gen_ * 4);
  CK(cudaMallocHost(&h_st_, sizeof(StepState)));
  CK(cudaMallocHost(&h_res_, sizeof(StepResult)));
  h_tok_cap_ = max_seq_ + 1;
  CK(cudaMallocHost(&h_tok_, h_tok_cap_ * 4));
  memset(h_st_, 0, sizeof(StepState));
  h_st_->finite = 1;
  h_st_->gather = 1;
  CK(cudaMemcpy(d_st_, h_st_, sizeof(StepState), cudaMemcpyHostToDevice));
  // RoPE inverse frequencies, computed as applyRope does (chpe_engine.zig:200-202)
  std::vector<float> invf(A.HD / 2);
  for (uint32_t i = 0; i < A.HD / 2; i++) {
    float fe = 2.0f * (float)i / (float)A.HD;
    invf[i] = 1.0f / powf(A.theta, fe);
  }
  d_invfreq_ = const_cast<float*>(upload_floats(invf));

  ops_ = new std::vector<Op>();
  if (tp_world_ == 1) build_step();  // tensor parallel: after tp_connect
}

Engine::~Engine() {
  free_batch_steps();
  if (graph_) cudaGraphExecDestroy(graph_);
  if (d_vlogits_) cudaFree(d_vlogits_);
  if (d_vres_) cudaFree(d_vres_);
  for (void* p : ipc_open_) cudaIpcCloseMemHandle(p);
  if (d_region_) cudaFree(d_region_);
  for (void* p : allocs_) cudaFree(p);
  if (d_arc_) cudaFree(d_arc_);
  for (const Shard& sh : shards_) cudaFree(sh.dev);
  if (h_st_) cudaFreeHost(h_st_);
  if (h_res_) cudaFreeHost(h_res_);
  if (h_tok_) cudaFreeHost(h_tok_);
  if (h_pages_) cudaFreeHost(h_pages_);
  if (stream_) cudaStreamDestroy(stream_);
  delete ops_;
}

// ---- planning one gemvLinear call site -------------------------------------
GemvSrc Engine::plan_linear(uint64_t tile_start, uint64_t num_tiles, uint32_t r_total,
                            uint32_t c_total, uint32_t x_len, int accumulate, int64_t bias_tile) {
  GemvSrc s{};
  s.r_total = r_total;
  s.c_total = c_total;
  s.x_len = x_len;
  s.arc = d_arc_;
  if (!f_.archive_valid || tile_start >= f_.record_count) {
    s.kind = accumulate ? SRC_NOOP : SRC_PATTERN;
    return s;
  }
  uint64_t avail = num_tiles < f_.record_count - tile_start ? num_tiles : f_.record_count - tile_start;
  s.n_tiles = (uint32_t)avail;
  s.tile0 = code_off(tile_start);
  s.stride = f_.stride;
  if (bias_tile >= 0 && (uint64_t)bias_tile < f_.record_count) {
    std::vector<float> b(r_total);
    unpack_bias((uint64_t)bias_tile, b.data(), r_total);
    s.bias = upload_floats(b);
  }
  if (f_.is_raw) {
    s.kind = SRC_RAW;
    s.fmt = f_.is_raw_fp16 ? FMT_F16 : (f_.quant_bits == 8 ? FMT_I8RAW : FMT_BF16);
    s.flat_limit = avail * f_.wpt;
    if (c_total % fmt_cw(s.fmt) != 0) throw std::runtime_error("raw tensor width not a multiple of the chunk width");
    return s;
  }
  const uint8_t* base = host_;
  auto cell_code = [&](uint64_t t) { return base + code_off(tile_start + t); };
  if (c_total > 2048) {  // gemvCellFlat, wpt 32768
    s.flat_limit = avail * 32768ull;
    uint64_t need = ((uint64_t)r_total * c_total + 32767) / 32768;
    uint64_t used = need < avail ? need : avail;
    int fmt = -1;
    bool uniform = true;
    for (uint64_t t = 0; t < used; t++) {
      const uint8_t* pl = cell_code(t) + 16384;
      uint32_t qb = pl[20];
      bool g = (rd64(pl + 24) & 1u) != 0;
      int f = qb == 4 ? (g ? FMT_W4G : FMT_W4SB) : qb == 2 ? (g ? FMT_W2G : FMT_W2SB) : FMT_ZERO;
      if (fmt < 0) fmt = f;
      if (f != fmt) uniform = false;
      uint32_t n = rd16(pl + 560);
      if (n > 0 && n <= 64) s.has_aux = 1;
    }
    if (fmt < 0) fmt = FMT_ZERO;
    s.fmt = fmt;
    bool fast = uniform && fmt != FMT_ZERO && (c_total % fmt_cw(fmt)) == 0;
    s.kind = fast ? SRC_FLAT : SRC_GEN_FLAT;
    return s;
  }
  // row-tiled cells (gemvTilePolymorphic), row_base prefix with the
  // reference's stop conditions (:1430-1442)
  std::vector<uint32_t> cells, rowsv;
  uint64_t row_base = 0;
  for (uint64_t t = 0; t < avail; t++) {
    if (row_base >= r_total) break;
    uint32_t rows = rd32(cell_code(t) + 16384 + 40);
    if (rows == 0) break;
    cells.push_back((uint32_t)t);
    rowsv.push_back(rows);
    row_base += rows;
  }
  uint32_t covered = (uint32_t)(row_base < r_total ? row_base : r_total);
  s.rows_covered = covered;
  int fmt = -1;
  bool uniform = !cells.empty();
  uint32_t crow = 0, ccol = 0;
  bool outl = false;
  for (size_t i = 0; i < cells.size(); i++) {
    const uint8_t* pl = cell_code(cells[i]) + 16384;
    uint32_t qb = pl[20];
    uint64_t fl = rd64(pl + 24);
    bool g = (fl & 1u) != 0;
    int f;
    switch (qb) {
      case 4: f = g ? FMT_W4G : FMT_W4SB; break;
      case 8: f = FMT_W8; break;
      case 16: f = (fl & CHPE_FLAG_RAW_FP16) ? FMT_F16 : FMT_BF16; break;
      case 32: f = FMT_F32; break;
      default: f = g ? FMT_W2G : FMT_W2SB; break;
    }
    uint32_t rows = rd32(pl + 40), cols = rd32(pl + 44);
    if (i == 0) { fmt = f; crow = rows; ccol = cols; outl = g && rows == 16; }
    if (f != fmt || rows != crow || cols != ccol) uniform = false;
  }
  s.fmt = fmt < 0 ? FMT_W4G : fmt;
  s.cell_rows = crow;
  s.cell_cols = ccol;
  // the fast row-tiled kernel takes full cells of 2048 columns
  const uint32_t full_rows = fmt == FMT_F16 || fmt == FMT_BF16 ? 4u : 16u;
  bool fast = uniform && fmt != FMT_W8 && fmt != FMT_F32 && ccol == 2048 && c_total == 2048 &&
              x_len == 2048 && crow == full_rows;
  if (fast) {
    s.kind = SRC_ROWTILE;
    s.outliers = (outl && (fmt == FMT_W4G || fmt == FMT_W2G)) ? OUTL_ADD : OUTL_NONE;
    if (s.outliers == OUTL_ADD) {
      // An additive outlier term whose 128 weights are all +0.0 adds exactly
      // 0 for finite x, so such tensors skip it.  (With an inf/NaN x the
      // reference's term would give NaN; the main dot is then non-finite too.)
      bool any = false;
      for (size_t i = 0; i < cells.size() && !any; i++) {
        const uint8_t* pl = cell_code(cells[i]) + 16384;
        for (int b = 560; b < 816 && !any; b++) any = pl[b] != 0;
      }
      if (!any) s.outliers = OUTL_NONE;
    }
    return s;
  }
  // per-row table for the generic kernel; every byte it may touch must lie
  // inside the uploaded archive plus its zeroed tail
  for (size_t i = 0; i < cells.size(); i++) {
    const uint8_t* pl = cell_code(cells[i]) + 16384;
    uint32_t qb = pl[20];
    uint64_t rows = rd32(pl + 40), cols = rd32(pl + 44);
    uint64_t bits = qb == 4 ? 4 : qb == 8 ? 8 : qb == 16 ? 16 : qb == 32 ? 32 : 2;
    uint64_t last = code_off(tile_start + cells[i]) + rows * cols * bits / 8 + 16384 + 2 * rows * cols / 128 + 1024;
    if (cols > (1u << 20) || last > len_ + (1ull << 20))
      throw std::runtime_error("cell geometry reaches outside the archive");
  }
  s.kind = SRC_GEN_ROWTILE;
  std::vector<uint32_t> rc(r_total, 0xFFFFFFFFu);
  std::vector<uint16_t> ri(r_total, 0);
  uint64_t rb = 0;
  for (size_t i = 0; i < cells.size(); i++) {
    for (uint32_t r = 0; r < rowsv[i] && rb + r < r_total; r++) {
      rc[rb + r] = cells[i];
      ri[rb + r] = (uint16_t)r;
    }
    rb += rowsv[i];
  }
  uint32_t* drc = nullptr;
  uint16_t* dri = nullptr;
  CK(cudaMalloc(&drc, rc.size() * 4));
  CK(cudaMalloc(&dri, ri.size() * 2 + 16));
  allocs_.push_back(drc);
  allocs_.push_back(dri);
  CK(cudaMemcpy(drc, rc.data(), rc.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dri, ri.data(), ri.size() * 2, cudaMemcpyHostToDevice));
  s.row_cell = drc;
  s.row_in_cell = dri;
  return s;
}

static bool is_fast(const GemvSrc& s) {
  return s.kind == SRC_RAW || s.kind == SRC_ROWTILE || s.kind == SRC_FLAT;
}

static size_t gemv_smem(int fmt, uint32_t ncols) {
  uint32_t cw = fmt_cw(fmt);
  uint32_t nchunks = (ncols + cw - 1) / cw;
  uint32_t nslots = (nchunks + 31) / 32;
  // x staged per lane slot, then one x-sum per (padded) chunk slot
  return ((size_t)nslots * 32 * cw + (size_t)nslots * 32 + 4) * sizeof(float);
}

static uint64_t weight_bytes(const GemvSrc& s) {
  if (s.kind == SRC_RAW) {
    uint64_t w = (uint64_t)s.r_total * s.c_total;
    if (w > s.flat_limit) w = s.flat_limit;
    return w * (s.fmt == FMT_I8RAW ? 1 : 2);
  }
  if (s.kind == SRC_FLAT) {
    uint64_t need = ((uint64_t)s.r_total * s.c_total + 32767) / 32768;
    if (need > s.n_tiles) need = s.n_tiles;
    return need * s.stride;
  }
  if (s.kind == SRC_ROWTILE) {
    uint64_t cells = (s.rows_covered + s.cell_rows - 1) / s.cell_rows;
    return cells * s.stride;
  }
  return 0;
}

// Algorithmic bytes of a call site: the codes and scales of the weights it
// actually needs (rows < r_total), no padding, metadata or unused tiles.
static double alg_bytes_of(const GemvSrc& s) {
  double w = (double)s.r_total * s.c_total;
  if (s.kind == SRC_ROWTILE) w = (double)s.rows_covered * s.c_total;
  if (s.kind == SRC_FLAT || s.kind == SRC_RAW) {  // weights of rows row0.. that the tiles hold
    const double first = (double)s.row0 * s.c_total;
    const double avail = (double)s.flat_limit > first ? (double)s.flat_limit - first : 0.0;
    if (w > avail) w = avail;
  }
  switch (s.fmt) {
    case FMT_W4G: return w * 0.5 + w / 128.0 * 2.0;
    case FMT_W2G: return w * 0.25 + w / 128.0 * 2.0;
    case FMT_W4SB: return w * 0.5;
    case FMT_W2SB: return w * 0.25;
    case FMT_W8: case FMT_I8RAW: return w;
    case FMT_F16: case FMT_BF16: return w * 2.0;
    case FMT_F32: return w * 4.0;
  }
  return 0.0;
}

void Engine::add_linear_ops(std::vector<Op>& ops, const GemvSrc* src_in, float* const* out, int nseg,
                            int epi, const float* x, const float* gamma, int check_layer,
                            uint32_t ncols, bool ignore_stop, const TpLink* tp) {
  const bool tp_on = tp && tp->world > 1;
  // A row-tiled 2/4-bit cell of 16 rows x 2048 columns has the byte layout of
  // a flat 32768-weight cell read at 2048 columns (codes row-major, group
  // scale of (row, col) at 48 + 2*(row*16 + col/128)).  Without additive
  // outliers and with every row covered, such tensors can take the flat
  // kernel's aligned-cell mode; opt-in (CHPE_ROWTILE_AS_FLAT=1), as the
  // row-block kernel measured faster on the 3B shapes.
  GemvSrc srcv[3] = {};
  const char* raf = getenv("CHPE_ROWTILE_AS_FLAT");
  bool as_flat = nseg <= 3 && raf && raf[0] == '1';
  for (int i = 0; i < nseg && as_flat; i++) {
    const GemvSrc& g = src_in[i];
    as_flat = g.kind == SRC_ROWTILE &&
              (g.fmt == FMT_W4G || g.fmt == FMT_W4SB || g.fmt == FMT_W2G || g.fmt == FMT_W2SB) &&
              g.cell_rows == 16 && g.cell_cols == 2048 && g.c_total == 2048 && ncols == 2048 &&
              g.outliers == OUTL_NONE && g.rows_covered == g.r_total && g.r_total % 16 == 0;
  }
  for (int i = 0; i < nseg && i < 3; i++) {
    srcv[i] = src_in[i];
    if (as_flat) {
      srcv[i].kind = SRC_FLAT;
      srcv[i].n_tiles = srcv[i].r_total / 16;
      srcv[i].flat_limit = (uint64_t)srcv[i].n_tiles * 32768ull;
      srcv[i].has_aux = 0;
      srcv[i].row0 = 0;
    }
  }
  const GemvSrc* src = nseg <= 3 ? srcv : src_in;
  const ChpeArch& A = *arch_;
  bool fused = true;
  for (int i = 0; i < nseg; i++) {
    if (!is_fast(src[i]) || src[i].kind != src[0].kind || src[i].fmt != src[0].fmt) fused = false;
    if (epi == EPI_SWIGLU && src[i].has_aux) fused = false;
    if (epi == EPI_SWIGLU && src[i].r_total != src[0].r_total) fused = false;
  }
  bool logits_aux = epi == EPI_LOGITS && src[0].has_aux;
  if (logits_aux) fused = false;

  auto make_gemv = [&](const GemvSrc* ss, float* const* oo, int n, int e, const float* xx,
                       const float* gg, int chk) {
    Op op;
    op.type = OP_GEMV;
    op.fmt = ss[0].fmt;
    op.kind = ss[0].kind;
    GemvLaunch& g = op.g;
    g.nseg = n;
    g.epi = e;
    uint32_t rows = 0;
    for (int i = 0; i < n; i++) {
      g.src[i] = ss[i];
      g.out[i] = oo[i];
      g.row_start[i] = rows;
      rows += ss[i].r_total;
      g.prefetch_bytes[i] = weight_bytes(ss[i]);
      g.prefetch_base[i] = d_arc_ + ss[i].tile0;
    }
    g.row_start[n] = rows;
    if (e == EPI_SWIGLU) { g.out[0] = oo[0]; g.row_start[1] = ss[0].r_total; }
    g.x = xx;
    g.gamma = gg;
    g.norm = gg != nullptr;
    g.eps = A.eps;
    g.ncols = ncols;
    g.check_layer = chk;
    g.st = d_st_;
    g.ignore_stop = ignore_stop;
    g.res = d_res_;
    g.gen_tokens = d_gen_;
    g.max_gen = (int32_t)max_gen_;
    for (int i = 0; i < n; i++)
      if (ss[i].has_aux) g.xn_out = d_xn_;
    size_t sm = gemv_smem(op.fmt, ncols);
    op.smem = sm;
    uint32_t jobs = e == EPI_SWIGLU ? ss[0].r_total : rows;
    // jobs a warp takes per iteration (gemv_nr)
    uint32_t jpi = (uint32_t)gemv_nr(op.fmt, op.kind);
    if (e == EPI_SWIGLU) jpi /= 2;
    if (sm > 16384) {
      op.threads = 512;
      uint32_t cap = (uint32_t)num_sms_;
      uint32_t need = (jobs + 16 * jpi - 1) / (16 * jpi);
      op.grid = dim3(need < cap ? need : cap);
    } else {
      op.threads = 256;
      uint32_t cap = (uint32_t)num_sms_ * 2u;
      uint32_t need = (jobs + 8 * jpi - 1) / (8 * jpi);
      op.grid = dim3(need < cap ? need : cap);
    }
    if (op.grid.x == 0) op.grid.x = 1;
    return op;
  };
  auto push_aux = [&](const GemvSrc& s, float* y, const float* xx) {
    if (!s.has_aux || s.kind != SRC_FLAT) return;
    Op op;
    op.type = OP_AUX;
    op.aux.src = s;
    op.aux.y = y;
    op.aux.x = xx;
    op.aux.st = ignore_stop ? nullptr : d_st_;
    uint64_t n = (uint64_t)s.n_tiles * 64;
    op.grid = dim3((uint32_t)((n + 255) / 256));
    op.threads = 256;
    ops.push_back(op);
  };

  // Row-block tensors (full 2048-wide rows, contiguous codes) go through the
  // TMA-pipelined kernel.
  auto tma_rows = [&](const GemvSrc& g) -> uint32_t {  // rows per block, 0 = not eligible
    if (ncols != 2048 || g.c_total != 2048) return 0;
    if (g.kind == SRC_ROWTILE) {
      uint32_t R = (g.fmt == FMT_F16 || g.fmt == FMT_BF16) ? 4u
                   : (g.fmt == FMT_W4G || g.fmt == FMT_W4SB || g.fmt == FMT_W2G || g.fmt == FMT_W2SB) ? 16u : 0u;
      if (!R || g.cell_rows != R || g.rows_covered != g.r_total || g.r_total % R) return 0;
      return R;
    }
    if (g.kind == SRC_RAW && (g.fmt == FMT_F16 || g.fmt == FMT_BF16) && g.stride == 16384 &&
        g.r_total % 4 == 0 && g.flat_limit >= (uint64_t)g.r_total * 2048)
      return 4;
    return 0;
  };
  // Flat cells and raw streams of any width go through the warp-specialised
  // flat TMA kernel when every segment is covered in full.
  auto flat_ok = [&](const GemvSrc& g) -> bool {
    const int f = g.fmt;
    uint32_t wpp;
    if (g.kind == SRC_FLAT && (f == FMT_W4G || f == FMT_W4SB || f == FMT_W2G || f == FMT_W2SB)) wpp = 32768;
    else if (g.kind == SRC_RAW && (f == FMT_F16 || f == FMT_BF16 || f == FMT_I8RAW)) wpp = 16384u * 8u / (uint32_t)fmt_bits(f);
    else return false;
    const uint32_t cw = (uint32_t)fmt_cw(f);
    const uint64_t w = (uint64_t)(g.row0 + g.r_total) * g.c_total;
    // a consumer warp's run of a piece (wpp/cw/16 chunks) spans at most two rows
    if (gamma && ncols > 16384) return false;  // the fused RMSNorm loads x in one batch
    return g.c_total == ncols && ncols % cw == 0 && (wpp / cw / kFlatConsumerWarps) * cw <= ncols &&
           w < (1ull << 32) && g.r_total > 0;
  };
  bool tma = fused && !getenv("CHPE_NO_TMA");
  bool flat = tma && !getenv("CHPE_NO_FLAT_TMA");
  for (int i = 0; i < nseg && flat; i++) flat = flat_ok(src[i]);
  if (flat) {
    Op op;
    op.type = OP_FLAT_TMA;
    op.fmt = src[0].fmt;
    op.kind = src[0].kind;
    op.threads = (int)kFlatThreads;
    op.role = epi == EPI_SWIGLU ? ROLE_GATEUP : epi == EPI_LOGITS ? ROLE_LMHEAD
              : (epi == EPI_ACCUM ? (ncols == arch_->D ? ROLE_O : ROLE_DOWN) : ROLE_QKV);
    FlatTmaLaunch& t = op.fl;
    uint32_t rows = 0;
    for (int i = 0; i < nseg; i++) {
      t.src[i] = src[i];
      t.out[i] = out[i];
      t.row_start[i] = rows;
      rows += src[i].r_total;
      op.alg_bytes += alg_bytes_of(src[i]);
    }
    t.row_start[nseg] = rows;
    if (epi == EPI_SWIGLU) t.row_start[1] = src[0].r_total;
    const uint32_t Rt = epi == EPI_SWIGLU ? src[0].r_total : rows;
    // per segment, its leading rows with any weight in the tiles (the rest
    // read as zero: the reference's flat loops stop at the available tiles)
    for (int i = 0; i < nseg; i++) {
      const uint64_t start = (uint64_t)src[i].row0 * ncols, lim = src[i].flat_limit;
      const uint64_t c = lim <= start ? 0 : (lim - start + ncols - 1) / ncols;
      t.cov[i] = (uint32_t)(c < src[i].r_total ? c : src[i].r_total);
    }
    if (epi == EPI_SWIGLU && t.cov[1] > t.cov[0]) t.cov[0] = t.cov[1];
    // Aligned cells (rows start at cell boundaries): 4/2-bit flat cells whose
    // width divides 32768 into 32..256 column chunks, every segment a whole
    // number of cells.
    uint32_t rc = 0;
    // Raw FP16 / BF16 / int8 streams the same, with their 16 KiB tiles as cells.
    {
      const uint32_t cw = (uint32_t)fmt_cw(op.fmt);
      const bool raw_ok = op.kind == SRC_RAW && (op.fmt == FMT_F16 || op.fmt == FMT_BF16 || op.fmt == FMT_I8RAW);
      const uint32_t wpp = op.kind == SRC_FLAT ? 32768u : 16384u * 8u / (uint32_t)fmt_bits(op.fmt);
      bool al = (op.kind == SRC_FLAT || raw_ok) && wpp % ncols == 0 && (ncols / cw) % 32u == 0 &&
                ncols / cw <= kFlatConsumers && kFlatConsumers % (ncols / cw) == 0 && !getenv("CHPE_NO_ALIGNED");
      const uint32_t cell_rows = wpp / ncols;
      for (int i = 0; i < nseg && al; i++)
        al = src[i].r_total % cell_rows == 0 && src[i].row0 % cell_rows == 0;
      if (al) rc = cell_rows;
    }
    // Tensor-core mode: aligned 4-bit group-scaled cells of 4096 or 8192
    // columns, every segment whole 16-row blocks and fully present (no rows
    // cut by the archive's end).  Taken for 8192 columns, and for 4096 when a
    // CTA gets 32 blocks or more (the LM head): measured on B200, the FFMA
    // decode of the two-CTA aligned mode is faster on the 9B's shorter
    // 4096-column launches (QKV, O, gate/up).  CHPE_FLAT_MMA=0 keeps the
    // FFMA decode everywhere, =1 takes the tensor cores wherever they apply.
    bool mma = false;
    {
      const char* e = getenv("CHPE_FLAT_MMA");
      const bool off = e && e[0] == '0', all = e && e[0] == '1';
      const uint32_t blocks = Rt / kMmaRows;
      const bool big = blocks >= 32u * (uint32_t)num_sms_;
      mma = rc && op.fmt == FMT_W4G && op.kind == SRC_FLAT && (ncols == 4096 || ncols == 8192) && !off &&
            (all || ncols == 8192 || big);
      for (int i = 0; i < nseg && mma; i++)
        mma = src[i].r_total % kMmaRows == 0 && src[i].row0 % kMmaRows == 0 &&
              (uint64_t)(src[i].row0 + src[i].r_total) * ncols <= src[i].flat_limit;
      if (mma) {
        // two blocks in the ring at least; a partial slot for every block in flight
        const uint32_t u = Rt / kMmaRows, g = u < (uint32_t)num_sms_ ? u : (uint32_t)num_sms_;
        const uint32_t rpc = kMmaRows * ((u + g - 1) / g), np = epi == EPI_SWIGLU ? 2u : 1u;
        const uint32_t f = flat_layout_mma(ncols, rpc, np, 0).total;
        uint32_t n = kFlatSmemLimit > f ? (kFlatSmemLimit - f) / kFlatStageBytes : 0u;
        if (n > kFlatStagesWanted) n = kFlatStagesWanted;
        const uint32_t cpb = kMmaRows / rc;
        // two blocks in the ring, one of them outside the stages that stage B
        if (n < 2 * cpb || n < flat_mma_b_stages(ncols) + cpb || (n + cpb - 1) / cpb + 1 > kMmaSlots) mma = false;
      }
    }
    const uint32_t RU = mma ? kMmaRows : rc ? rc : 1u, Ut = Rt / RU;
    const uint32_t G = Ut < (uint32_t)num_sms_ ? Ut : (uint32_t)num_sms_;
    t.rc = rc;
    t.nseg = nseg;
    t.epi = epi;
    t.ncols = ncols;
    t.rpc = RU * ((Ut + G - 1) / G);
    t.x = x;
    t.gamma = gamma;
    t.norm = gamma != nullptr;
    t.eps = arch_->eps;
    t.check_layer = check_layer;
    t.st = d_st_;
    t.ignore_stop = ignore_stop;
    t.res = d_res_;
    t.gen_tokens = d_gen_;
    t.max_gen = (int32_t)max_gen_;
    t.xn_out = nullptr;
    for (int i = 0; i < nseg; i++)
      if (src[i].has_aux) t.xn_out = d_xn_;
    if (tp_on) t.tp = *tp;
    {
      // CHPE_FLAT_PREFETCH=n: at most n pieces requested before the
      // dependency wait (default: every free stage)
      const char* e = getenv("CHPE_FLAT_PREFETCH");
      t.npre = e ? (uint32_t)atoi(e) : 0u;
    }
    // Row blocks on the tensor cores (gemv_rowblk.cuh): 4-bit group-scaled
    // flat cells whose rows do not start at cell boundaries (the down
    // projections), one segment, no fused norm, no down_aux fix-ups, rows in
    // whole 8-row units and present in the tiles.  Taken on one GPU for rows
    // of more than one column part (the 72B's 231 groups: measured on B200
    // 50.0 us against 51.7 us for the column-owner FFMA decode); for the
    // 9B's 96 groups the column owners are faster (16.5 against 19.3 us),
    // and so they are for the 72B's tensor-parallel slices (46.1 against
    // 49.5 us per layer at 2 GPUs).  CHPE_FLAT_ROWBLK=0 keeps every call on
    // the FFMA decode, =1 takes the tensor cores wherever they apply.
    {
      const char* e = getenv("CHPE_FLAT_ROWBLK");
      const uint32_t G = ncols / 128u, ncp = (G + kRbPartGroups - 1) / kRbPartGroups;
      const bool want = e ? e[0] == '1' : (ncp > 1 && !tp_on);
      const bool rb = want && !rc && op.kind == SRC_FLAT && op.fmt == FMT_W4G && nseg == 1 &&
                      !gamma && (epi == EPI_ACCUM || epi == EPI_STORE) && ncols % 128u == 0 &&
                      src[0].r_total % kRbUnit == 0 && !src[0].has_aux && ncp <= kRbMaxParts &&
                      (uint64_t)ncp * src[0].r_total <= rb_part_cap_ &&
                      (uint64_t)(src[0].row0 + src[0].r_total) * ncols <= src[0].flat_limit;
      if (rb) {
        const uint32_t gpn = (G + ncp - 1) / ncp, Ut = src[0].r_total / kRbUnit;
        const uint32_t nrr = Ut < (uint32_t)num_sms_ / ncp ? Ut : (uint32_t)num_sms_ / ncp;
        const uint32_t rpc = kRbUnit * ((Ut + nrr - 1) / nrr);
        const RbLayout l0 = rowblk_layout(gpn, rpc, 0);
        uint32_t n = kFlatSmemLimit > l0.total ? (kFlatSmemLimit - l0.total) / l0.stage : 0u;
        if (n > kRbMaxStages) n = kRbMaxStages;
        // two 8-row blocks in the ring, one of them outside the B staging
        if (nrr >= 1 && n >= 2 * kRbUnit && n >= l0.nb + kRbUnit) {
          t.mode = FLAT_ROWBLK;
          t.rc = ncp;
          t.nw = gpn;
          t.nst = n;
          t.rpc = rpc;
          t.part_buf = d_rb_part_;
          t.part_cnt = d_rb_cnt_;
          op.threads = (int)kRbThreads;
          op.smem = rowblk_layout(gpn, rpc, n).total;
          op.grid = dim3(nrr * ncp);
          ops.push_back(op);
          return;
        }
      }
    }
    const uint32_t nparts = epi == EPI_SWIGLU ? 2u : 1u;
    const uint32_t cw = (uint32_t)fmt_cw(op.fmt);
    const uint32_t fixed = mma ? flat_layout_mma(ncols, t.rpc, nparts, 0).total
                               : flat_layout(ncols, cw, t.rpc, nparts, 0).total;
    const uint32_t budget = kFlatSmemLimit > fixed ? kFlatSmemLimit - fixed : 0u;
    uint32_t nst = budget / kFlatStageBytes;
    if (nst > kFlatStagesWanted) nst = kFlatStagesWanted;
    if (mma) {
      t.mode = FLAT_MMA;
      t.nw = kFlatConsumerWarps;
      t.nst = nst;
      op.smem = flat_layout_mma(ncols, t.rpc, nparts, nst).total;
      op.grid = dim3(G);
      ops.push_back(op);
      for (int i = 0; i < nseg; i++) push_aux(src[i], epi == EPI_SWIGLU ? nullptr : out[i], gamma ? d_xn_ : x);
      return;
    }
    // Aligned launches whose shared memory fits twice per SM run 8 consumer
    // warps per CTA and two CTAs per SM (grid up to twice the SMs).
    uint32_t nw = 16, G8 = 0, rpc8 = 0, nst8 = 0;
    {
      const char* one = getenv("CHPE_FLAT_ONE_CTA");
      // (8 warps: a row's chunks must fit the 256 consumer lanes)
      const uint32_t ncpr = ncols / (uint32_t)fmt_cw(op.fmt);
      if (rc && !(one && one[0] == '1') && (!gamma || ncols <= 8192) && ncpr <= 256u && 256u % ncpr == 0) {
        G8 = Ut < 2u * (uint32_t)num_sms_ ? Ut : 2u * (uint32_t)num_sms_;
        rpc8 = RU * ((Ut + G8 - 1) / G8);
        const uint32_t f8 = flat_layout(ncols, cw, rpc8, nparts, 0, 8).total;
        nst8 = kFlatSmemHalf > f8 ? (kFlatSmemHalf - f8) / kFlatStageBytes : 0u;
        if (nst8 > kFlatStagesWanted) nst8 = kFlatStagesWanted;
        if (nst8 >= 3) nw = 8;
      }
    }
    t.nw = nw;
    // Column owners: rows that do not start at cell boundaries with 384..960
    // 16-byte chunks (32 weights each; 384..480 for 64-weight chunks), so
    // that at least 4/5 of the first slots are busy (the down projections:
    // 924 chunks on the 72B, 384 on the 9B; the 3B's 344 measured faster in
    // the stream mode), or FP16/BF16 rows of 384..1440 chunks of 8 weights
    // with or without the fused norm (the 72B FP16 projections of 8192
    // columns; the stream mode's per-piece reduction over 16 weights per
    // lane held them near 2 TB/s).  x sits in registers, so the ring takes
    // the shared memory x would have used.  CHPE_FLAT_COLOWN=0 keeps such
    // calls on the stream mode.
    t.mode = rc ? FLAT_ALIGNED : FLAT_STREAM;
    {
      const uint32_t ncc = ncols / cw, sl = cw <= 8 ? 3u : cw <= 32 ? 2u : 1u, lanes = kFlatColownWarps * 32u;
      const char* co = getenv("CHPE_FLAT_COLOWN");
      const bool on = !(co && co[0] == '0');
      const uint32_t fixed_co = flat_layout(ncols, cw, t.rpc, nparts, 0, kFlatColownWarps, false).total;
      uint32_t nst_co = kFlatSmemLimit > fixed_co ? (kFlatSmemLimit - fixed_co) / kFlatStageBytes : 0u;
      if (nst_co > kFlatStagesWanted) nst_co = kFlatStagesWanted;
      // wider FP16 / BF16 rows: eight slots per lane (x in as many registers
      // as two slots of 32-weight chunks)
      const bool wide = op.kind == SRC_RAW && (op.fmt == FMT_F16 || op.fmt == FMT_BF16) && ncc > sl * lanes &&
                        ncc <= 8u * lanes;
      // the ring holds every piece of the rows one iteration decodes (4, or 2
      // in the eight-slot mode)
      const uint64_t span = (uint64_t)(wide ? 2u : 4u) * ncols * (uint64_t)fmt_bits(op.fmt) / 8u;
      const bool fits = (span + 16383u) / 16384u + 1u <= nst_co;
      if (on && fits && !rc && (!gamma || cw <= 8) && 5u * ncc >= 4u * lanes && (ncc <= sl * lanes || wide) &&
          nst_co >= 6) {
        t.mode = wide ? FLAT_COLOWN8 : FLAT_COLOWN;
        t.nw = kFlatColownWarps;
        op.threads = (int)kFlatColownThreads;
        nst = nst_co;
      }
    }
    if (nw == 8) {
      t.nst = nst8;
      t.rpc = rpc8;
      op.threads = (int)kFlatThreadsHalf;
      op.smem = flat_layout(ncols, cw, rpc8, nparts, nst8, 8).total;
      op.grid = dim3(G8);
      ops.push_back(op);
      for (int i = 0; i < nseg; i++) push_aux(src[i], epi == EPI_SWIGLU ? nullptr : out[i], gamma ? d_xn_ : x);
      return;
    }
    if (nst >= 2) {
      t.nst = nst;
      op.smem = flat_layout(ncols, cw, t.rpc, nparts, nst, t.nw, t.mode != FLAT_COLOWN && t.mode != FLAT_COLOWN8).total;
      op.grid = dim3(G);
      ops.push_back(op);
      for (int i = 0; i < nseg; i++) push_aux(src[i], epi == EPI_SWIGLU ? nullptr : out[i], gamma ? d_xn_ : x);
      return;
    }
  }
  if (tp_on) throw std::runtime_error("tensor parallel: a projection does not fit the flat TMA kernel");
  for (int i = 0; i < nseg && tma; i++) tma = tma_rows(src[i]) != 0;
  if (tma) {
    Op op;
    op.type = OP_TMA;
    op.fmt = src[0].fmt;
    op.kind = src[0].kind;
    op.threads = 512;
    op.role = epi == EPI_SWIGLU ? ROLE_GATEUP : epi == EPI_LOGITS ? ROLE_LMHEAD
              : (epi == EPI_ACCUM ? (ncols == arch_->D ? ROLE_O : ROLE_DOWN) : ROLE_QKV);
    TmaLaunch& t = op.tm;
    const uint32_t R = tma_rows(src[0]);
    uint32_t units = 0;
    for (int i = 0; i < nseg; i++) {
      t.src[i] = src[i];
      t.out[i] = out[i];
      t.unit_start[i] = units;
      units += src[i].r_total / R;
      op.alg_bytes += alg_bytes_of(src[i]);
    }
    t.unit_start[nseg] = units;
    if (epi == EPI_SWIGLU) t.unit_start[1] = src[0].r_total / R;
    t.nseg = nseg;
    t.epi = epi;
    t.x = x;
    t.gamma = gamma;
    t.norm = gamma != nullptr;
    t.eps = arch_->eps;
    t.check_layer = check_layer;
    t.st = d_st_;
    t.ignore_stop = ignore_stop;
    t.res = d_res_;
    t.gen_tokens = d_gen_;
    t.max_gen = (int32_t)max_gen_;
    t.payload = src[0].kind == SRC_ROWTILE && src[0].fmt != FMT_F16 && src[0].fmt != FMT_BF16;
    const uint32_t rowb = 2048u * (uint32_t)fmt_bits(src[0].fmt) / 8u;
    const uint32_t part = R * rowb + (t.payload ? kPayloadHead : 0u);
    const uint32_t stage = ((epi == EPI_SWIGLU ? 2u : 1u) * part + 127u) & ~127u;
    op.smem = kTmaStageOff + (size_t)kTmaStages * stage;
    const uint32_t jobs = epi == EPI_SWIGLU ? t.unit_start[1] : units;
    op.grid = dim3(jobs < (uint32_t)num_sms_ ? jobs : (uint32_t)num_sms_);
    ops.push_back(op);
    return;
  }

  if (fused) {
    Op op = make_gemv(src, out, nseg, epi, x, gamma, check_layer);
    op.role = epi == EPI_SWIGLU ? ROLE_GATEUP : epi == EPI_LOGITS ? ROLE_LMHEAD
              : (epi == EPI_ACCUM ? (ncols == arch_->D ? ROLE_O : ROLE_DOWN) : ROLE_QKV);
    for (int i = 0; i < nseg; i++) op.alg_bytes += alg_bytes_of(src[i]);
    ops.push_back(op);
    for (int i = 0; i < nseg; i++) push_aux(src[i], epi == EPI_SWIGLU ? nullptr : out[i], gamma ? d_xn_ : x);
    return;
  }
  // Decomposed: normalise once, then one op per tensor.
  const float* xin = x;
  if (gamma) {
    Op op;
    op.type = OP_NORM;
    op.nm = NormLaunch{x, gamma, d_xn_, ncols, A.eps, check_layer, d_st_, ignore_stop ? 1 : 0};
    op.grid = dim3((ncols + 255) / 256);
    op.threads = 256;
    ops.push_back(op);
    xin = d_xn_;
  }
  float* seg_out[3] = {out[0], nseg > 1 ? out[1] : nullptr, nseg > 2 ? out[2] : nullptr};
  if (epi == EPI_SWIGLU) { seg_out[0] = d_tmp_; seg_out[1] = d_tmp2_; }
  for (int i = 0; i < nseg; i++) {
    const GemvSrc& s = src[i];
    int e = epi == EPI_ACCUM ? EPI_ACCUM : EPI_STORE;
    if (s.kind == SRC_NOOP) continue;
    if (s.kind == SRC_PATTERN) {
      Op op;
      op.type = OP_PATTERN;
      op.pt = PatternLaunch{seg_out[i], s.r_total, ignore_stop ? nullptr : d_st_};
      op.grid = dim3((s.r_total + 255) / 256);
      ops.push_back(op);
      continue;
    }
    if (is_fast(s)) {
      Op op = make_gemv(&s, &seg_out[i], 1, e, xin, nullptr, -1);
      ops.push_back(op);
      push_aux(s, seg_out[i], xin);
      continue;
    }
    Op op;
    op.type = s.kind == SRC_GEN_ROWTILE ? OP_GEN_ROW : OP_GEN_FLAT;
    op.gen = GenLaunch{s, seg_out[i], xin, e == EPI_ACCUM, ignore_stop ? nullptr : d_st_};
    uint32_t need = (s.r_total + 7) / 8, cap = (uint32_t)num_sms_ * 8;
    op.grid = dim3(need < cap ? need : cap);
    ops.push_back(op);
  }
  if (epi == EPI_SWIGLU) {
    Op op;
    op.type = OP_SWIGLU;
    op.sw = SwigluLaunch{d_tmp_, d_tmp2_, out[0], src[0].r_total, d_st_};
    op.grid = dim3((src[0].r_total + 255) / 256);
    ops.push_back(op);
  }
  if (epi == EPI_LOGITS) {
    Op op;
    op.type = OP_ARGMAX;
    op.am = ArgmaxLaunch{out[0], src[0].r_total, src[0].kind == SRC_PATTERN ? 1 : 0, d_hidden_,
                         A.D, d_st_, d_res_, d_gen_, (int32_t)max_gen_};
    op.grid = dim3((uint32_t)num_sms_);
    ops.push_back(op);
  }
}

// Embedding of the step's token (unpackEmbedRow, chpe_engine.zig:1491-1552).
void Engine::push_embed(std::vector<Op>& ops) {
  const ChpeArch& A = *arch_;
  Op op;
  op.type = OP_EMBED;
  op.role = ROLE_EMBED;
  EmbedLaunch& e = op.em;
  e.arc = arc_for(0);
  e.record_count = f_.record_count;
  e.stride = f_.stride;
  e.prefix = f_.is_raw ? 0 : (f_.is_dense ? 64 : 3072 + 64);
  e.D = A.D;
  e.hidden = d_hidden_;
  e.st = d_st_;
  e.res = d_res_;
  e.use_state = 1;
  if (!f_.archive_valid || f_.record_count == 0) e.mode = EMB_PATTERN;
  else if (f_.is_raw_fp16) e.mode = EMB_RAW_F16;
  else if (f_.is_raw) e.mode = f_.quant_bits == 8 ? EMB_RAW_I8 : EMB_RAW_BF16;
  else e.mode = EMB_CELL;
  op.grid = dim3((A.D + 255) / 256);
  ops.push_back(op);
}

// The LM head source (computeLmHead, chpe_engine.zig:1554-1660): an untied
// span of cells, tied embedding cells, or tied raw rows.
GemvSrc Engine::plan_lm_head() {
  const ChpeArch& A = *arch_;
  GemvSrc lm{};
  int64_t lhs, lht;
  chpe_lm_head_span(arch_id_, &lhs, &lht);
  if (!f_.archive_valid || f_.record_count == 0) {
    lm.kind = SRC_PATTERN;
    lm.r_total = A.V;
  } else if (lhs >= 0 && (uint64_t)lhs < f_.record_count) {
    lm = plan_linear((uint64_t)lhs, (uint64_t)lht, A.V, A.D, A.D, 0, -1);
  } else if (!f_.is_raw) {
    // tied embedding cells, 16 rows each, unpackEmbedRowCell semantics
    lm.kind = SRC_ROWTILE;
    lm.arc = d_arc_;
    lm.r_total = A.V;
    lm.c_total = A.D;
    lm.x_len = A.D;
    lm.cell_rows = 16;
    lm.cell_cols = A.D;
    lm.tile0 = code_off(0);
    lm.stride = f_.stride;
    lm.rows_covered = A.V;
    uint64_t ncell = (A.V + 15) / 16;
    if (ncell > f_.record_count) throw std::runtime_error("tied LM head: archive has too few records");
    int fmt = -1;
    bool repl = false;
    for (uint64_t t = 0; t < ncell; t++) {
      const uint8_t* pl = host_ + code_off(t) + 16384;
      uint32_t qb = pl[20], rows = rd32(pl + 40);
      bool g = (rd64(pl + 24) & 1u) != 0;
      if ((rows != 16 && rows != 0) || qb == 8)
        throw std::runtime_error("tied LM head: embedding cells must hold 16 rows of 2/4-bit codes");
      int f = qb == 2 ? FMT_W2G : ((g || qb == 4) ? FMT_W4G : FMT_W4SB);
      if (fmt < 0) fmt = f;
      if (f != fmt) throw std::runtime_error("tied LM head: mixed embedding cell formats");
      if (t == 0) repl = g;
      if (g != repl) throw std::runtime_error("tied LM head: mixed outlier flags");
    }
    lm.fmt = fmt;
    lm.outliers = (repl && fmt != FMT_W4SB) ? OUTL_REPLACE : OUTL_NONE;
  } else {
    // tied raw FP16/BF16 embedding rows
    uint32_t rpt = 8192 / A.D ? 8192 / A.D : 1;
    uint64_t tiles = (A.V + rpt - 1) / rpt;
    if (tiles > f_.record_count) tiles = f_.record_count;
    lm.kind = SRC_RAW;
    lm.fmt = f_.is_raw_fp16 ? FMT_F16 : FMT_BF16;
    lm.arc = d_arc_;
    lm.r_total = A.V;
    lm.c_total = A.D;
    lm.x_len = A.D;
    lm.tile0 = code_off(0);
    lm.stride = f_.stride;
    lm.flat_limit = tiles * 8192ull;
    lm.n_tiles = (uint32_t)tiles;
  }
  return lm;
}

// ---- tensor parallelism ------------------------------------------------------
void Engine::tp_export(uint8_t* handle64) const {
  cudaIpcMemHandle_t h;
  CK(cudaSetDevice(device_));
  CK(cudaIpcGetMemHandle(&h, d_region_));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle64, &h, 64);
}

void Engine::tp_connect(const uint8_t* handles, int world) {
  if (world != tp_world_) throw std::runtime_error("tp_connect: world size differs from init");
  if (!ipc_open_.empty() || !ops_->empty()) throw std::runtime_error("tp_connect: already connected");
  CK(cudaSetDevice(device_));
  for (int r = 0; r < world; r++) {
    if (r == tp_rank_) {
      tp_delta_[r] = 0;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handles + 64 * r, 64);
    void* p = nullptr;
    CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    ipc_open_.push_back(p);
    tp_delta_[r] = (long long)((uint8_t*)p - d_region_);
  }
  build_step_tp();
}

// One decode step over this rank's slices.  Every projection is split by
// output rows (contiguous flat ranges of the row-major weight stream): q/k/v
// by heads, O and down by hidden rows, gate/up by FFN rows, the LM head by
// vocabulary rows.  Each output element is computed whole on one rank, with
// the same kernel and summation order as on one GPU, so results do not depend
// on the rank count.  Exchanges (written by the producing kernel straight into
// every rank's region, then counted): attention heads -> attn, O rows ->
// hidden, SwiGLU rows -> mlp, down rows -> hidden, logits (when gathered).
void Engine::build_step_tp() {
  const ChpeArch& A = *arch_;
  std::vector<Op>& ops = *ops_;
  ops.clear();
  const uint32_t N = (uint32_t)tp_world_, R = (uint32_t)tp_rank_;
  if (!f_.archive_valid || f_.record_count == 0)
    throw std::runtime_error("tensor parallel: needs a valid archive");
  ChpeTpSlice sl;
  if (chpe_tp_slice_of(arch_id_, (int)R, (int)N, &sl) != 0)
    throw std::runtime_error("tensor parallel: heads, hidden, FFN and vocabulary must split evenly over the ranks");
  const uint32_t hq = sl.hq, h0 = sl.h0, kv0 = sl.kv0, kvl = sl.kvl;
  const uint32_t dl = sl.dl, d0 = sl.d0, fl = sl.fl, f0 = sl.f0, vl = sl.vl, v0 = sl.v0;
  const uint32_t qd = A.H * A.HD, kvd = A.KV * A.HD;
  // arrivals per (step, layer) of each exchange: every rank launches the same
  // grids, so N x this rank's grid of the producing op
  const int nsp = attn_splits(num_sms_, (int)kvl, (int)max_seq_);
  const unsigned long long u_att = (unsigned long long)N * kvl;  // one reporter CTA per kv head
  unsigned long long u_o = 0, u_gu = 0, u_dn = 0;
  auto units_of_last = [&]() { return (unsigned long long)N * ops.back().grid.x; };
  TpLink base{};
  base.world = (int32_t)N;
  base.rank = (int32_t)R;
  for (int r = 0; r < kTpMax; r++) base.delta[r] = tp_delta_[r];
  base.sh = d_tpsh_;
  base.err = &d_st_->err;
  base.wait_polls = wait_polls_;
  base.wait_sig = -1;
  base.signal_sig = -1;
  base.wait_per_step = A.L;
  auto link = [&](int wait_sig, uint32_t wait_index, unsigned long long units, int signal_sig, int bcast) {
    TpLink t = base;
    t.wait_sig = wait_sig;
    t.wait_index = wait_index;
    t.wait_units = units;
    t.signal_sig = signal_sig;
    t.bcast = bcast;
    return t;
  };
  auto narrow = [&](GemvSrc s, uint32_t r0, uint32_t n) {
    if (s.kind != SRC_FLAT && s.kind != SRC_RAW)
      throw std::runtime_error("tensor parallel: every projection must be flat cells or a raw stream");
    if (s.has_aux) throw std::runtime_error("tensor parallel: down_aux replacement cells are not supported");
    s.row0 = r0;
    s.r_total = n;
    if (s.bias) s.bias += r0;
    // the slice's tiles lie in one uploaded run: address it there
    const uint64_t wpt = s.kind == SRC_RAW ? f_.wpt : 32768ull;
    const uint64_t t0 = (s.tile0 - 4096) / f_.stride;
    const uint64_t ta = t0 + (uint64_t)r0 * s.c_total / wpt;
    const uint64_t tb = t0 + ((uint64_t)(r0 + n) * s.c_total - 1) / wpt;
    if (ta >= t0 + s.n_tiles) {  // rows past the tensor's tiles: the kernel reads none of them
      s.arc = arc_for(0);
      return s;
    }
    s.arc = arc_for(ta);
    if (arc_for(tb < t0 + s.n_tiles ? tb : t0 + s.n_tiles - 1) != s.arc)
      throw std::runtime_error("tensor parallel: a slice spans two uploaded runs");
    return s;
  };

  push_embed(ops);
  std::vector<float> gam(A.D);
  for (uint32_t l = 0; l < A.L; l++) {
    ChpeLayerInfo li;
    chpe_layer_info(arch_id_, f_.is_raw, l, &li);
    unpack_norm((uint64_t)li.input_norm, gam.data());
    const float* g_in = upload_floats(gam);
    unpack_norm((uint64_t)li.post_norm, gam.data());
    const float* g_post = upload_floats(gam);
    GemvSrc qkv[3] = {
        narrow(plan_linear(li.q_proj, li.q_tiles, qd, A.D, A.D, 0, li.q_bias), h0 * A.HD, hq * A.HD),
        narrow(plan_linear(li.k_proj, li.k_tiles, kvd, A.D, A.D, 0, li.k_bias), kv0 * A.HD, kvl * A.HD),
        narrow(plan_linear(li.v_proj, li.v_tiles, kvd, A.D, A.D, 0, li.v_bias), kv0 * A.HD, kvl * A.HD)};
    float* qkv_out[3] = {d_q_, d_k_, d_v_};
    TpLink t_qkv = link(l ? SIG_DOWN : -1, l, u_dn, -1, 0);
    add_linear_ops(ops, qkv, qkv_out, 3, EPI_STORE, d_hidden_, g_in, (int)l - 1, A.D, false, &t_qkv);
    {
      Op op;
      op.type = OP_ATTN;
      op.role = ROLE_ATTN;
      op.hd = (int)A.HD;
      AttnLaunch& at = op.at;
      at.q = d_q_;
      at.k = d_k_;
      at.v = d_v_;
      if (kvl != kvl_) throw std::runtime_error("tensor parallel: kv heads differ from the cache layout");
      at.kc = d_kc_ + (size_t)l * layer_kv_elems_;  // this rank's kv heads only
      at.vc = d_vc_ + (size_t)l * layer_kv_elems_;
      at.pages = d_pages_;
      at.page_shift = kKvPageShift;
      at.n_pages = n_pages_;
      at.out = d_attn_ + (size_t)h0 * A.HD;
      at.part = d_part_;
      at.counters = d_counters_;
      at.inv_freq = d_invfreq_;
      at.st = d_st_;
      at.H = (int)hq;
      at.KV = (int)kvl;
      at.HD = (int)A.HD;
      at.nsplit = nsp;
      at.max_seq = (int32_t)max_seq_;
      at.tp = link(-1, 0, 0, SIG_ATT, 1);
      op.grid = dim3(nsp, kvl);
      op.threads = (int)(hq / kvl) * 32;
      if (op.threads < (int)A.HD / 2) op.threads = (int)A.HD / 2;
      if (op.threads < 128) op.threads = 128;
      ops.push_back(op);
    }
    GemvSrc o = narrow(plan_linear(li.o_proj, li.o_tiles, A.D, A.D, A.D, 1, -1), d0, dl);
    float* o_out[1] = {d_hidden_ + d0};
    TpLink t_o = link(SIG_ATT, l + 1, u_att, SIG_O, 1);
    add_linear_ops(ops, &o, o_out, 1, EPI_ACCUM, d_attn_, nullptr, -1, A.D, false, &t_o);
    u_o = units_of_last();
    GemvSrc gu[2] = {narrow(plan_linear(li.gate_proj, li.gate_tiles, A.F, A.D, A.D, 0, -1), f0, fl),
                     narrow(plan_linear(li.up_proj, li.up_tiles, A.F, A.D, A.D, 0, -1), f0, fl)};
    float* gu_out[2] = {d_mlp_ + f0, nullptr};
    TpLink t_gu = link(SIG_O, l + 1, u_o, SIG_GU, 1);
    add_linear_ops(ops, gu, gu_out, 2, EPI_SWIGLU, d_hidden_, g_post, -1, A.D, false, &t_gu);
    u_gu = units_of_last();
    GemvSrc dn = narrow(plan_linear(li.down_proj, li.down_tiles, A.D, A.F, A.F, 1, -1), d0, dl);
    float* dn_out[1] = {d_hidden_ + d0};
    TpLink t_dn = link(SIG_GU, l + 1, u_gu, SIG_DOWN, 1);
    add_linear_ops(ops, &dn, dn_out, 1, EPI_ACCUM, d_mlp_, nullptr, -1, A.F, false, &t_dn);
    u_dn = units_of_last();
  }
  unpack_norm((uint64_t)chpe_final_norm_index(arch_id_, f_.is_raw), gam.data());
  const float* g_fin = upload_floats(gam);
  GemvSrc lm = narrow(plan_lm_head(), v0, vl);
  float* lm_out[1] = {d_logits_ + v0};
  TpLink t_lm = link(SIG_DOWN, A.L, u_dn, SIG_LM, 1);
  add_linear_ops(ops, &lm, lm_out, 1, EPI_LOGITS, d_hidden_, g_fin, -1, A.D, true, &t_lm);
  ops.back().fl.tp.lm_units = units_of_last();
}

// ---- the decode step: forwardDecode (chpe_engine.zig:1663-1803) ------------
void Engine::build_step() {
  const ChpeArch& A = *arch_;
  std::vector<Op>& ops = *ops_;
  ops.clear();
  push_embed(ops);
  const uint32_t qd = A.H * A.HD, kvd = A.KV * A.HD;
  std::vector<float> gam(A.D);
  for (uint32_t l = 0; l < A.L; l++) {
    ChpeLayerInfo li;
    chpe_layer_info(arch_id_, f_.is_raw, l, &li);
    unpack_norm((uint64_t)li.input_norm, gam.data());
    const float* g_in = upload_floats(gam);
    unpack_norm((uint64_t)li.post_norm, gam.data());
    const float* g_post = upload_floats(gam);
    GemvSrc qkv[3] = {plan_linear(li.q_proj, li.q_tiles, qd, A.D, A.D, 0, li.q_bias),
                      plan_linear(li.k_proj, li.k_tiles, kvd, A.D, A.D, 0, li.k_bias),
                      plan_linear(li.v_proj, li.v_tiles, kvd, A.D, A.D, 0, li.v_bias)};
    float* qkv_out[3] = {d_q_, d_k_, d_v_};
    add_linear_ops(ops, qkv, qkv_out, 3, EPI_STORE, d_hidden_, g_in, (int)l - 1, A.D, false);
    {
      Op op;
      op.type = OP_ATTN;
      op.role = ROLE_ATTN;
      op.hd = (int)A.HD;
      AttnLaunch& at = op.at;
      at.q = d_q_;
      at.k = d_k_;
      at.v = d_v_;
      at.kc = d_kc_ + (size_t)l * layer_kv_elems_;
      at.vc = d_vc_ + (size_t)l * layer_kv_elems_;
      at.pages = d_pages_;
      at.page_shift = kKvPageShift;
      at.n_pages = n_pages_;
      at.out = d_attn_;
      at.part = d_part_;
      at.counters = d_counters_;
      at.inv_freq = d_invfreq_;
      at.st = d_st_;
      at.H = (int)A.H;
      at.KV = (int)A.KV;
      at.HD = (int)A.HD;
      at.nsplit = nsplit_;
      at.max_seq = (int32_t)max_seq_;
      op.grid = dim3(nsplit_, A.KV);
      op.threads = (int)(A.H / A.KV) * 32;
      if (op.threads < (int)A.HD / 2) op.threads = (int)A.HD / 2;
      if (op.threads < 128) op.threads = 128;
      ops.push_back(op);
    }
    GemvSrc o = plan_linear(li.o_proj, li.o_tiles, A.D, A.D, A.D, 1, -1);
    float* o_out[1] = {d_hidden_};
    add_linear_ops(ops, &o, o_out, 1, EPI_ACCUM, d_attn_, nullptr, -1, A.D, false);
    GemvSrc gu[2] = {plan_linear(li.gate_proj, li.gate_tiles, A.F, A.D, A.D, 0, -1),
                     plan_linear(li.up_proj, li.up_tiles, A.F, A.D, A.D, 0, -1)};
    float* gu_out[2] = {d_mlp_, nullptr};
    add_linear_ops(ops, gu, gu_out, 2, EPI_SWIGLU, d_hidden_, g_post, -1, A.D, false);
    GemvSrc dn = plan_linear(li.down_proj, li.down_tiles, A.D, A.F, A.F, 1, -1);
    float* dn_out[1] = {d_hidden_};
    add_linear_ops(ops, &dn, dn_out, 1, EPI_ACCUM, d_mlp_, nullptr, -1, A.F, false);
  }
  // final norm + LM head (computeLmHead, :1554-1660) + argmax (:1775-1802)
  unpack_norm((uint64_t)chpe_final_norm_index(arch_id_, f_.is_raw), gam.data());
  const float* g_fin = upload_floats(gam);
  GemvSrc lm = plan_lm_head();
  float* lm_out[1] = {d_logits_};
  add_linear_ops(ops, &lm, lm_out, 1, EPI_LOGITS, d_hidden_, g_fin, -1, A.D, true);

}

int Engine::kernels_per_step() const { return (int)ops_->size(); }

// ---- launching --------------------------------------------------------------
template <typename Kern, typename Arg>
static void launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, const Arg& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CK(cudaLaunchKernelEx(&cfg, kern, a));
}

template <int FMT, int KIND, int TH, int NR, int UNR>
static void launch_gemv_t(const Op& op, cudaStream_t s) {
  auto k = gemv_kernel<FMT, KIND, TH, NR, UNR>;
  static bool configured = false;
  if (!configured) {
    CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    configured = true;
  }
  launch_pdl(k, op.grid, dim3(TH), op.smem, s, op.g);
}

template <int FMT, int KIND>
static void launch_gemv_k(const Op& op, cudaStream_t s) {
  constexpr int NR = gemv_nr(FMT, KIND), UNR = gemv_unr(FMT, KIND);
  if (op.threads == 512) launch_gemv_t<FMT, KIND, 512, NR, UNR>(op, s);
  else launch_gemv_t<FMT, KIND, 256, NR, UNR>(op, s);
}

static void launch_gemv(const Op& op, cudaStream_t s) {
  switch (op.kind) {
    case SRC_RAW:
      switch (op.fmt) {
        case FMT_F16: return launch_gemv_k<FMT_F16, SRC_RAW>(op, s);
        case FMT_BF16: return launch_gemv_k<FMT_BF16, SRC_RAW>(op, s);
        case FMT_I8RAW: return launch_gemv_k<FMT_I8RAW, SRC_RAW>(op, s);
      }
      break;
    case SRC_ROWTILE:
      switch (op.fmt) {
        case FMT_W4G: return launch_gemv_k<FMT_W4G, SRC_ROWTILE>(op, s);
        case FMT_W4SB: return launch_gemv_k<FMT_W4SB, SRC_ROWTILE>(op, s);
        case FMT_W2G: return launch_gemv_k<FMT_W2G, SRC_ROWTILE>(op, s);
        case FMT_W2SB: return launch_gemv_k<FMT_W2SB, SRC_ROWTILE>(op, s);
        case FMT_F16: return launch_gemv_k<FMT_F16, SRC_ROWTILE>(op, s);
        case FMT_BF16: return launch_gemv_k<FMT_BF16, SRC_ROWTILE>(op, s);
        case FMT_F32: return launch_gemv_k<FMT_F32, SRC_ROWTILE>(op, s);
      }
      break;
    case SRC_FLAT:
      switch (op.fmt) {
        case FMT_W4G: return launch_gemv_k<FMT_W4G, SRC_FLAT>(op, s);
        case FMT_W4SB: return launch_gemv_k<FMT_W4SB, SRC_FLAT>(op, s);
        case FMT_W2G: return launch_gemv_k<FMT_W2G, SRC_FLAT>(op, s);
        case FMT_W2SB: return launch_gemv_k<FMT_W2SB, SRC_FLAT>(op, s);
      }
      break;
  }
  throw std::runtime_error("no GEMV kernel for this (format, layout)");
}

template <int FMT>
static void launch_tma_t(const Op& op, cudaStream_t s) {
  auto k = gemv_tma_kernel<FMT, kTmaStages>;
  static bool configured = false;
  if (!configured) {
    CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024));
    configured = true;
  }
  launch_pdl(k, op.grid, dim3(512), op.smem, s, op.tm);
}

static void launch_tma(const Op& op, cudaStream_t s) {
  switch (op.fmt) {
    case FMT_W4G: return launch_tma_t<FMT_W4G>(op, s);
    case FMT_W4SB: return launch_tma_t<FMT_W4SB>(op, s);
    case FMT_W2G: return launch_tma_t<FMT_W2G>(op, s);
    case FMT_W2SB: return launch_tma_t<FMT_W2SB>(op, s);
    case FMT_F16: return launch_tma_t<FMT_F16>(op, s);
    case FMT_BF16: return launch_tma_t<FMT_BF16>(op, s);
  }
  throw std::runtime_error("no TMA kernel for this format");
}

template <int FMT, int KIND, int MODE = FLAT_STREAM>
static void launch_flat_t(const Op& op, cudaStream_t s) {
  if constexpr (MODE == FLAT_ALIGNED) {
    if (op.fl.nw == 8) {
      auto k8 = gemv_flat_tma_kernel<FMT, KIND, MODE, 8>;
      static bool configured8 = false;
      if (!configured8) {
        CK(cudaFuncSetAttribute(k8, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFlatSmemHalf));
        configured8 = true;
      }
      launch_pdl(k8, op.grid, dim3(kFlatThreadsHalf), op.smem, s, op.fl);
      return;
    }
  }
  constexpr int NWT = MODE == FLAT_COLOWN || MODE == FLAT_COLOWN8 ? (int)kFlatColownWarps : 16;
  auto k = gemv_flat_tma_kernel<FMT, KIND, MODE, NWT>;
  static bool configured = false;
  if (!configured) {
    CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFlatSmemLimit));
    configured = true;
  }
  launch_pdl(k, op.grid, dim3(NWT * 32 + 32), op.smem, s, op.fl);
}

template <int NGW>
static void launch_rowblk_t(const Op& op, cudaStream_t s) {
  static bool configured = false;
  if (!configured) {
    CK(cudaFuncSetAttribute(gemv_rowblk_kernel<NGW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFlatSmemLimit));
    configured = true;
  }
  launch_pdl(gemv_rowblk_kernel<NGW>, op.grid, dim3(kRbThreads), op.smem, s, op.fl);
}

static void launch_flat(const Op& op, cudaStream_t s) {
  if (op.fl.mode == FLAT_ROWBLK) {
    switch ((op.fl.nw + kRbWarps - 1) / kRbWarps) {  // groups per warp, rounded up to even
      case 1: case 2: return launch_rowblk_t<2>(op, s);
      case 3: case 4: return launch_rowblk_t<4>(op, s);
      case 5: case 6: return launch_rowblk_t<6>(op, s);
      default: return launch_rowblk_t<8>(op, s);
    }
  }
  if (op.kind == SRC_FLAT && op.fl.mode == FLAT_MMA && op.fmt == FMT_W4G)
    return launch_flat_t<FMT_W4G, SRC_FLAT, FLAT_MMA>(op, s);
  if (op.kind == SRC_FLAT && op.fl.mode == FLAT_ALIGNED) {
    switch (op.fmt) {
      case FMT_W4G: return launch_flat_t<FMT_W4G, SRC_FLAT, FLAT_ALIGNED>(op, s);
      case FMT_W4SB: return launch_flat_t<FMT_W4SB, SRC_FLAT, FLAT_ALIGNED>(op, s);
      case FMT_W2G: return launch_flat_t<FMT_W2G, SRC_FLAT, FLAT_ALIGNED>(op, s);
      case FMT_W2SB: return launch_flat_t<FMT_W2SB, SRC_FLAT, FLAT_ALIGNED>(op, s);
    }
  } else if (op.kind == SRC_RAW && op.fl.mode == FLAT_ALIGNED) {
    switch (op.fmt) {
      case FMT_F16: return launch_flat_t<FMT_F16, SRC_RAW, FLAT_ALIGNED>(op, s);
      case FMT_BF16: return launch_flat_t<FMT_BF16, SRC_RAW, FLAT_ALIGNED>(op, s);
      case FMT_I8RAW: return launch_flat_t<FMT_I8RAW, SRC_RAW, FLAT_ALIGNED>(op, s);
    }
  } else if (op.kind == SRC_FLAT && op.fl.mode == FLAT_COLOWN) {
    switch (op.fmt) {
      case FMT_W4G: return launch_flat_t<FMT_W4G, SRC_FLAT, FLAT_COLOWN>(op, s);
      case FMT_W4SB: return launch_flat_t<FMT_W4SB, SRC_FLAT, FLAT_COLOWN>(op, s);
      case FMT_W2G: return launch_flat_t<FMT_W2G, SRC_FLAT, FLAT_COLOWN>(op, s);
      case FMT_W2SB: return launch_flat_t<FMT_W2SB, SRC_FLAT, FLAT_COLOWN>(op, s);
    }
  } else if (op.kind == SRC_RAW && op.fl.mode == FLAT_COLOWN) {
    switch (op.fmt) {
      case FMT_F16: return launch_flat_t<FMT_F16, SRC_RAW, FLAT_COLOWN>(op, s);
      case FMT_BF16: return launch_flat_t<FMT_BF16, SRC_RAW, FLAT_COLOWN>(op, s);
      case FMT_I8RAW: return launch_flat_t<FMT_I8RAW, SRC_RAW, FLAT_COLOWN>(op, s);
    }
  } else if (op.kind == SRC_RAW && op.fl.mode == FLAT_COLOWN8) {
    switch (op.fmt) {
      case FMT_F16: return launch_flat_t<FMT_F16, SRC_RAW, FLAT_COLOWN8>(op, s);
      case FMT_BF16: return launch_flat_t<FMT_BF16, SRC_RAW, FLAT_COLOWN8>(op, s);
    }
  } else if (op.kind == SRC_FLAT) {
    switch (op.fmt) {
      case FMT_W4G: return launch_flat_t<FMT_W4G, SRC_FLAT>(op, s);
      case FMT_W4SB: return launch_flat_t<FMT_W4SB, SRC_FLAT>(op, s);
      case FMT_W2G: return launch_flat_t<FMT_W2G, SRC_FLAT>(op, s);
      case FMT_W2SB: return launch_flat_t<FMT_W2SB, SRC_FLAT>(op, s);
    }
  } else if (op.kind == SRC_RAW) {
    switch (op.fmt) {
      case FMT_F16: return launch_flat_t<FMT_F16, SRC_RAW>(op, s);
      case FMT_BF16: return launch_flat_t<FMT_BF16, SRC_RAW>(op, s);
      case FMT_I8RAW: return launch_flat_t<FMT_I8RAW, SRC_RAW>(op, s);
    }
  }
  throw std::runtime_error("no flat TMA kernel for this (format, layout)");
}

static const char* fmt_name(int fmt) {
  static const char* N[] = {"W4G", "W4SB", "W2G", "W2SB", "W8", "F16", "BF16", "F32", "I8RAW", "ZERO"};
  return fmt >= 0 && fmt <= 9 ? N[fmt] : "?";
}
static const char* kind_name(int kind) {
  static const char* N[] = {"NOOP", "PATTERN", "RAW", "ROWTILE", "FLAT", "GEN_ROWTILE", "GEN_FLAT"};
  return kind >= 0 && kind <= 6 ? N[kind] : "?";
}

int Engine::profile_step(float* op_ms, int* op_roles, int cap) {
  if (!graph_) throw std::runtime_error("run forward() first");
  if ((uint64_t)pos_ + 1 > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  kv_ensure((uint64_t)pos_ + 1);
  const std::vector<Op>& ops = *ops_;
  const int n = (int)ops.size();
  std::vector<cudaEvent_t> ev(n + 1);
  for (auto& e : ev) CK(cudaEventCreate(&e));
  int32_t one = 1, zero = 0;
  CK(cudaMemcpyAsync(&d_st_->feed_argmax, &one, 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(&d_st_->gather, &zero, 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaEventRecord(ev[0], stream_));
  for (int i = 0; i < n; i++) {
    launch(ops[i], stream_);
    CK(cudaEventRecord(ev[i + 1], stream_));
  }
  CK(cudaMemcpyAsync(&d_st_->feed_argmax, &zero, 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(&d_st_->gather, &one, 4, cudaMemcpyHostToDevice, stream_));
  sync_result();
  for (int i = 0; i < n && i < cap; i++) {
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
    if (op_ms) op_ms[i] = ms;
    if (op_roles) op_roles[i] = ops[i].role;
  }
  for (auto& e : ev) cudaEventDestroy(e);
  pos_ += 1;
  return n;
}

double Engine::step_weight_bytes() const {
  double b = 0;
  for (const Op& op : *ops_) b += op.alg_bytes;
  return b;
}

std::string Engine::role_kernel_name(int role) const {
  for (const Op& op : *ops_) {
    if (op.role != role) continue;
    const std::string fk = std::string("<") + fmt_name(op.fmt) + "," + kind_name(op.kind) + ">";
    switch (op.type) {
      case OP_FLAT_TMA:
        if (op.fl.mode == FLAT_MMA) return "gemv_flat_tma_kernel[mma]" + fk;
        if (op.fl.mode == FLAT_ROWBLK) return "gemv_rowblk_kernel[mma]" + fk;
        return std::string(op.fl.mode == FLAT_ALIGNED
                               ? (op.fl.nw == 8 ? "gemv_flat_tma_kernel[aligned, 2 CTAs/SM]" : "gemv_flat_tma_kernel[aligned]")
                           : op.fl.mode == FLAT_COLOWN ? "gemv_flat_tma_kernel[column owners]"
                           : op.fl.mode == FLAT_COLOWN8 ? "gemv_flat_tma_kernel[column owners, 8 slots]"
                                                       : "gemv_flat_tma_kernel") + fk;
      case OP_TMA: return "gemv_tma_kernel" + fk;
      case OP_GEMV: return "gemv_kernel" + fk;
      case OP_ATTN: return "attention_kernel<" + std::to_string(op.hd) + ">";
      case OP_EMBED: return "embed_kernel";
      case OP_GEN_ROW: return "gemv_generic_rowtile";
      case OP_GEN_FLAT: return "gemv_generic_flat";
      default: return "op" + std::to_string(op.type);
    }
  }
  return "";
}

void Engine::launch(const Op& op, cudaStream_t s) const {
  switch (op.type) {
    case OP_FLAT_TMA: return launch_flat(op, s);
    case OP_TMA: return launch_tma(op, s);
    case OP_GEMV: return launch_gemv(op, s);
    case OP_GEN_ROW: return launch_pdl(gemv_generic_rowtile, op.grid, dim3(256), 0, s, op.gen);
    case OP_GEN_FLAT: return launch_pdl(gemv_generic_flat, op.grid, dim3(256), 0, s, op.gen);
    case OP_AUX: return launch_pdl(flat_aux_fix, op.grid, dim3(256), 0, s, op.aux);
    case OP_ATTN:
      if (op.hd == 128) return launch_pdl(attention_kernel<128>, op.grid, dim3(op.threads), 0, s, op.at);
      if (op.hd == 256) return launch_pdl(attention_kernel<256>, op.grid, dim3(op.threads), 0, s, op.at);
      throw std::runtime_error("unsupported head_dim");
    case OP_EMBED: return launch_pdl(embed_kernel, op.grid, dim3(256), 0, s, op.em);
    case OP_NORM: return launch_pdl(rmsnorm_kernel, op.grid, dim3(256), 0, s, op.nm);
    case OP_SWIGLU: return launch_pdl(swiglu_kernel, op.grid, dim3(256), 0, s, op.sw);
    case OP_PATTERN: return launch_pdl(pattern_kernel, op.grid, dim3(256), 0, s, op.pt);
    case OP_ARGMAX: return launch_pdl(argmax_kernel, op.grid, dim3(256), 0, s, op.am);
  }
}

void Engine::record(cudaStream_t s) const {
  for (const Op& op : *ops_) launch(op, s);
}

void Engine::ensure_graph() {
  if (graph_) return;
  // configure kernel attributes outside capture
  cudaStream_t cs;
  CK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
  record(stream_);  // warm launch also sets function attributes; result is discarded
  CK(cudaStreamSynchronize(stream_));
  cudaGraph_t g;
  CK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
  record(cs);
  CK(cudaStreamEndCapture(cs, &g));
  CK(cudaGraphInstantiate(&graph_, g, 0));
  CK(cudaGraphDestroy(g));
  CK(cudaStreamDestroy(cs));
}

// ---- paged KV cache ---------------------------------------------------------
// Host bookkeeping of the page table.  Every API call that runs steps ends by
// synchronising the engine stream, so the pinned mirror is never rewritten
// while an earlier copy of it is still pending.
void Engine::kv_ensure(uint64_t end_pos) {
  if (end_pos > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  const uint32_t need = (uint32_t)((end_pos + kKvPage - 1) >> kKvPageShift);
  if (need <= mapped_) return;
  if (need > n_pages_) throw std::runtime_error("KV page pool exhausted");
  for (uint32_t lp = mapped_; lp < need; lp++) {
    if (free_pages_.empty()) throw std::runtime_error("KV page pool exhausted");
    h_pages_[lp] = free_pages_.back();
    free_pages_.pop_back();
  }
  CK(cudaMemcpyAsync(d_pages_ + mapped_, h_pages_ + mapped_, (size_t)(need - mapped_) * 4,
                     cudaMemcpyHostToDevice, stream_));
  mapped_ = need;
}

void Engine::kv_reset() {
  // back onto the stack in reverse, so the same order comes out again
  for (uint32_t lp = mapped_; lp-- > 0;) free_pages_.push_back(h_pages_[lp]);
  mapped_ = 0;
}

void Engine::kv_set_page_order(const uint32_t* order, uint32_t n) {
  if (n != n_pages_) throw std::runtime_error("page order must list every page of the pool once");
  std::vector<char> seen(n_pages_, 0);
  for (uint32_t i = 0; i < n; i++) {
    if (order[i] >= n_pages_ || seen[order[i]]) throw std::runtime_error("page order is not a permutation");
    seen[order[i]] = 1;
  }
  CK(cudaStreamSynchronize(stream_));
  mapped_ = 0;
  free_pages_.assign(order, order + n);
  std::reverse(free_pages_.begin(), free_pages_.end());
}

uint32_t Engine::kv_page_table(uint32_t* out, uint32_t cap) const {
  for (uint32_t i = 0; i < mapped_ && i < cap; i++) out[i] = h_pages_[i];
  return mapped_;
}

void Engine::kv_load(uint32_t layer, uint32_t pos0, uint32_t n, const float* k, const float* v) {
  const ChpeArch& A = *arch_;
  if (layer >= A.L) throw std::runtime_error("layer out of range");
  if ((uint64_t)pos0 + n > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  if (n == 0) return;
  CK(cudaSetDevice(device_));
  kv_ensure((uint64_t)pos0 + n);
  const size_t full = (size_t)A.KV * A.HD, mine = (size_t)kvl_ * A.HD;
  std::vector<__half> hk((size_t)kKvPage * mine), hv((size_t)kKvPage * mine);
  __half* kb = d_kc_ + (size_t)layer * layer_kv_elems_;
  __half* vb = d_vc_ + (size_t)layer * layer_kv_elems_;
  for (uint32_t p = pos0; p < pos0 + n;) {
    const uint32_t lp = p >> kKvPageShift, in = p & (kKvPage - 1);
    uint32_t run = kKvPage - in;
    if (run > pos0 + n - p) run = pos0 + n - p;
    for (uint32_t r = 0; r < run; r++) {
      const float* ks = k + (size_t)(p - pos0 + r) * full + (size_t)kv0_ * A.HD;
      const float* vs = v + (size_t)(p - pos0 + r) * full + (size_t)kv0_ * A.HD;
      for (size_t i = 0; i < mine; i++) {
        hk[r * mine + i] = __float2half_rn(ks[i]);
        hv[r * mine + i] = __float2half_rn(vs[i]);
      }
    }
    const size_t row = (size_t)h_pages_[lp] * kKvPage + in;
    CK(cudaMemcpyAsync(kb + row * mine, hk.data(), run * mine * 2, cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(vb + row * mine, hv.data(), run * mine * 2, cudaMemcpyHostToDevice, stream_));
    CK(cudaStreamSynchronize(stream_));  // the staging vectors are reused
    p += run;
  }
}

void Engine::run_steps(size_t n) {
  for (size_t i = 0; i < n; i++) CK(cudaGraphLaunch(graph_, stream_));
}

void Engine::sync_result() {
  CK(cudaMemcpyAsync(h_res_, d_res_, sizeof(StepResult), cudaMemcpyDeviceToHost, stream_));
  CK(cudaMemcpyAsync(&h_st_->err, &d_st_->err, 4, cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  last_ = *h_res_;
  if (h_st_->err) {
    // Every kernel returned (the waits are bounded); clear the flag so the
    // next call starts clean, and report the timeout.
    h_st_->err = 0;
    CK(cudaMemcpyAsync(&d_st_->err, &h_st_->err, 4, cudaMemcpyHostToDevice, stream_));
    CK(cudaStreamSynchronize(stream_));
    throw std::runtime_error("a device wait timed out (bounded wait; the step's results are invalid)");
  }
}

void Engine::debug_wait_timeout(uint32_t polls) {
  CK(cudaSetDevice(device_));
  WaitProbeLaunch P{};
  P.tp.world = 2;  // a wait only reads this rank's own counters
  P.tp.rank = 0;
  P.tp.sh = d_tpsh_;
  P.tp.err = &d_st_->err;
  P.tp.wait_polls = polls ? polls : 1;
  P.st = d_st_;
  P.kind = 7;  // no exchange signals this slot
  wait_probe_kernel<<<1, 32, 0, stream_>>>(P);
  CK(cudaGetLastError());
  sync_result();
}

// Positions start_pos.. for the given tokens (forwardDecode per token).
void Engine::forward(const uint32_t* toks, size_t n, uint32_t start_pos) {
  if (n == 0) return;
  if (ops_->empty()) throw std::runtime_error("tensor parallel engine: call tp_connect first");
  if ((uint64_t)start_pos + n > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  if (start_pos == 0) kv_reset();  // a new sequence
  kv_ensure((uint64_t)start_pos + n);
  if (!graph_) {
    // The single-token step graph (later steps and the benchmarks need it,
    // even when the whole prompt goes through the batched step).  The
    // warm-up launch inside ensure_graph runs one step on whatever state is
    // current; run it at start_pos, whose KV rows are overwritten below.
    h_st_->token = (int32_t)toks[0];
    h_st_->pos = (int32_t)start_pos;
    h_st_->feed_argmax = 0;
    h_st_->stop = 0;
    h_st_->best = 0;
    h_st_->finite = 1;
    h_st_->done_ctas = 0;
    h_st_->n_gen = 0;
    CK(cudaMemcpyAsync(d_st_, h_st_, sizeof(StepState), cudaMemcpyHostToDevice, stream_));
    ensure_graph();
  }
  {
    // Batched prefill: whole chunks of 8 tokens through the batched step
    // (each weight read once per chunk on the tensor cores); the rest, and
    // archives that cannot take it, token by token.  CHPE_PREFILL_BATCHED=0
    // keeps every token on the single-token step.
    const char* pb = getenv("CHPE_PREFILL_BATCHED");
    size_t done = 0;
    const auto tb = now_ns();
    if (n >= 8 && !(pb && pb[0] == '0') && tp_world_ == 1) {
      while (n - done >= 8 && verify_batched(toks + done, 8, start_pos + (uint32_t)done, nullptr, nullptr))
        done += 8;
    }
    if (done == n) {
      last_ns_ = now_ns() - tb;
      return;
    }
    toks += done;
    n -= done;
    start_pos += (uint32_t)done;
  }
  auto t0 = now_ns();
  h_st_->token = (int32_t)toks[0];
  h_st_->pos = (int32_t)start_pos;
  h_st_->feed_argmax = 0;
  h_st_->stop = 0;
  h_st_->best = 0;
  h_st_->finite = 1;
  h_st_->done_ctas = 0;
  h_st_->n_gen = 0;
  CK(cudaMemcpyAsync(d_st_, h_st_, sizeof(StepState), cudaMemcpyHostToDevice, stream_));
  if (n + 1 > h_tok_cap_) throw std::runtime_error("token buffer too small");
  for (size_t i = 0; i < n; i++) {
    h_tok_[i] = toks[i];
    if (i > 0)
      CK(cudaMemcpyAsync(&d_st_->token, &h_tok_[i], 4, cudaMemcpyHostToDevice, stream_));
    CK(cudaGraphLaunch(graph_, stream_));
  }
  sync_result();
  last_ns_ = now_ns() - t0;
  pos_ = start_pos + (uint32_t)n;
}

void Engine::generate(const uint32_t* prompt, size_t n_prompt, size_t n_gen, uint32_t* out_tokens) {
  if (n_prompt == 0) throw std::runtime_error("empty prompt");
  if (n_prompt + n_gen > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  forward(prompt, n_prompt, 0);
  if (n_gen == 0) return;
  kv_ensure(n_prompt + n_gen);
  // the last prompt step's argmax is the first generated token
  out_tokens[0] = last_.argmax_token;
  int32_t one = 1, zero = 0;
  CK(cudaMemcpyAsync(&d_st_->feed_argmax, &one, 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(&d_st_->n_gen, &zero, 4, cudaMemcpyHostToDevice, stream_));
  run_steps(n_gen - 1);
  std::vector<int32_t> g(n_gen);
  if (n_gen > 1)
    CK(cudaMemcpyAsync(g.data(), d_gen_, (n_gen - 1) * 4, cudaMemcpyDeviceToHost, stream_));
  CK(cudaMemcpyAsync(&d_st_->feed_argmax, &zero, 4, cudaMemcpyHostToDevice, stream_));
  sync_result();
  for (size_t i = 1; i < n_gen; i++) out_tokens[i] = (uint32_t)g[i - 1];
  pos_ = (uint32_t)(n_prompt + n_gen - 1);
}

void Engine::verify(const uint32_t* toks, size_t m, uint32_t pos, float* logits_out, uint32_t* argmax_out) {
  if (m == 0) return;
  last_verify_batched_ = 0;
  if (verify_batched(toks, m, pos, logits_out, argmax_out)) {
    last_verify_batched_ = 1;
    return;
  }
  if ((uint64_t)pos + m > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  if (m + 1 > h_tok_cap_) throw std::runtime_error("too many candidates");
  if (pos == 0) kv_reset();
  kv_ensure((uint64_t)pos + m);
  if (!graph_) {
    // build the graph with a warm step at the first candidate's position (its
    // cache entry is rewritten below)
    forward(toks, 1, pos);
  }
  const size_t V = arch_->V;
  if (m > vcap_) {
    if (d_vlogits_) cudaFree(d_vlogits_);
    if (d_vres_) cudaFree(d_vres_);
    CK(cudaMalloc(&d_vlogits_, m * V * 4));
    CK(cudaMalloc(&d_vres_, m * sizeof(StepResult)));
    vcap_ = m;
  }
  h_st_->token = (int32_t)toks[0];
  h_st_->pos = (int32_t)pos;
  h_st_->feed_argmax = 0;
  h_st_->stop = 0;
  h_st_->best = 0;
  h_st_->finite = 1;
  h_st_->done_ctas = 0;
  h_st_->n_gen = 0;
  CK(cudaMemcpyAsync(d_st_, h_st_, sizeof(StepState), cudaMemcpyHostToDevice, stream_));
  auto t0 = now_ns();
  // m decode steps back to back on the device; each step's logits and result
  // are copied aside before the next step reuses the buffers
  for (size_t i = 0; i < m; i++) {
    h_tok_[i] = toks[i];
    if (i > 0) CK(cudaMemcpyAsync(&d_st_->token, &h_tok_[i], 4, cudaMemcpyHostToDevice, stream_));
    CK(cudaGraphLaunch(graph_, stream_));
    CK(cudaMemcpyAsync(d_vlogits_ + i * V, d_logits_, V * 4, cudaMemcpyDeviceToDevice, stream_));
    CK(cudaMemcpyAsync(d_vres_ + i, d_res_, sizeof(StepResult), cudaMemcpyDeviceToDevice, stream_));
  }
  std::vector<StepResult> res(m);
  CK(cudaMemcpyAsync(res.data(), d_vres_, m * sizeof(StepResult), cudaMemcpyDeviceToHost, stream_));
  if (logits_out) CK(cudaMemcpyAsync(logits_out, d_vlogits_, m * V * 4, cudaMemcpyDeviceToHost, stream_));
  sync_result();
  last_ns_ = now_ns() - t0;
  if (argmax_out)
    for (size_t i = 0; i < m; i++) argmax_out[i] = res[i].argmax_token;
  pos_ = pos + (uint32_t)m;
}

// Prompt-lookup draft: the up-to-m tokens that followed the latest earlier
// occurrence of the sequence's last n tokens (n = ngram .. 1).
static size_t lookup_draft(const std::vector<uint32_t>& h, uint32_t ngram, size_t m, uint32_t* d) {
  const size_t H = h.size();
  for (size_t n = ngram; n >= 1; n--) {
    if (n >= H) continue;
    for (size_t s = H - n; s-- > 0;) {  // candidate start of an earlier match
      bool eq = true;
      for (size_t j = 0; j < n && eq; j++) eq = h[s + j] == h[H - n + j];
      if (!eq) continue;
      size_t k = 0;
      for (; k < m && s + n + k < H; k++) d[k] = h[s + n + k];
      if (k > 0) return k;
    }
  }
  return 0;
}

void Engine::speculative_generate(const uint32_t* prompt, size_t n_prompt, size_t n_gen, uint32_t draft,
                                  uint32_t ngram, uint32_t* out, uint64_t* stats) {
  if (n_prompt == 0) throw std::runtime_error("empty prompt");
  if (n_prompt + n_gen > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  if (draft + 1 > h_tok_cap_) throw std::runtime_error("draft longer than the token buffer");
  uint64_t rounds = 0, proposed = 0, accepted = 0;
  forward(prompt, n_prompt, 0);
  if (n_gen == 0) return;
  std::vector<uint32_t> hist(prompt, prompt + n_prompt);
  uint32_t x = last_.argmax_token;  // emitted, not yet run through the model
  size_t produced = 0;
  out[produced++] = x;
  hist.push_back(x);
  uint32_t pos = (uint32_t)n_prompt;  // x's position
  std::vector<uint32_t> chunk(draft + 1), am(draft + 1);
  while (produced < n_gen) {
    size_t m = draft;
    if (m > n_gen - produced) m = n_gen - produced;
    if ((uint64_t)pos + m + 1 > max_seq_) m = max_seq_ - pos - 1;
    chunk[0] = x;
    m = lookup_draft(hist, ngram ? ngram : 1, m, chunk.data() + 1);
    verify(chunk.data(), m + 1, pos, nullptr, am.data());
    rounds++;
    proposed += m;
    size_t k = 0;
    while (k < m && am[k] == chunk[k + 1]) k++;
    accepted += k;
    for (size_t i = 0; i < k && produced < n_gen; i++) {
      out[produced++] = chunk[i + 1];
      hist.push_back(chunk[i + 1]);
    }
    if (produced < n_gen) {
      out[produced++] = am[k];
      hist.push_back(am[k]);
    }
    x = am[k];
    pos += (uint32_t)(k + 1);
  }
  if (stats) {
    stats[0] = rounds;
    stats[1] = proposed;
    stats[2] = accepted;
  }
}

float Engine::timed_greedy_steps(size_t n) {
  if (!graph_) throw std::runtime_error("run forward() first");
  if ((uint64_t)pos_ + n > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  kv_ensure((uint64_t)pos_ + n);
  int32_t one = 1, zero = 0;
  CK(cudaMemcpyAsync(&d_st_->feed_argmax, &one, 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(&d_st_->n_gen, &zero, 4, cudaMemcpyHostToDevice, stream_));
  // greedy steps need only the argmax: ranks keep their own logit slices
  CK(cudaMemcpyAsync(&d_st_->gather, &zero, 4, cudaMemcpyHostToDevice, stream_));
  cudaEvent_t a, b;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  CK(cudaStreamSynchronize(stream_));
  CK(cudaEventRecord(a, stream_));
  run_steps(n);
  CK(cudaEventRecord(b, stream_));
  CK(cudaMemcpyAsync(&d_st_->feed_argmax, &zero, 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(&d_st_->gather, &one, 4, cudaMemcpyHostToDevice, stream_));
  sync_result();
  float ms = 0;
  CK(cudaEventElapsedTime(&ms, a, b));
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  pos_ += (uint32_t)n;
  return ms;
}

double Engine::timed_host_steps(const uint32_t* toks, size_t n, float* logits_host) {
  if (!graph_) throw std::runtime_error("run forward() first");
  if ((uint64_t)pos_ + n > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  kv_ensure((uint64_t)pos_ + n);
  CK(cudaStreamSynchronize(stream_));
  uint64_t t0 = now_ns();
  for (size_t i = 0; i < n; i++) {
    h_tok_[i % h_tok_cap_] = toks[i];
    CK(cudaMemcpyAsync(&d_st_->token, &h_tok_[i % h_tok_cap_], 4, cudaMemcpyHostToDevice, stream_));
    CK(cudaGraphLaunch(graph_, stream_));
    CK(cudaMemcpyAsync(logits_host, d_logits_, (size_t)arch_->V * 4, cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(h_res_, d_res_, sizeof(StepResult), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
  }
  uint64_t t1 = now_ns();
  last_ = *h_res_;
  pos_ += (uint32_t)n;
  return (double)(t1 - t0) / 1e6;
}

void Engine::copy_logits(float* out) const {
  CK(cudaMemcpy(out, d_logits_, (size_t)arch_->V * 4, cudaMemcpyDeviceToHost));
}

void Engine::bench_role(int role, int rounds, float* avg_ms, double* bytes_per_launch, int* launches,
                        bool flush_l2) {
  if (tp_world_ > 1)
    throw std::runtime_error("per-role timing launches one role alone; not available with tensor parallelism");
  std::vector<const Op*> sel;
  for (const Op& op : *ops_)
    if (op.role == role) sel.push_back(&op);
  if (sel.empty()) throw std::runtime_error("no op with that role");
  double bytes = 0;
  for (const Op* op : sel) bytes += op->alg_bytes;
  // Save the step state (the LM head's finalisation advances it), clear the
  // stop flag so layer ops run, and restore the state afterwards.
  StepState saved;
  CK(cudaMemcpyAsync(h_st_, d_st_, sizeof(StepState), cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  saved = *h_st_;
  int32_t zero = 0;
  CK(cudaMemcpyAsync(&d_st_->stop, &zero, 4, cudaMemcpyHostToDevice, stream_));
  for (const Op* op : sel) launch(*op, stream_);  // warm-up round
  cudaEvent_t a, b;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  CK(cudaStreamSynchronize(stream_));
  float ms = 0;
  if (!flush_l2) {
    CK(cudaEventRecord(a, stream_));
    for (int r = 0; r < rounds; r++)
      for (const Op* op : sel) launch(*op, stream_);
    CK(cudaEventRecord(b, stream_));
    CK(cudaEventSynchronize(b));
    CK(cudaEventElapsedTime(&ms, a, b));
  } else {
    const size_t fb = 256ull << 20;  // twice the L2
    void* flush = nullptr;
    CK(cudaMalloc(&flush, fb));
    for (int r = 0; r < rounds; r++)
      for (const Op* op : sel) {
        CK(cudaMemsetAsync(flush, r & 0xff, fb, stream_));
        CK(cudaEventRecord(a, stream_));
        launch(*op, stream_);
        CK(cudaEventRecord(b, stream_));
        CK(cudaEventSynchronize(b));
        float one = 0.f;
        CK(cudaEventElapsedTime(&one, a, b));
        ms += one;
      }
    cudaFree(flush);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  *h_st_ = saved;
  CK(cudaMemcpyAsync(d_st_, h_st_, sizeof(StepState), cudaMemcpyHostToDevice, stream_));
  CK(cudaStreamSynchronize(stream_));
  int n = rounds * (int)sel.size();
  *avg_ms = ms / (float)n;
  *bytes_per_launch = bytes / (double)sel.size();
  *launches = n;
}

// ---- probes used by the parity tests ----------------------------------------
void Engine::debug_gemv_linear(uint64_t tile_start, uint64_t num_tiles, const float* x,
                               uint64_t x_len, float* y, uint64_t r_total, uint64_t c_total,
                               int accumulate, int64_t bias_tile) {
  GemvSrc s = plan_linear(tile_start, num_tiles, (uint32_t)r_total, (uint32_t)c_total,
                          (uint32_t)x_len, accumulate, bias_tile);
  float *dx = nullptr, *dy = nullptr;
  CK(cudaMalloc(&dx, x_len * 4 + 16));
  CK(cudaMalloc(&dy, r_total * 4 + 16));
  CK(cudaMemcpy(dx, x, x_len * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dy, y, r_total * 4, cudaMemcpyHostToDevice));
  // clear the step state's stop flag for the probe
  int32_t zero = 0;
  CK(cudaMemcpy(&d_st_->stop, &zero, 4, cudaMemcpyHostToDevice));
  std::vector<Op> ops;
  float* outs[1] = {dy};
  add_linear_ops(ops, &s, outs, 1, accumulate ? EPI_ACCUM : EPI_STORE, dx, nullptr, -1,
                 (uint32_t)c_total, false);
  for (const Op& op : ops) launch(op, stream_);
  CK(cudaStreamSynchronize(stream_));
  CK(cudaMemcpy(y, dy, r_total * 4, cudaMemcpyDeviceToHost));
  cudaFree(dx);
  cudaFree(dy);
}

void Engine::debug_attention(uint32_t layer, uint32_t pos, const float* q, const float* k,
                             const float* v, float* out) {
  const ChpeArch& A = *arch_;
  if (layer >= A.L || pos >= max_seq_) throw std::runtime_error("layer or position out of range");
  kv_ensure((uint64_t)pos + 1);
  const Op* att = nullptr;
  uint32_t seen = 0;
  for (const Op& op : *ops_)
    if (op.type == OP_ATTN && seen++ == layer) att = &op;
  if (!att) throw std::runtime_error("no attention op");
  const size_t nq = (size_t)A.H * A.HD, nkv = (size_t)A.KV * A.HD;
  CK(cudaMemcpyAsync(d_q_, q, nq * 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(d_k_, k, nkv * 4, cudaMemcpyHostToDevice, stream_));
  CK(cudaMemcpyAsync(d_v_, v, nkv * 4, cudaMemcpyHostToDevice, stream_));
  // step state: this position, no early exit
  CK(cudaMemcpyAsync(h_st_, d_st_, sizeof(StepState), cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  StepState saved = *h_st_;
  h_st_->pos = (int32_t)pos;
  h_st_->stop = 0;
  CK(cudaMemcpyAsync(d_st_, h_st_, sizeof(StepState), cudaMemcpyHostToDevice, stream_));
  launch(*att, stream_);
  CK(cudaMemcpyAsync(out, d_attn_, nq * 4, cudaMemcpyDeviceToHost, stream_));
  CK(cudaStreamSynchronize(stream_));
  *h_st_ = saved;
  CK(cudaMemcpyAsync(d_st_, h_st_, sizeof(StepState), cudaMemcpyHostToDevice, stream_));
  CK(cudaStreamSynchronize(stream_));
}

void Engine::debug_embed(uint32_t token, float* out) {
  Op op = (*ops_)[0];
  float* d = nullptr;
  CK(cudaMalloc(&d, arch_->D * 4));
  CK(cudaMemcpy(d, out, arch_->D * 4, cudaMemcpyHostToDevice));
  op.em.hidden = d;
  op.em.use_state = 0;
  op.em.token = token;
  launch(op, stream_);
  CK(cudaStreamSynchronize(stream_));
  CK(cudaMemcpy(out, d, arch_->D * 4, cudaMemcpyDeviceToHost));
  cudaFree(d);
}

void Engine::debug_dequant_cell(uint64_t tile, int flat, float* out, uint64_t cap, uint64_t* n_out) {
  if (f_.is_raw || tile >= f_.record_count) throw std::runtime_error("not a cell");
  const uint8_t* pl = host_ + code_off(tile) + 16384;
  uint64_t n = flat ? 32768 : (uint64_t)rd32(pl + 40) * rd32(pl + 44);
  if (n > cap) n = cap;
  float* d = nullptr;
  CK(cudaMalloc(&d, n * 4 + 16));
  DequantLaunch P{d_arc_ + code_off(tile), flat, d, (uint32_t)n};
  dequant_kernel<<<64, 256, 0, stream_>>>(P);
  CK(cudaGetLastError());
  CK(cudaStreamSynchronize(stream_));
  CK(cudaMemcpy(out, d, n * 4, cudaMemcpyDeviceToHost));
  cudaFree(d);
  *n_out = n;
}

}  // namespace chpe
