// engine_verify.cu -- the batched decode step: NT tokens (4 or 8) at
// consecutive positions through every layer at once, each weight read once
// for all of them through the tcgen05 GEMM (bgemm_tc.cuh).  It serves
// chpe_verify (speculative verification: candidate i sees the KV entries of
// candidates < i) and prompt chunks.  The result equals NT forwardDecode
// steps (chpe_engine.zig:1663-1803) up to f32 rounding.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "attention.cuh"
#include "aux_kernels.cuh"
#include "bgemm_tc.cuh"
#include "engine.h"

namespace chpe {

#define CKV(x)                                                                              \
  do {                                                                                      \
    cudaError_t e_ = (x);                                                                   \
    if (e_ != cudaSuccess)                                                                  \
      throw std::runtime_error(std::string(#x) + ": " + cudaGetErrorString(e_));            \
  } while (0)

// Plans one batched GEMM call; false when a segment cannot take the
// tensor-core path (not 4-bit group-scaled flat cells, down_aux fix-ups,
// rows not whole 128-row blocks, rows past the tensor's tiles).
bool plan_bgemm(const GemvSrc* src, int nseg, int epi, uint32_t C, int nt, int num_sms, BgemmLaunch& B,
                uint32_t& smem) {
  memset(&B, 0, sizeof(B));
  if (C == 0 || C % 128u || nseg < 1 || nseg > 3 || (nt != 4 && nt != 8)) return false;
  uint32_t rows = 0;
  for (int i = 0; i < nseg; i++) {
    const GemvSrc& s = src[i];
    if (s.kind != SRC_FLAT || s.fmt != FMT_W4G || s.has_aux || s.c_total != C || s.r_total == 0 ||
        s.r_total % kBgRows)
      return false;
    // rows the tiles hold in full; a row cut by the last tile is not taken
    const uint64_t avail = s.flat_limit / C;
    if (s.flat_limit % C != 0 && avail < (uint64_t)s.row0 + s.r_total) return false;
    B.rows_avail[i] = (uint32_t)(avail < (uint64_t)s.row0 + s.r_total ? avail : (uint64_t)s.row0 + s.r_total);
    B.src[i] = s;
    B.row_start[i] = rows;
    rows += s.r_total;
  }
  B.row_start[nseg] = rows;
  if (epi == EPI_SWIGLU && (nseg != 2 || src[0].r_total != src[1].r_total)) return false;
  const uint32_t G = C / 128u, nb = rows / kBgRows;
  uint32_t ks = (G + kBgMaxGroups - 1) / kBgMaxGroups;
  const uint32_t fill = (2u * (uint32_t)num_sms + nb - 1) / nb;  // two CTAs per SM at least
  if (fill > ks) ks = fill;
  if (ks > G) ks = G;
  B.nseg = nseg;
  B.epi = epi;
  B.C = C;
  B.ksplit = ks;
  B.nunits = nb * ks;
  B.rows_total = rows;
  smem = bg_smem((uint32_t)nt, (G + ks - 1) / ks).total;
  return true;
}

void launch_bgemm(int nt, const BgemmLaunch& B, uint32_t smem, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B.nunits);
  cfg.blockDim = dim3(kBgThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchConfig_t pc = cfg;  // the B-piece preparation: one CTA per group, a warp per token
  pc.gridDim = dim3(B.C / 128u);
  pc.blockDim = dim3(32u * (uint32_t)nt);
  pc.dynamicSmemBytes = 0;
  if (nt == 4) {
    static bool set4 = false;
    if (!set4) {
      CKV(cudaFuncSetAttribute(bgemm_w4_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      set4 = true;
    }
    CKV(cudaLaunchKernelEx(&pc, bgemm_prep_kernel<4>, B));
    CKV(cudaLaunchKernelEx(&cfg, bgemm_w4_kernel<4>, B));
  } else {
    static bool set8 = false;
    if (!set8) {
      CKV(cudaFuncSetAttribute(bgemm_w4_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      set8 = true;
    }
    CKV(cudaLaunchKernelEx(&pc, bgemm_prep_kernel<8>, B));
    CKV(cudaLaunchKernelEx(&cfg, bgemm_w4_kernel<8>, B));
  }
}

void Engine::debug_bgemm(uint64_t tile_start, uint64_t num_tiles, const float* x, int nt, float* y,
                         uint64_t r_total, uint64_t c_total, int accumulate) {
  CKV(cudaSetDevice(device_));
  GemvSrc s = plan_linear(tile_start, num_tiles, (uint32_t)r_total, (uint32_t)c_total, (uint32_t)c_total,
                          accumulate, -1);
  BgemmLaunch B;
  uint32_t smem = 0;
  if (!plan_bgemm(&s, 1, accumulate ? EPI_ACCUM : EPI_STORE, (uint32_t)c_total, nt, num_sms_, B, smem))
    throw std::runtime_error("this call cannot take the batched tensor-core GEMM");
  const size_t nx = (size_t)nt * c_total, ny = (size_t)nt * r_total;
  const size_t npart = (size_t)B.ksplit * nt * B.rows_total, nblk = B.rows_total / kBgRows;
  float *dx = nullptr, *dy = nullptr, *dp = nullptr;
  uint32_t* dc = nullptr;
  int32_t* flags = nullptr;
  CKV(cudaMalloc(&dx, nx * 4));
  CKV(cudaMalloc(&dy, ny * 4));
  CKV(cudaMalloc(&dp, npart * 4));
  CKV(cudaMalloc(&dc, nblk * 4));
  CKV(cudaMalloc(&flags, 8));
  uint8_t* dpieces = nullptr;
  float* dpxsc = nullptr;
  CKV(cudaMalloc(&dpieces, (size_t)(c_total / 128) * 128 * 4 * nt));
  CKV(cudaMalloc(&dpxsc, (size_t)(c_total / 128) * nt * 8));
  B.pieces = dpieces;
  B.pxsc = dpxsc;
  CKV(cudaMemcpy(dx, x, nx * 4, cudaMemcpyHostToDevice));
  CKV(cudaMemcpy(dy, y, ny * 4, cudaMemcpyHostToDevice));
  CKV(cudaMemset(dc, 0, nblk * 4));
  CKV(cudaMemset(flags, 0, 8));
  B.x = dx;
  B.x_stride = (uint32_t)c_total;
  B.out[0] = dy;
  B.out_stride = (uint32_t)r_total;
  B.part = dp;
  B.counters = dc;
  B.bad = flags;
  B.err = flags + 1;
  // CHPE_BGEMM_TRACE=<file>: per-CTA timer samples of this launch are
  // written there (entry, prologue end, main loop end, exit), as u64
  const char* trace_path = getenv("CHPE_BGEMM_TRACE");
  unsigned long long* dtrace = nullptr;
  if (trace_path) {
    CKV(cudaMalloc(&dtrace, (size_t)B.nunits * 32 + 48 * 8));
    CKV(cudaMemset(dtrace, 0, (size_t)B.nunits * 32 + 48 * 8));
    B.trace = dtrace;
  }
  launch_bgemm(nt, B, smem, stream_, false);
  CKV(cudaGetLastError());
  CKV(cudaStreamSynchronize(stream_));
  if (dtrace) {
    std::vector<unsigned long long> h((size_t)B.nunits * 4 + 48);
    CKV(cudaMemcpy(h.data(), dtrace, h.size() * 8, cudaMemcpyDeviceToHost));
    cudaFree(dtrace);
    if (FILE* f = fopen(trace_path, "wb")) {
      fwrite(h.data(), 8, h.size(), f);
      fclose(f);
    }
  }
  int32_t h[2] = {0, 0};
  CKV(cudaMemcpy(y, dy, ny * 4, cudaMemcpyDeviceToHost));
  CKV(cudaMemcpy(h, flags, 8, cudaMemcpyDeviceToHost));
  cudaFree(dx);
  cudaFree(dy);
  cudaFree(dp);
  cudaFree(dc);
  cudaFree(flags);
  cudaFree(dpieces);
  cudaFree(dpxsc);
  if (h[1]) throw std::runtime_error("a device wait timed out in the batched GEMM");
}

// ---- the batched step -------------------------------------------------------

// RoPE on the K of every token of the step and both caches' rows for their
// positions (st->pos + token), exactly as the decode attention kernel rotates
// and rounds the current position's K/V before appending it
// (chpe_engine.zig:1688-1698).
struct RopeAppendLaunch {
  const float* qkv;  // [nt][stride]: q | k | v
  uint32_t stride, qd;
  __half *kc, *vc;   // this layer's pools
  const uint32_t* pages;
  int32_t page_shift;
  uint32_t n_pages;
  const float* inv_freq;
  const StepState* st;
  int32_t KV, HD, max_seq;
};
static __global__ void rope_append_kernel(const __grid_constant__ RopeAppendLaunch P) {
  pdl_wait();
  const int t = blockIdx.x, h = blockIdx.y, HD = P.HD;
  const int pos = P.st->pos + t;
  if (pos < 0 || pos >= P.max_seq) return;
  uint32_t pg = P.pages[pos >> P.page_shift];
  if (pg >= P.n_pages) pg = 0;
  const size_t row = ((size_t)pg << P.page_shift) + (size_t)(pos & ((1 << P.page_shift) - 1));
  const size_t base = (row * P.KV + h) * HD;
  const float* k = P.qkv + (size_t)t * P.stride + P.qd + (size_t)h * HD;
  const float* v = k + (size_t)P.KV * HD;
  const float pf = (float)pos;
  for (int i = threadIdx.x; i < HD / 2; i += blockDim.x) {
    const float th = pf * P.inv_freq[i];
    const float c = cosf(th), s = sinf(th);
    const float x0 = k[i], x1 = k[i + HD / 2];
    P.kc[base + i] = __float2half_rn(x0 * c - x1 * s);
    P.kc[base + i + HD / 2] = __float2half_rn(x0 * s + x1 * c);
  }
  for (int i = threadIdx.x; i < HD; i += blockDim.x) P.vc[base + i] = __float2half_rn(v[i]);
  pdl_launch_dependents();
}

// Per token: the ForwardResult (chpe_engine.zig:1775-1802) from the LM head's
// argmax key and finiteness flag, the logit of token 0 and the norm of the
// hidden vector after the layer loop; then the keys are reset.
struct BatchFinalLaunch {
  unsigned long long* best;
  uint32_t* finite;
  const float* logits;
  uint32_t V;
  const float* hidden;
  uint32_t D;
  StepResult* res;
  const StepState* st;
};
static __global__ void __launch_bounds__(256) batch_final_kernel(const __grid_constant__ BatchFinalLaunch P) {
  pdl_wait();
  const int t = blockIdx.x;
  __shared__ float red[8];
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < P.D; i += 256) {
    const float h = P.hidden[(size_t)t * P.D + i];
    ss = fmaf(h, h, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < 8; w++) tot += red[w];
    const unsigned long long b = P.best[t];
    StepResult R;
    R.argmax_token = b ? 0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull) : 0u;
    R.max_logit = b ? key_value(b) : -1e30f;
    R.token0_logit = P.logits[(size_t)t * P.V];
    R.hidden_norm = sqrtf(tot);
    R.all_finite = (int32_t)P.finite[t];
    R.pos = P.st->pos + t;
    P.res[t] = R;
    P.best[t] = 0ull;
    P.finite[t] = 1u;
  }
}

enum BOpType : int32_t { BOP_EMBED = 0, BOP_GEMM, BOP_ROPE, BOP_ATTN, BOP_FINAL };

struct BOp {
  int32_t type = 0, hd = 128;
  int32_t role = 0;       // chpe_bench_kernel's role numbers (0: other)
  double alg_bytes = 0;   // algorithmic weight bytes (codes + scales of the rows used)
  dim3 grid{1, 1, 1}, block{256, 1, 1};
  uint32_t smem = 0;
  BgemmLaunch bg{};
  AttnLaunch at{};
  EmbedLaunch em{};
  RopeAppendLaunch rp{};
  BatchFinalLaunch fn{};
};

struct BatchStep {
  int nt = 4;
  std::vector<BOp> ops;
  std::vector<void*> dev;  // device allocations
  float *h = nullptr, *qkv = nullptr, *attn = nullptr, *mlp = nullptr, *logits = nullptr, *part = nullptr;
  float* apart = nullptr;
  uint32_t *cnt = nullptr, *fin = nullptr, *acnt = nullptr;
  unsigned long long* best = nullptr;
  int32_t *flags = nullptr, *toks = nullptr;
  StepState* st = nullptr;
  StepResult* res = nullptr;
  int32_t* h_toks = nullptr;   // pinned
  StepState* h_st = nullptr;   // pinned
  StepResult* h_res = nullptr; // pinned
  int32_t* h_flags = nullptr;  // pinned
  cudaGraphExec_t graph = nullptr;
  bool ran = false;
};

template <typename Kern, typename Arg>
static void launch_v(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, const Arg& a) {
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
  CKV(cudaLaunchKernelEx(&cfg, kern, a));
}

static void run_bop(const BatchStep& B, const BOp& op, cudaStream_t s);

static void run_bops(const BatchStep& B, cudaStream_t s) {
  for (const BOp& op : B.ops) run_bop(B, op, s);
}

static void run_bop(const BatchStep& B, const BOp& op, cudaStream_t s) {
  {
    switch (op.type) {
      case BOP_EMBED: launch_v(embed_kernel, op.grid, op.block, 0, s, op.em); break;
      case BOP_GEMM: launch_bgemm(B.nt, op.bg, op.smem, s, true); break;
      case BOP_ROPE: launch_v(rope_append_kernel, op.grid, op.block, 0, s, op.rp); break;
      case BOP_ATTN:
        if (op.hd == 128) launch_v(attention_kernel<128>, op.grid, op.block, 0, s, op.at);
        else launch_v(attention_kernel<256>, op.grid, op.block, 0, s, op.at);
        break;
      case BOP_FINAL: launch_v(batch_final_kernel, op.grid, op.block, 0, s, op.fn); break;
    }
  }
}

void Engine::free_batch_steps() {
  for (int i = 0; i < 2; i++) {
    BatchStep* B = bsteps_[i];
    if (!B) continue;
    if (B->graph) cudaGraphExecDestroy(B->graph);
    for (void* p : B->dev) cudaFree(p);
    if (B->h_toks) cudaFreeHost(B->h_toks);
    if (B->h_st) cudaFreeHost(B->h_st);
    if (B->h_res) cudaFreeHost(B->h_res);
    if (B->h_flags) cudaFreeHost(B->h_flags);
    delete B;
    bsteps_[i] = nullptr;
  }
}

std::string Engine::batch_unavailable_reason(int nt) {
  const int i = nt == 4 ? 0 : 1;
  if (nt != 4 && nt != 8) return "the batched step takes 4 or 8 tokens";
  if (tp_world_ > 1) return "tensor parallelism: the batched step runs on one GPU";
  batch_step(nt);
  return bstep_state_[i] == 1 ? std::string() : bstep_why_[i];
}

BatchStep* Engine::batch_step(int nt) {
  const int idx = nt == 4 ? 0 : 1;
  if (bstep_state_[idx] == 1) return bsteps_[idx];
  if (bstep_state_[idx] == -1) return nullptr;
  auto refuse = [&](const std::string& why) -> BatchStep* {
    bstep_state_[idx] = -1;
    bstep_why_[idx] = why;
    return nullptr;
  };
  if (tp_world_ > 1) return refuse("tensor parallelism: the batched step runs on one GPU");
  if (!f_.archive_valid || f_.record_count == 0 || f_.is_raw)
    return refuse("the batched step needs a cell archive");
  const ChpeArch& A = *arch_;
  // Q3: a W8 embedding cell leaves rows >= 8 of the hidden vector as the
  // previous step left them, which a batch of tokens cannot reproduce
  for (uint64_t t = 0; t < (A.V + 15) / 16 && t < f_.record_count; t++)
    if (host_[code_off(t) + 16384 + 20] == 8) return refuse("W8 embedding cells (rows the reference leaves stale)");
  CKV(cudaSetDevice(device_));
  BatchStep* B = new BatchStep();
  B->nt = nt;
  auto dalloc = [&](size_t bytes) -> void* {
    void* p = nullptr;
    CKV(cudaMalloc(&p, bytes < 256 ? 256 : bytes));
    CKV(cudaMemset(p, 0, bytes < 256 ? 256 : bytes));
    B->dev.push_back(p);
    return p;
  };
  const uint32_t qd = A.H * A.HD, kvd = A.KV * A.HD, qkvs = qd + 2 * kvd;
  B->h = (float*)dalloc((size_t)nt * A.D * 4);
  B->qkv = (float*)dalloc((size_t)nt * qkvs * 4);
  B->attn = (float*)dalloc((size_t)nt * qd * 4);
  B->mlp = (float*)dalloc((size_t)nt * A.F * 4);
  B->logits = (float*)dalloc((size_t)nt * A.V * 4);
  B->best = (unsigned long long*)dalloc(8 * 8);
  B->fin = (uint32_t*)dalloc(8 * 4);
  B->flags = (int32_t*)dalloc(16);
  B->st = (StepState*)dalloc(sizeof(StepState));
  B->toks = (int32_t*)dalloc(8 * 4);
  B->res = (StepResult*)dalloc(8 * sizeof(StepResult));
  const int G = (int)(A.H / A.KV);
  B->apart = (float*)dalloc((size_t)nt * A.KV * nsplit_ * G * (A.HD + 4) * 4);
  float* ssq[2] = {(float*)dalloc((size_t)(A.D / kBgRows + 1) * nt * 4),
                   (float*)dalloc((size_t)(A.D / kBgRows + 1) * nt * 4)};
  const float* ssq_prev = nullptr;  // sums of squares the last residual update wrote
  int ssq_next = 0;
  B->acnt = (uint32_t*)dalloc((size_t)nt * A.KV * 4);
  {
    std::vector<uint32_t> ones(8, 1u);
    CKV(cudaMemcpy(B->fin, ones.data(), 32, cudaMemcpyHostToDevice));
  }
  CKV(cudaMallocHost(&B->h_toks, 8 * 4));
  CKV(cudaMallocHost(&B->h_st, sizeof(StepState)));
  CKV(cudaMallocHost(&B->h_res, 8 * sizeof(StepResult)));
  CKV(cudaMallocHost(&B->h_flags, 16));
  size_t part_max = 0, cnt_max = 0;
  std::string why;
  auto gemm = [&](const GemvSrc* src, int nseg, int epi, uint32_t C, const float* x, uint32_t xs,
                  const float* gamma, float* const* out, uint32_t os, int role) -> bool {
    BOp op;
    op.type = BOP_GEMM;
    op.role = role;
    if (!plan_bgemm(src, nseg, epi, C, nt, num_sms_, op.bg, op.smem)) return false;
    for (int i = 0; i < nseg; i++)
      op.alg_bytes += (double)(op.bg.rows_avail[i] > src[i].row0 ? op.bg.rows_avail[i] - src[i].row0 : 0u) *
                      C * (0.5 + 2.0 / 128.0);
    op.bg.x = x;
    op.bg.x_stride = xs;
    op.bg.gamma = gamma;
    op.bg.eps = A.eps;
    for (int i = 0; i < nseg; i++) op.bg.out[i] = out[i];
    op.bg.out_stride = os;
    if (gamma) {
      op.bg.ssq_in = ssq_prev;
      op.bg.ssq_n = A.D / kBgRows;
    }
    if (epi == EPI_ACCUM) {
      op.bg.ssq_out = ssq[ssq_next];
      ssq_next ^= 1;
      ssq_prev = op.bg.ssq_out;
    }
    const size_t pm = (size_t)op.bg.ksplit * nt * op.bg.rows_total;
    if (pm > part_max) part_max = pm;
    if (op.bg.rows_total / kBgRows > cnt_max) cnt_max = op.bg.rows_total / kBgRows;
    B->ops.push_back(op);
    return true;
  };
  try {
    {  // embedding of every token
      BOp op;
      op.type = BOP_EMBED;
      op.role = 7;
      EmbedLaunch& e = op.em;
      e.arc = d_arc_;
      e.record_count = f_.record_count;
      e.stride = f_.stride;
      e.prefix = f_.is_dense ? 64 : 3072 + 64;
      e.D = A.D;
      e.hidden = B->h;
      e.st = B->st;
      e.res = d_res_;
      e.use_state = 2;
      e.tokens = B->toks;
      e.mode = EMB_CELL;
      op.grid = dim3((A.D + 255) / 256, nt);
      B->ops.push_back(op);
    }
    std::vector<float> gam(A.D);
    for (uint32_t l = 0; l < A.L && why.empty(); l++) {
      ChpeLayerInfo li;
      chpe_layer_info(arch_id_, f_.is_raw, l, &li);
      unpack_norm((uint64_t)li.input_norm, gam.data());
      const float* g_in = upload_floats(gam);
      unpack_norm((uint64_t)li.post_norm, gam.data());
      const float* g_post = upload_floats(gam);
      GemvSrc qkv[3] = {plan_linear(li.q_proj, li.q_tiles, qd, A.D, A.D, 0, li.q_bias),
                        plan_linear(li.k_proj, li.k_tiles, kvd, A.D, A.D, 0, li.k_bias),
                        plan_linear(li.v_proj, li.v_tiles, kvd, A.D, A.D, 0, li.v_bias)};
      float* qkv_out[3] = {B->qkv, B->qkv + qd, B->qkv + qd + kvd};
      if (!gemm(qkv, 3, EPI_STORE, A.D, B->h, A.D, g_in, qkv_out, qkvs, 1)) {
        why = "layer " + std::to_string(l) + " QKV is not 4-bit group-scaled flat cells in 128-row blocks";
        break;
      }
      {
        BOp op;
        op.type = BOP_ROPE;
        RopeAppendLaunch& r = op.rp;
        r.qkv = B->qkv;
        r.stride = qkvs;
        r.qd = qd;
        r.kc = d_kc_ + (size_t)l * layer_kv_elems_;
        r.vc = d_vc_ + (size_t)l * layer_kv_elems_;
        r.pages = d_pages_;
        r.page_shift = kKvPageShift;
        r.n_pages = n_pages_;
        r.inv_freq = d_invfreq_;
        r.st = B->st;
        r.KV = (int)A.KV;
        r.HD = (int)A.HD;
        r.max_seq = (int)max_seq_;
        op.grid = dim3(nt, A.KV);
        op.block = dim3(A.HD / 2 < 32 ? 32 : A.HD / 2);
        B->ops.push_back(op);
      }
      {
        BOp op;
        op.type = BOP_ATTN;
        op.role = 2;
        op.hd = (int)A.HD;
        AttnLaunch& at = op.at;
        at.q = B->qkv;
        at.k = B->qkv + qd;
        at.v = B->qkv + qd + kvd;
        at.kc = d_kc_ + (size_t)l * layer_kv_elems_;
        at.vc = d_vc_ + (size_t)l * layer_kv_elems_;
        at.out = B->attn;
        at.part = B->apart;
        at.counters = B->acnt;
        at.inv_freq = d_invfreq_;
        at.st = B->st;
        at.H = (int)A.H;
        at.KV = (int)A.KV;
        at.HD = (int)A.HD;
        at.nsplit = nsplit_;
        at.max_seq = (int32_t)max_seq_;
        at.pages = d_pages_;
        at.page_shift = kKvPageShift;
        at.n_pages = n_pages_;
        at.batched = 1;
        at.q_tok = qkvs;
        at.out_tok = qd;
        at.part_tok = (uint32_t)(A.KV * nsplit_ * G * (A.HD + 4));
        op.grid = dim3(nsplit_, A.KV, nt);
        int th = G * 32;
        if (th < (int)A.HD / 2) th = (int)A.HD / 2;
        if (th < 128) th = 128;
        op.block = dim3(th);
        B->ops.push_back(op);
      }
      GemvSrc o = plan_linear(li.o_proj, li.o_tiles, A.D, A.D, A.D, 1, -1);
      float* o_out[1] = {B->h};
      if (!gemm(&o, 1, EPI_ACCUM, A.D, B->attn, qd, nullptr, o_out, A.D, 3)) {
        why = "layer " + std::to_string(l) + " O is not 4-bit group-scaled flat cells in 128-row blocks";
        break;
      }
      GemvSrc gu[2] = {plan_linear(li.gate_proj, li.gate_tiles, A.F, A.D, A.D, 0, -1),
                       plan_linear(li.up_proj, li.up_tiles, A.F, A.D, A.D, 0, -1)};
      float* gu_out[2] = {B->mlp, nullptr};
      if (!gemm(gu, 2, EPI_SWIGLU, A.D, B->h, A.D, g_post, gu_out, A.F, 4)) {
        why = "layer " + std::to_string(l) + " gate/up is not 4-bit group-scaled flat cells in 128-row blocks";
        break;
      }
      GemvSrc dn = plan_linear(li.down_proj, li.down_tiles, A.D, A.F, A.F, 1, -1);
      float* dn_out[1] = {B->h};
      if (!gemm(&dn, 1, EPI_ACCUM, A.F, B->mlp, A.F, nullptr, dn_out, A.D, 5)) {
        why = "layer " + std::to_string(l) + " down is not 4-bit group-scaled flat cells in 128-row blocks";
        break;
      }
    }
    if (why.empty()) {
      unpack_norm((uint64_t)chpe_final_norm_index(arch_id_, f_.is_raw), gam.data());
      const float* g_fin = upload_floats(gam);
      GemvSrc lm = plan_lm_head();
      float* lm_out[1] = {B->logits};
      if (!gemm(&lm, 1, EPI_LOGITS, A.D, B->h, A.D, g_fin, lm_out, A.V, 6))
        why = "the LM head is not 4-bit group-scaled flat cells in 128-row blocks";
    }
    if (!why.empty()) {
      for (void* p : B->dev) cudaFree(p);
      cudaFreeHost(B->h_toks);
      cudaFreeHost(B->h_st);
      cudaFreeHost(B->h_res);
      cudaFreeHost(B->h_flags);
      delete B;
      return refuse(why);
    }
    {
      BOp op;
      op.type = BOP_FINAL;
      op.fn = BatchFinalLaunch{B->best, B->fin, B->logits, A.V, B->h, A.D, B->res, B->st};
      op.grid = dim3(nt);
      B->ops.push_back(op);
    }
    B->part = (float*)dalloc(part_max * 4);
    B->cnt = (uint32_t*)dalloc(cnt_max * 4);
    const uint32_t gmax = (A.F > A.D ? A.F : A.D) / 128u + 1u;
    uint8_t* pieces = (uint8_t*)dalloc((size_t)gmax * 128u * 4u * nt);
    float* pxsc = (float*)dalloc((size_t)gmax * nt * 8u);
    for (BOp& op : B->ops) {
      if (op.type != BOP_GEMM) continue;
      op.bg.pieces = pieces;
      op.bg.pxsc = pxsc;
      op.bg.part = B->part;
      op.bg.counters = B->cnt;
      op.bg.best = B->best;
      op.bg.finite = B->fin;
      op.bg.bad = B->flags;
      op.bg.err = B->flags + 1;
    }
  } catch (...) {
    for (void* p : B->dev) cudaFree(p);
    delete B;
    throw;
  }
  bsteps_[idx] = B;
  bstep_state_[idx] = 1;
  return B;
}

int Engine::profile_verify(size_t m, uint32_t pos, float* role_ms, double* role_bytes, int cap) {
  const int nt = m <= 4 ? 4 : 8;
  BatchStep* B = batch_step(nt);
  if (!B) throw std::runtime_error("the batched step does not apply: " + bstep_why_[nt == 4 ? 0 : 1]);
  if ((uint64_t)pos + nt > max_seq_) throw std::runtime_error("sequence exceeds max_seq_len");
  CKV(cudaSetDevice(device_));
  kv_ensure((uint64_t)pos + nt);
  for (int i = 0; i < nt; i++) B->h_toks[i] = (int32_t)(1000 + i);
  memset(B->h_st, 0, sizeof(StepState));
  B->h_st->pos = (int32_t)pos;
  B->h_st->finite = 1;
  CKV(cudaMemcpyAsync(B->toks, B->h_toks, 8 * 4, cudaMemcpyHostToDevice, stream_));
  CKV(cudaMemcpyAsync(B->st, B->h_st, sizeof(StepState), cudaMemcpyHostToDevice, stream_));
  const size_t n = B->ops.size();
  std::vector<cudaEvent_t> ev(n + 1);
  for (auto& e : ev) CKV(cudaEventCreate(&e));
  CKV(cudaEventRecord(ev[0], stream_));
  for (size_t i = 0; i < n; i++) {
    run_bop(*B, B->ops[i], stream_);
    CKV(cudaEventRecord(ev[i + 1], stream_));
  }
  CKV(cudaStreamSynchronize(stream_));
  for (int r = 0; r < cap; r++) {
    role_ms[r] = 0.f;
    role_bytes[r] = 0.0;
  }
  for (size_t i = 0; i < n; i++) {
    float ms = 0.f;
    CKV(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
    const int r = B->ops[i].role;
    if (r >= 0 && r < cap) {
      role_ms[r] += ms;
      role_bytes[r] += B->ops[i].alg_bytes;
    }
  }
  for (auto& e : ev) cudaEventDestroy(e);
  return (int)n;
}

bool Engine::verify_batched(const uint32_t* toks, size_t m, uint32_t pos, float* logits_out, uint32_t* argmax_out) {
  const char* env = getenv("CHPE_VERIFY_BATCHED");
  if (env && env[0] == '0') return false;
  if (tp_world_ > 1 || m == 0 || m > 8) return false;
  const int nt = m <= 4 ? 4 : 8;
  if ((uint64_t)pos + (uint64_t)nt > max_seq_) return false;
  BatchStep* B = batch_step(nt);
  if (!B) return false;
  const ChpeArch& A = *arch_;
  CKV(cudaSetDevice(device_));
  if (pos == 0) kv_reset();
  kv_ensure((uint64_t)pos + nt);
  const uint64_t t0 = []() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
  }();
  // candidates, padded with the last one: the padding's KV entries lie at
  // positions the sequence has not reached and are rewritten before any read
  for (int i = 0; i < nt; i++) B->h_toks[i] = (int32_t)toks[(size_t)i < m ? i : m - 1];
  memset(B->h_st, 0, sizeof(StepState));
  B->h_st->pos = (int32_t)pos;
  B->h_st->finite = 1;
  CKV(cudaMemcpyAsync(B->toks, B->h_toks, 8 * 4, cudaMemcpyHostToDevice, stream_));
  CKV(cudaMemcpyAsync(B->st, B->h_st, sizeof(StepState), cudaMemcpyHostToDevice, stream_));
  CKV(cudaMemsetAsync(B->flags, 0, 16, stream_));
  if (B->graph) {
    CKV(cudaGraphLaunch(B->graph, stream_));
  } else {
    run_bops(*B, stream_);
  }
  CKV(cudaGetLastError());
  const size_t V = A.V;
  CKV(cudaMemcpyAsync(B->h_res, B->res, (size_t)nt * sizeof(StepResult), cudaMemcpyDeviceToHost, stream_));
  CKV(cudaMemcpyAsync(B->h_flags, B->flags, 16, cudaMemcpyDeviceToHost, stream_));
  CKV(cudaStreamSynchronize(stream_));
  if (B->h_flags[1]) throw std::runtime_error("a device wait timed out in the batched step");
  if (B->h_flags[0]) return false;  // a residual the early-exit check could react to: sequential steps
  if (logits_out) CKV(cudaMemcpy(logits_out, B->logits, m * V * 4, cudaMemcpyDeviceToHost));
  // the last candidate's logits and result become the engine's last step
  CKV(cudaMemcpyAsync(d_logits_, B->logits + (m - 1) * V, V * 4, cudaMemcpyDeviceToDevice, stream_));
  CKV(cudaMemcpyAsync(d_res_, B->res + (m - 1), sizeof(StepResult), cudaMemcpyDeviceToDevice, stream_));
  h_st_->pos = (int32_t)(pos + m);
  CKV(cudaMemcpyAsync(&d_st_->pos, &h_st_->pos, 4, cudaMemcpyHostToDevice, stream_));
  CKV(cudaStreamSynchronize(stream_));
  for (size_t i = 0; i < m; i++)
    if (argmax_out) argmax_out[i] = B->h_res[i].argmax_token;
  last_ = B->h_res[m - 1];
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  last_ns_ = (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec - t0;
  pos_ = pos + (uint32_t)m;
  if (!B->graph && !B->ran) {
    // the first run set every kernel attribute: record the step as a graph
    B->ran = true;
    cudaStream_t cs;
    CKV(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    cudaGraph_t g;
    CKV(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    run_bops(*B, cs);
    CKV(cudaStreamEndCapture(cs, &g));
    CKV(cudaGraphInstantiate(&B->graph, g, 0));
    CKV(cudaGraphDestroy(g));
    CKV(cudaStreamDestroy(cs));
  }
  return true;
}

}  // namespace chpe
