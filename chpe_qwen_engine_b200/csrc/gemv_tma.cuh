// gemv_tma.cuh -- row-block GEMV with a TMA pipeline through shared memory.
//
// For tensors stored as blocks of R full 2048-wide rows with contiguous codes:
// the row-tiled cells of the 3B archives (W4/W2: 16 rows of 1024/512 bytes,
// FP16/BF16 cells: 4 rows of 4096 bytes) and the raw FP16/BF16 tiles of the
// 3B raw archives (4 rows per 16 KiB tile).  This is the reference's
// gemvTilePolymorphic path (chpe_engine.zig:223-581, dispatch :1430-1442) and
// the raw dotSegment path for 2048 columns (:1194-1254, :1455-1479), plus the
// tied LM head over embedding cells (:1582-1611, unpackEmbedRowCell :1288-1394).
//
// Each CTA (512 threads, one per SM) owns a contiguous range of blocks.  Thread
// 0 streams them with cp.async.bulk into a NST-stage ring of shared memory;
// each stage has an mbarrier the bulk copies complete on.  The first NST
// blocks are requested before the programmatic-dependent-launch wait, so they
// arrive while the previous kernel finishes.  Consumers hold x in registers
// (a warp covers whole rows, or a quarter row for FP16/BF16), read the codes
// from shared memory and decode them as gemv.cuh does.  Every mbarrier wait is
// bounded; on a timeout the kernel records StepState::err, drains the copies it
// issued (again bounded) and returns.
#pragma once
#include "gemv.cuh"

namespace chpe {

template <int FMT> struct RowBlock;
template <> struct RowBlock<FMT_W4G> { static constexpr int R = 16, WPR = 1; };
template <> struct RowBlock<FMT_W4SB> { static constexpr int R = 16, WPR = 1; };
template <> struct RowBlock<FMT_W2G> { static constexpr int R = 16, WPR = 1; };
template <> struct RowBlock<FMT_W2SB> { static constexpr int R = 16, WPR = 1; };
template <> struct RowBlock<FMT_F16> { static constexpr int R = 4, WPR = 4; };
template <> struct RowBlock<FMT_BF16> { static constexpr int R = 4, WPR = 4; };

struct TmaLaunch {
  GemvSrc src[3];
  float* out[3];
  uint32_t unit_start[4];  // prefix of blocks over segments (SwiGLU: blocks of segment 0)
  int32_t nseg;
  int32_t epi;
  const float* x;          // hidden when norm != 0, else the input vector
  const float* gamma;
  float eps;
  int32_t norm;
  int32_t check_layer;
  StepState* st;
  int32_t ignore_stop;
  StepResult* res;
  int32_t* gen_tokens;
  int32_t max_gen;
  uint32_t payload;        // 1: also copy the first 832 payload bytes of each block
};

constexpr uint32_t kPayloadHead = 832;  // tile metadata, dims, group scales, row outliers
constexpr uint32_t kTmaStageOff = 9216;  // x copy 8 KiB, barriers 256 B, partials 512 B, pad

// Last-CTA finalisation of a step (chpe_engine.zig:1775-1802): argmax key,
// finiteness, token-0 logit, hidden norm; advances the step state.
CHPE_DEV void finalize_logits(StepState* st, StepResult* res, float token0, float hidden_ss,
                              int32_t* gen_tokens, int32_t max_gen) {
  __threadfence();
  unsigned long long b = atomicAdd(&st->best, 0ull);
  StepResult Rr;
  Rr.argmax_token = b ? 0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull) : 0u;
  Rr.max_logit = b ? key_value(b) : -1e30f;
  Rr.token0_logit = token0;
  Rr.hidden_norm = sqrtf(hidden_ss);
  Rr.all_finite = (int32_t)atomicAdd(&st->finite, 0u);
  Rr.pos = st->pos;
  *res = Rr;
  if (gen_tokens && st->n_gen < max_gen) gen_tokens[st->n_gen] = (int32_t)Rr.argmax_token;
  st->n_gen += 1;
  st->pos += 1;
  st->best = 0ull;
  st->finite = 1u;
  st->done_ctas = 0u;
}

template <int FMT, int NST>
__global__ void __launch_bounds__(512, 1) gemv_tma_kernel(const __grid_constant__ TmaLaunch P) {
  using FI = FmtInfo<FMT>;
  constexpr int R = RowBlock<FMT>::R, WPR = RowBlock<FMT>::WPR;
  constexpr int CW = FI::CW, QPC = CW / 4;
  constexpr int CPW = 2048 / CW / WPR;  // chunks per warp-row segment
  constexpr int SL = CPW / 32;          // chunk slots per lane
  constexpr uint32_t ROWB = 2048u * FI::BITS / 8;
  static_assert(R * WPR == 16, "16 warps cover one block");
  static_assert(SL >= 1 && CPW % 32 == 0, "row geometry");

  extern __shared__ __align__(128) uint8_t tsm[];
  float* xsh = reinterpret_cast<float*>(tsm);                  // x, lane-permuted (xpos)
  uint64_t* bars = reinterpret_cast<uint64_t*>(tsm + 8192);   // NST (<= 32) barriers
  float* red = reinterpret_cast<float*>(tsm + 8192 + 256);    // [2 units][2 parts][32] partials
  uint8_t* stages = tsm + kTmaStageOff;
  __shared__ float sred[16];
  __shared__ unsigned long long kbest[16];
  __shared__ uint32_t kfin[16];
  __shared__ int is_last;

  const uint32_t tid = threadIdx.x, warp = tid >> 5, L = tid & 31;
  const bool swig = P.epi == EPI_SWIGLU;
  const uint32_t nparts = swig ? 2u : 1u;
  const uint32_t part_bytes = (uint32_t)R * ROWB + (P.payload ? kPayloadHead : 0u);
  const uint32_t stage_bytes = (nparts * part_bytes + 127u) & ~127u;
  const uint32_t total_units = swig ? P.unit_start[1] : P.unit_start[P.nseg];
  const uint32_t u0 = (uint32_t)((uint64_t)total_units * blockIdx.x / gridDim.x);
  const uint32_t u1 = (uint32_t)((uint64_t)total_units * (blockIdx.x + 1) / gridDim.x);
  const uint32_t nmine = u1 - u0;

  // block u of the launch -> (segment, block index inside the segment)
  auto locate = [&](uint32_t u, uint32_t& seg, uint32_t& k) {
    seg = 0;
    if (!swig)
      while ((int)seg + 1 < P.nseg && u >= P.unit_start[seg + 1]) seg++;
    k = u - P.unit_start[seg];
  };
  auto issue = [&](uint32_t i) {  // thread 0: block u0+i into stage i % NST
    uint8_t* dst = stages + (i % NST) * stage_bytes;
    uint64_t* bar = &bars[i % NST];
    mbar_expect_tx(bar, nparts * part_bytes);
    uint32_t seg, k;
    locate(u0 + i, seg, k);
    for (uint32_t p = 0; p < nparts; p++) {
      const GemvSrc& s = P.src[swig ? p : seg];
      const uint8_t* blk = s.arc + s.tile0 + (uint64_t)k * s.stride;
      bulk_g2s(dst + p * part_bytes, blk, (uint32_t)R * ROWB, bar);
      if (P.payload) bulk_g2s(dst + p * part_bytes + R * ROWB, blk + 16384, kPayloadHead, bar);
    }
  };

  if (tid == 0) {
    for (int i = 0; i < NST; i++) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t npre = nmine < (uint32_t)NST ? nmine : (uint32_t)NST;
  if (tid == 0)
    for (uint32_t i = 0; i < npre; i++) issue(i);

  // Waits for the copies of blocks [from, issued) before an early return.
  auto drain = [&](uint32_t from) {
    if (tid != 0) return;
    uint32_t issued = from + NST < nmine ? from + NST : nmine;
    if (issued < npre) issued = npre;
    for (uint32_t i = from; i < issued; i++) mbar_wait(&bars[i % NST], (i / NST) & 1u);
  };

  pdl_wait();
  if (!P.ignore_stop && P.st->stop) {
    drain(0);
    return;
  }

  // ---- x: RMSNorm'ed hidden or the plain input, into registers ------------
  float tot = 0.f;
  {
    const float4 v = reinterpret_cast<const float4*>(P.x)[tid];  // 512 threads x 4 = 2048
    if (P.norm) {
      float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      ss = warp_sum(ss);
      if (L == 0) sred[warp] = ss;
      __syncthreads();
      for (int w = 0; w < 16; w++) tot += sred[w];
      if (P.check_layer >= 0) {
        const int l = P.check_layer;
        const bool cond = l < 3 || (l >= 8 && l <= 16) || !isfinite(P.x[0]);
        if (cond && !isfinite(tot)) {
          if (blockIdx.x == 0 && tid == 0) P.st->stop = 1;
          drain(0);
          return;
        }
      }
      const float inv = 1.0f / sqrtf(tot / 2048.0f + P.eps);
      const float4 g = reinterpret_cast<const float4*>(P.gamma)[tid];
      float4 o;
      o.x = v.x * inv * g.x;
      o.y = v.y * inv * g.y;
      o.z = v.z * inv * g.z;
      o.w = v.w * inv * g.w;
      *reinterpret_cast<float4*>(&xsh[xpos<CW>(4 * tid)]) = o;
    } else {
      *reinterpret_cast<float4*>(&xsh[xpos<CW>(4 * tid)]) = v;
    }
  }
  __syncthreads();
  const uint32_t rw = warp / WPR, wq = warp % WPR;  // row in block, quarter of the row
  f2x xp[SL][CW / 2];  // this lane's x, as packed pairs
  float xsm[SL];
#pragma unroll
  for (int j = 0; j < SL; j++) {
    // x is staged lane-permuted (xpos): quad q of chunk c = L + 32*jj sits at
    // ((jj*QPC + q)*32 + L)*4, so these 128-bit loads are conflict free
    const uint32_t jj = (wq * CPW) / 32 + j;
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < QPC; q++) {
      const float4 t = xquad<CW>(xsh, jj, q, L);
      xp[j][2 * q] = pack2(t.x, t.y);
      xp[j][2 * q + 1] = pack2(t.z, t.w);
      s += (t.x + t.y) + (t.z + t.w);
    }
    xsm[j] = s;
  }
  pdl_launch_dependents();

  unsigned long long lbest = 0ull;
  uint32_t lfin = 1u;
  for (uint32_t i = 0; i < nmine; i++) {
    const uint32_t stage = i % NST;
    const bool ok = mbar_wait(&bars[stage], (i / NST) & 1u);
    if (__syncthreads_or(!ok)) {  // one decision for the whole CTA
      if (tid == 0) atomicExch(&P.st->err, 1);
      drain(i);
      return;
    }
    const uint8_t* sp = stages + stage * stage_bytes;
    uint32_t seg, k;
    locate(u0 + i, seg, k);
    float part[2];
#pragma unroll
    for (uint32_t p = 0; p < 2; p++) {
      part[p] = 0.f;
      if (p >= nparts) break;
      const GemvSrc& s = P.src[swig ? p : seg];
      const uint8_t* rowp = sp + p * part_bytes + rw * ROWB;
      const uint8_t* pl = sp + p * part_bytes + R * ROWB;  // payload head copy
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < SL; j++) {
        const uint32_t ch = wq * CPW + L + 32u * j;  // chunk index in the row
        const uint4 v = *reinterpret_cast<const uint4*>(rowp + 16u * ch);
        f2x a0 = 0ull, a1 = 0ull;
#pragma unroll
        for (int q = 0; q < QPC; q++) quad_fma<FMT>(v, q, xp[j][2 * q], xp[j][2 * q + 1], (q & 1) ? a1 : a0);
        const float d = chunk_finish<FMT>(a0, a1, xsm[j]);
        if constexpr (FI::GROUPED) {
          acc = fmaf(d, ld_f16(pl + 48 + 2 * (rw * 16 + ch * CW / 128)), acc);
        } else if constexpr (FI::SB) {
          acc = fmaf(ld_f32(pl + 36), xsm[j], fmaf(d, ld_f32(pl + 32), acc));
        } else {
          acc += d;
        }
      }
      if constexpr (FI::GROUPED && R == 16) {
        if (s.outliers != OUTL_NONE && L < 8) {
          // row outliers (chpe_engine.zig:244-256, 309-315) or, for the tied
          // LM head, replacements (:1335-1344, :1369-1378)
          const uint32_t col = ld_u16(pl + 816 + 2 * L);
          if (col < s.x_len) {
            const float w = ld_f16(pl + 560 + 2 * (rw * 8 + L));
            const float xcol = xsh[xpos<CW>(col)];
            if (s.outliers == OUTL_ADD) {
              acc = fmaf(w, xcol, acc);
            } else {
              bool later = false;
              for (uint32_t k2 = L + 1; k2 < 8; k2++) later |= ld_u16(pl + 816 + 2 * k2) == col;
              if (!later) {
                const float sc = ld_f16(pl + 48 + 2 * (rw * 16 + (col >> 7)));
                float dec;
                if constexpr (FI::BITS == 4) {
                  const uint8_t b = rowp[col / 2];
                  dec = ((float)((col & 1) ? (b >> 4) & 15 : b & 15) - 8.0f) * sc;
                } else {
                  const float CB[4] = {0.f, 1.f, -2.f, -1.f};
                  const uint8_t b = rowp[col / 4];
                  dec = CB[(b >> (2 * (col & 3))) & 3] * sc;
                }
                acc = fmaf(w - dec, xcol, acc);
              }
            }
          }
        }
      }
      part[p] = warp_sum(acc);
    }
    float rowv[2] = {part[0], part[1]};
    if constexpr (WPR > 1) {
      float* rb = red + (i & 1u) * 64;
      if (L == 0) { rb[warp] = part[0]; rb[32 + warp] = part[1]; }
    }
    __syncthreads();  // stage consumed (and quarter-row partials visible)
    if (tid == 0 && i + NST < nmine) {
      fence_proxy_async_smem();
      issue(i + NST);
    }
    if constexpr (WPR > 1) {
      if (wq != 0) continue;
      const float* rb = red + (i & 1u) * 64;
      rowv[0] = rb[warp] + rb[warp + 1] + rb[warp + 2] + rb[warp + 3];
      rowv[1] = rb[32 + warp] + rb[32 + warp + 1] + rb[32 + warp + 2] + rb[32 + warp + 3];
    }
    if (L != 0) continue;
    const uint32_t r = k * R + rw;
    if (swig) {
      P.out[0][r] = silu_ref(rowv[0]) * rowv[1];
      continue;
    }
    const GemvSrc& s = P.src[seg];
    float* y = P.out[seg];
    const float d = rowv[0];
    if (P.epi == EPI_LOGITS) {
      y[r] = d;
      if (!isfinite(d)) lfin = 0u;
      if (d > -1e30f) {
        const unsigned long long kk = argmax_key(d, r);
        lbest = kk > lbest ? kk : lbest;
      }
    } else if (P.epi == EPI_ACCUM) {
      float v = y[r] + d;
      if (s.bias) v += s.bias[r];
      y[r] = v;
    } else {
      y[r] = s.bias ? d + s.bias[r] : d;
    }
  }
  if (P.epi == EPI_LOGITS) {
    if (L == 0) { kbest[warp] = lbest; kfin[warp] = lfin; }
    __syncthreads();
    if (tid == 0) {
      unsigned long long b = 0ull;
      uint32_t f = 1u;
      for (int w = 0; w < 16; w++) { b = kbest[w] > b ? kbest[w] : b; f &= kfin[w]; }
      if (b) atomicMax(&P.st->best, b);
      if (!f) atomicAnd(&P.st->finite, 0u);
      __threadfence();
      is_last = atomicAdd(&P.st->done_ctas, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last && tid == 0) finalize_logits(P.st, P.res, __ldcg(P.out[0]), tot, P.gen_tokens, P.max_gen);
  }
}

}  // namespace chpe
