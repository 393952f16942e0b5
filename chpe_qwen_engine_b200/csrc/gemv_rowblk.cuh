// gemv_rowblk.cuh -- batch-1 GEMV over 4-bit group-scaled flat cells whose
// rows do not start at cell boundaries (the down projections: 29568 columns
// on the 72B, 12288 on the 9B), with the products on the tensor cores.
//
// The flat stream (gemvCellFlat, chpe_engine.zig:583-703) holds the
// row-major [rows x cols] weights in 32768-weight cells, each with its group
// scales in the cell payload.  cols is a multiple of 128, so every 128-weight
// group lies in one row: group j of row r is flat group F = r * G + j (G =
// cols / 128), in cell F / 256 at code offset (F % 256) * 64 and scale
// payload + 48 + 2 (F % 256).
//
// Work split: the columns are cut into ncp parts of at most 120 groups, and
// CTA q * ncp + p takes part p of the rows [R0, R1) of row range q (whole
// 8-row units).  Warp w of the CTA owns the groups p0 + w + 15 i of the part
// (at most 8) with their B operand in registers for the whole launch, so
// shared memory holds only the ring.  A ring stage is one row's part: its
// codes (one bulk copy, or two where the part crosses a cell boundary) and
// one or two windows of its scales.  The first stages are requested before
// the programmatic dependent-launch wait.
//
// Products: the m16n8k32 integer decode of the aligned MMA mode (gemv.cuh,
// mma_b_put_quad): the code bytes masked with 0x0F0F0F0F and 0xF0F0F0F0 are
// the u8 A operand, the int8 pieces of x are B.  A block is 8 consecutive
// rows (MMA rows g = 0..7; rows 8..15 of the operand are zero): once its 8
// stages have landed, every warp runs its groups over them, and the 15 warps'
// partial row sums meet in a shared slot where the warp that arrives last
// adds them in warp order.  With ncp > 1 the parts' row sums go to a global
// [part][row] buffer; the last CTA of the row range to arrive (arrival
// counter, reset by it) adds them in part order and writes the outputs, so
// results do not depend on timing.
//
// Waits are bounded (kMaxWaitPolls); a timeout records StepState::err, the
// consumers stop, the producer waits (bounded) for the copies it issued and
// the CTA writes no output.
#pragma once
#include "gemv.cuh"
#include "gemv_flat_tma.cuh"

namespace chpe {

constexpr uint32_t kRbUnit = 8;                      // rows per block and per unit of the CTA split
// 15 consumer warps + 1 producer = 16 warps, four per scheduler: 128
// registers per thread (17 warps would leave 96)
constexpr uint32_t kRbWarps = 15;
constexpr uint32_t kRbThreads = kRbWarps * 32 + 32;  // + 1 producer warp
constexpr uint32_t kRbMaxGroups = 8;                 // groups per warp (B registers): NGW <= 8
constexpr uint32_t kRbPartGroups = kRbWarps * kRbMaxGroups;  // groups per column part
constexpr uint32_t kRbMaxParts = 4;
constexpr uint32_t kRbMaxStages = 32;
constexpr uint32_t kRbSlots = 4;                     // per-block partial slots

struct RbLayout {
  // bytes per stage (== 64 mod 128: rows g and g + 1 of a block, which one
  // quarter-warp of 16-byte A loads reads, sit in distinct banks), scale window
  uint32_t stage, win;
  uint32_t bst;         // B staging (over the last stages, until the consumers hold B in registers)
  uint32_t xs, bp, bc, wacc, bars, total;
  uint32_t nb;          // stages covered by the B staging
};
// Per stage: the part's codes of one row (gp x 64 bytes), then two windows
// of its scales.
__host__ __device__ inline RbLayout rowblk_layout(uint32_t gp, uint32_t rpc, uint32_t nst) {
  RbLayout l;
  l.win = (2u * gp + 30u + 15u) & ~15u;
  l.stage = gp * 64u + 2u * l.win;
  l.stage += (64u - (l.stage & 127u) + 128u) & 127u;
  l.nb = (gp * 512u + l.stage - 1u) / l.stage;
  l.bst = (nst >= l.nb ? nst - l.nb : 0u) * l.stage;
  l.xs = nst * l.stage;                            // (1/S, x sum) per group of the part
  l.bp = l.xs + kRbPartGroups * 8u;                // [slot][warp][8 rows]
  l.bc = l.bp + kRbSlots * kRbWarps * kRbUnit * 4u;
  l.wacc = l.bc + kRbSlots * 4u;                   // row sums [rpc]
  l.bars = (l.wacc + rpc * 4u + 15u) & ~15u;
  l.total = l.bars + 2u * kRbMaxStages * 8u;
  return l;
}

// The row-block fields of FlatTmaLaunch: P.rc = column parts (ncp), P.nw =
// groups per part (at most 15 NGW), P.rpc = max rows per CTA; P.part_buf
// [ncp][rows] and P.part_cnt [2][row ranges] (arrival counters, abort flags;
// zero between launches).  One segment, P.epi EPI_ACCUM or EPI_STORE, rows a
// multiple of kRbUnit, every row present in the tiles (checked by the host).
template <int NGW>
__global__ void __launch_bounds__(kRbThreads, 1) gemv_rowblk_kernel(const __grid_constant__ FlatTmaLaunch P) {
  static_assert(NGW >= 1 && NGW <= (int)kRbMaxGroups, "groups per warp");
  extern __shared__ __align__(128) uint8_t rsm[];
  constexpr uint32_t NW = kRbWarps, NCT = NW * 32;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, L = tid & 31u;
  const uint32_t C = P.ncols, G = C >> 7, nst = P.nst, ncp = P.rc, gpn = P.nw;
  const uint32_t q = blockIdx.x / ncp, p = blockIdx.x - q * ncp, nrr = gridDim.x / ncp;
  const uint32_t p0 = p * gpn, gp = G - p0 < gpn ? G - p0 : gpn;  // this part's groups [p0, p0 + gp)
  const RbLayout lay = rowblk_layout(gpn, P.rpc, nst);
  float* xsc = reinterpret_cast<float*>(rsm + lay.xs);
  float* bpart = reinterpret_cast<float*>(rsm + lay.bp);
  uint32_t* bcnt = reinterpret_cast<uint32_t*>(rsm + lay.bc);
  float* wacc = reinterpret_cast<float*>(rsm + lay.wacc);
  uint64_t* full = reinterpret_cast<uint64_t*>(rsm + lay.bars);
  uint64_t* empty = full + kRbMaxStages;
  __shared__ int s_abort, s_last;
  __shared__ volatile int s_bad;

  const GemvSrc& S = P.src[0];
  const uint32_t Ut = P.row_start[1] / kRbUnit;
  const uint32_t R0 = kRbUnit * (uint32_t)((uint64_t)Ut * q / nrr);
  const uint32_t R1 = kRbUnit * (uint32_t)((uint64_t)Ut * (q + 1) / nrr);
  const uint32_t nrows = R1 - R0, nblk = nrows / kRbUnit;

  if (tid == 0) {
    s_abort = 0;
    s_bad = 0;
    for (uint32_t i = 0; i < nst; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // ---- producer warp: lane r issues row i0 + r of each batch -------------------
  if (warp == NW) {
    uint32_t issued = 0;
    auto issue = [&](uint32_t i) {  // stage i % nst <- row R0 + i, groups [p0, p0 + gp)
      const uint32_t s = i % nst;
      const uint32_t F0 = (S.row0 + R0 + i) * G + p0, k0 = F0 >> 8, f0 = F0 & 255u;
      const uint32_t n1 = 256u - f0 < gp ? 256u - f0 : gp;  // groups in the first cell
      const uint32_t sa = (48u + 2u * f0) & ~15u;
      const uint32_t sb1 = ((48u + 2u * (f0 + n1) + 15u) & ~15u) - sa;
      const uint32_t sb2 = n1 < gp ? ((48u + 2u * (gp - n1) + 15u) & ~15u) - 48u : 0u;
      uint8_t* dst = rsm + s * lay.stage;
      const uint8_t* t0 = S.arc + S.tile0 + (uint64_t)k0 * S.stride;
      mbar_expect_tx(&full[s], gp * 64u + sb1 + sb2);
      bulk_g2s(dst, t0 + f0 * 64u, n1 * 64u, &full[s]);
      bulk_g2s(dst + gpn * 64u, t0 + 16384u + sa, sb1, &full[s]);
      if (n1 < gp) {
        const uint8_t* t1 = t0 + S.stride;
        bulk_g2s(dst + n1 * 64u, t1, (gp - n1) * 64u, &full[s]);
        bulk_g2s(dst + gpn * 64u + lay.win, t1 + 16384u + 48u, sb2, &full[s]);
      }
    };
    auto drain = [&]() {  // copies in flight complete before the CTA exits
      const uint32_t from = issued > nst ? issued - nst : 0u;
      for (uint32_t i = from; i < issued; i++) mbar_wait(&full[i % nst], (i / nst) & 1u);
    };
    {
      // the last nb stages hold the B staging until the consumers' prologue ends
      uint32_t nfree = nst - lay.nb;
      if (P.npre && P.npre < nfree) nfree = P.npre;
      const uint32_t npre = nrows < nfree ? nrows : nfree;
      for (uint32_t i = L; i < npre; i += 32u) issue(i);
      issued = npre;
    }
    __syncthreads();  // consumers' prologue done: B in registers, s_abort final
    if (s_abort) {
      if (L == 0) drain();
      return;
    }
    while (issued < nrows) {
      // a batch of up to 8 rows (the stages one block releases), one per lane
      const uint32_t nb8 = nrows - issued < kRbUnit ? nrows - issued : kRbUnit;
      const uint32_t i = issued + L;
      bool ok = true;
      if (L < nb8 && i >= nst) ok = mbar_wait_or_abort(&empty[i % nst], ((i / nst) - 1u) & 1u, &s_bad);
      if (!__all_sync(0xffffffffu, ok)) {
        if (L == 0) {
          atomicExch(&P.st->err, 1);
          s_bad = 1;
        }
        break;
      }
      if (L < nb8) {
        fence_proxy_async_smem();
        issue(i);
      }
      issued += nb8;
    }
    if (L == 0) drain();
    return;
  }

  // ---- consumers: B pieces of the part's x into registers ---------------------
  pdl_wait();
  if (tid == 0) {
    int ab = (!P.ignore_stop && P.st->stop) ? 1 : 0;
    if (!ab && !tp_wait(P.tp)) {  // inputs from the other ranks
      atomicExch(&P.st->err, 1);
      ab = 1;
    }
    s_abort = ab;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
  const uint32_t g = L >> 2, t = L & 3u;
  uint2 breg[NGW][4];
  if (!s_abort) {
    for (uint32_t i = tid; i < nrows; i += NCT) wacc[i] = 0.f;
    for (uint32_t i = tid; i < kRbSlots; i += NCT) bcnt[i] = 0u;
    const float4* x4 = reinterpret_cast<const float4*>(P.x) + 32u * p0;
    // warp w stages the part's groups w, w + NW, ...: lane L holds quad 32 jl
    // + L (every load in flight before the first is used)
    float4 xv[NGW];
#pragma unroll
    for (int i = 0; i < NGW; i++) {
      const uint32_t jl = warp + NW * (uint32_t)i;
      xv[i] = jl < gp ? x4[32u * jl + L] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < NGW; i++) {
      const uint32_t jl = warp + NW * (uint32_t)i;
      if (jl < gp) mma_b_put_quad(rsm + lay.bst, xsc, 32u * jl + L, xv[i], L);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
    const uint2* bfr = reinterpret_cast<const uint2*>(rsm + lay.bst) + t * kMmaPieces + (g < kMmaPieces ? g : 0u);
#pragma unroll
    for (uint32_t i = 0; i < (uint32_t)NGW; i++) {
      const uint32_t jl = warp + NW * i;
#pragma unroll
      for (uint32_t k = 0; k < 4; k++)
        breg[i][k] = (g < kMmaPieces && jl < gp) ? bfr[jl * (4u * 4u * kMmaPieces) + k * 4u * kMmaPieces]
                                                 : make_uint2(0u, 0u);
    }
  }
  __syncthreads();  // with the producer: the staging stages are free, the abort decision is final
  if (s_abort) {
    if (tid == 0) {
      if (ncp > 1) {
        // the row range's outputs stay unwritten: mark it, and arrive
        atomicExch(&P.part_cnt[nrr + q], 1u);
        __threadfence();
        if (atomicAdd(&P.part_cnt[q], 1u) == ncp - 1u) {
          P.part_cnt[q] = 0u;
          P.part_cnt[nrr + q] = 0u;
          tp_signal_n(P.tp, P.tp.signal_sig, ncp);
        }
      } else {
        tp_signal(P.tp, P.tp.signal_sig);  // every CTA arrives once per launch
      }
    }
    return;
  }
  pdl_launch_dependents();

  // ---- main loop: 8-row blocks ------------------------------------------------
  // pieces 2t and 2t+1 sit in this lane's two D columns
  const float pw0 = t == 0u ? 1.0f : t == 1u ? 6.103515625e-05f : 0.0f;          // 128^-(2t)
  const float pw1 = t == 0u ? 7.8125e-03f : t == 1u ? 4.76837158203125e-07f : 0.0f;  // 128^-(2t+1)
  const float corr = t == 0u ? 8.0f : 0.0f;  // the x-sum term, once per row (lane t = 0)
  bool bad = false;
  for (uint32_t b = 0; b < nblk && !bad; b++) {
    const uint32_t i0 = b * kRbUnit;
    for (uint32_t r = 0; r < kRbUnit; r++) {
      const uint32_t i = i0 + r;
      if (!mbar_wait_or_abort(&full[i % nst], (i / nst) & 1u, &s_bad)) {
        bad = true;
        break;
      }
    }
    if (bad) break;
    // row g of the block: its stage, and where its part's groups fall in cells
    const uint8_t* stg = rsm + ((i0 + g) % nst) * lay.stage;
    const uint32_t F0 = (S.row0 + R0 + i0 + g) * G + p0;
    const uint32_t sa = (48u + 2u * (F0 & 255u)) & ~15u, k0 = F0 >> 8;
    float acc = 0.f;
#pragma unroll
    for (uint32_t i = 0; i < (uint32_t)NGW; i++) {
      // every iteration runs (the warp's groups past the part have zero
      // operands and add nothing), so the groups' loads and MMAs interleave
      const uint32_t jl = warp + NW * i;
      const bool on = jl < gp;
      const uint4 w = on ? *reinterpret_cast<const uint4*>(stg + jl * 64u + t * 16u) : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t F = F0 + jl;
      const uint32_t so = (F >> 8) == k0 ? 48u + 2u * (F & 255u) - sa : lay.win + 2u * (F & 255u);
      const float sc = on ? ld_f16(stg + gpn * 64u + so) : 0.f;
      const float invS = on ? xsc[2 * jl] : 0.f, xs = on ? xsc[2 * jl + 1] : 0.f;
      // four independent MMAs (k-steps x lo/hi), added in s32: exact
      int d[4][4] = {};
#pragma unroll
      for (uint32_t ks = 0; ks < 2; ks++) {
        const uint32_t a0 = word_of(w, (int)(2 * ks)), a2 = word_of(w, (int)(2 * ks + 1));
        mma_u8s8_16832(d[2 * ks], a0 & 0x0F0F0F0Fu, 0u, a2 & 0x0F0F0F0Fu, 0u, breg[i][2 * ks].x, breg[i][2 * ks].y);
        mma_u8s8_16832(d[2 * ks + 1], a0 & 0xF0F0F0F0u, 0u, a2 & 0xF0F0F0F0u, 0u, breg[i][2 * ks + 1].x,
                       breg[i][2 * ks + 1].y);
      }
      const int e0 = (d[0][0] + d[1][0]) + (d[2][0] + d[3][0]), e1 = (d[0][1] + d[1][1]) + (d[2][1] + d[3][1]);
      const float v = fmaf(s32_exact(e1), pw1, s32_exact(e0) * pw0);
      acc = fmaf(sc, fmaf(v, invS, -corr * xs), acc);
    }
    __syncwarp();
    if (L == 0)
      for (uint32_t r = 0; r < kRbUnit; r++) mbar_arrive(&empty[(i0 + r) % nst]);
    // lanes t = 0 and 1 hold pieces n = 0,1 and n = 2,3; t = 2, 3 zeros
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    const uint32_t slot = b % kRbSlots;
    float* bp = bpart + slot * (NW * kRbUnit);
    if (t == 0u) bp[warp * kRbUnit + g] = acc;
    __threadfence_block();
    __syncwarp();
    uint32_t last = 0;
    if (L == 0) last = atomicAdd(&bcnt[slot], 1u) == NW - 1u ? 1u : 0u;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      // every warp's partials of this block are in: add them in warp order
      __threadfence_block();
      if (L < kRbUnit) {
        float sum = 0.f;
#pragma unroll
        for (uint32_t w = 0; w < NW; w++) sum += bp[w * kRbUnit + L];
        wacc[i0 + L] = sum;
      }
      if (L == 0) bcnt[slot] = 0u;
      __syncwarp();
    }
  }
  if (bad && L == 0) {
    atomicExch(&P.st->err, 1);
    s_bad = 1;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");

  // ---- the row range's parts meet; its last CTA writes the outputs ----------
  if (ncp > 1) {
    if (!s_bad)
      for (uint32_t lr = tid; lr < nrows; lr += NCT) P.part_buf[(size_t)p * P.row_start[1] + R0 + lr] = wacc[lr];
    __threadfence();
    asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
    if (tid == 0) {
      if (s_bad) atomicExch(&P.part_cnt[nrr + q], 1u);
      __threadfence();
      s_last = atomicAdd(&P.part_cnt[q], 1u) == ncp - 1u;
      if (s_last) {
        if (atomicExch(&P.part_cnt[nrr + q], 0u) != 0u) s_bad = 1;
        P.part_cnt[q] = 0u;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
    if (!s_last) return;  // the last CTA of the row range signals for all of them
    __threadfence();
    if (s_bad) {
      if (tid == 0) tp_signal_n(P.tp, P.tp.signal_sig, ncp);
      return;
    }
    for (uint32_t lr = tid; lr < nrows; lr += NCT) {
      float v = 0.f;
      for (uint32_t pp = 0; pp < ncp; pp++) v += __ldcg(P.part_buf + (size_t)pp * P.row_start[1] + R0 + lr);
      wacc[lr] = v;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
  } else if (s_bad) {
    if (tid == 0) tp_signal(P.tp, P.tp.signal_sig);
    return;
  }

  // ---- epilogue: rows of this row range ---------------------------------------
  float* y = P.out[0];
  for (uint32_t lr = tid; lr < nrows; lr += NCT) {
    const uint32_t r = R0 + lr;
    const float d0 = wacc[lr];
    if (P.epi == EPI_ACCUM) {
      float v = y[r] + d0;
      if (S.bias) v += S.bias[r];
      tp_put(P.tp, y, r, v);
    } else {
      tp_put(P.tp, y, r, S.bias ? d0 + S.bias[r] : d0);
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
  if (tid == 0) tp_signal_n(P.tp, P.tp.signal_sig, ncp);
}

}  // namespace chpe
