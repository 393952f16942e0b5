// gemv_flat_tma.cuh -- GEMV over flat weight streams with a warp-specialised
// TMA pipeline.
//
// Covers the two layouts whose rows run across tile boundaries:
//   * flat cells (gemvCellFlat, chpe_engine.zig:583-703, dispatch :1443-1454):
//     each 32768-weight cell holds a slice of the row-major [rows x cols]
//     stream, with its scales in the cell payload (group g = offset/128 of the
//     cell, or one scale/bias per cell);
//   * raw tiles (dotSegment, :1194-1254, :1455-1479): one contiguous FP16 /
//     BF16 / int8 stream.
// Every tensor of the 72B and 9B archives and the 3B down projection (11008
// columns) take one of these.
//
// Work split: CTA b owns rows [Rt*b/G, Rt*(b+1)/G) of the concatenated call
// (q|k|v, or gate and up for SwiGLU), i.e. one contiguous flat range per
// tensor.  The range is cut at tile boundaries into pieces of at most one
// tile (16 KiB of codes).  A producer warp streams the pieces with
// cp.async.bulk into an NST-stage ring; full[s] completes on the copied bytes,
// empty[s] on one arrival per consumer warp, so no CTA-wide barrier sits in
// the loop.  The first NST pieces are requested before the programmatic
// dependent-launch wait.
//
// Consumers: 16 warps.  Warp w decodes chunks [w*CPWARP, (w+1)*CPWARP) of each
// piece (2 chunks per lane for 16 KiB pieces), lane L the chunks
// w*CPWARP + L + 32j, all of its code loads issued before the decode.  A warp's run spans at most two
// rows (CPWARP*CW <= cols, checked by the host), so a lane keeps two partial
// sums; the warp reduces them and lane 0 adds them to its own per-row slots
// wacc[part][warp][row].  After the last piece the slots are summed over the
// warps in a fixed order, so results do not depend on timing.  x sits in
// shared memory in the lane-permuted layout (xpos), which keeps the quad
// loads of consecutive chunks conflict free, with one x-sum per chunk.
//
// Waits are bounded (kMaxWaitPolls); a timeout records StepState::err, the
// CTA stops consuming, the producer waits (bounded) for the copies it issued
// and the outputs of the CTA are not written.
#pragma once
#include "gemv.cuh"
#include "gemv_tma.cuh"

namespace chpe {

struct FlatTmaLaunch {
  GemvSrc src[3];
  float* out[3];
  uint32_t row_start[4];   // prefix of rows over segments (SwiGLU: [0, rows])
  int32_t nseg;
  int32_t epi;
  uint32_t ncols;          // x length = columns of every segment
  uint32_t rpc;            // max rows per CTA (size of the per-warp row slots)
  uint32_t nst;            // stages in the ring (<= kFlatMaxStages)
  uint32_t rc;             // aligned cells: rows per cell (32768 / cols); CTA rows are multiples
  uint32_t mode;           // FlatMode the launch was planned for (host side)
  uint32_t nw;             // consumer warps the launch was planned for (16, or 8 for two CTAs per SM)
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
  float* xn_out;           // normalised x for the down_aux fix-up op (or null)
  TpLink tp;               // tensor-parallel wait / exchange / signal (world 1: none)
  uint32_t npre;           // pieces (rows) requested before the dependency wait at most (0: the free stages)
  uint32_t cov[3];         // per segment (SwiGLU: cov[0] for the gate/up pair): its leading rows that
                           // have weights in the tiles; the CTAs split these, the rest are zero sums
  float* part_buf;         // ROWBLK with column parts: [part][rows] row sums
  uint32_t* part_cnt;      // ROWBLK with column parts: arrival counters and abort flags per row range
};

// codes + payload head (832) rounded to 128, + 64 so that consecutive stages
// sit half a bank row apart (the MMA mode reads one row of each of two cells
// per load)
constexpr uint32_t kFlatStageBytes = 16384 + 896 + 64;
constexpr uint32_t kFlatMaxStages = 16;
// Consumer warps per CTA: 16 (one CTA per SM), or 8 for aligned launches
// whose shared memory fits twice per SM, so that the next launch's CTAs are
// resident and streaming while this one's finish.
constexpr uint32_t kFlatConsumerWarps = 16;         // each decodes 1/16 of every piece
constexpr uint32_t kFlatConsumers = kFlatConsumerWarps * 32;
constexpr uint32_t kFlatThreads = kFlatConsumers + 32;  // + 1 producer warp
constexpr uint32_t kFlatThreadsHalf = 8 * 32 + 32;      // 8 consumer warps + 1 producer
// Column-owner launches run 15 consumer warps: 16 warps in all, four per
// scheduler, which leaves each thread 128 registers (17 warps would cap it at
// 96) for x in registers.
constexpr uint32_t kFlatColownWarps = 15;
constexpr uint32_t kFlatColownThreads = kFlatColownWarps * 32 + 32;
constexpr uint32_t kFlatMaxRanges = 8;

struct FlatRange {
  uint32_t src;     // index into src[]
  uint32_t part;    // 0, or 1 for the up half of SwiGLU
  uint32_t fa0, fb0;// tensor-relative flat weight range [fa0, fb0)
  uint32_t k0;      // first tile
  uint32_t pstart;  // index of its first piece
  int32_t lrbase;   // tensor row + lrbase = CTA-local row
  uint32_t pad;
};

struct FlatLayout {
  uint32_t x, xs, wacc, bars, ranges, total;
  uint32_t bp, bc;  // MMA mode: per-block partial sums and their arrival counters
};

// MMA mode (FLAT_MMA): 16-row blocks, x as int8 B fragments (four pieces per
// value, one power-of-two exponent per 128-column group).
constexpr uint32_t kMmaRows = 16;
constexpr uint32_t kMmaSlots = 8;   // per-block partial slots (host: >= ceil(nst / cells per block) + 1)
// B fragments ([group][kstep][kind][t][piece] x 8 bytes) are staged in the
// ring's last stages, which the producer fills only after every consumer warp
// has copied its groups' fragments into registers.
__host__ __device__ inline uint32_t flat_mma_b_stages(uint32_t ncols) {
  return ((ncols / 128u) * 2u * 2u * 4u * kMmaPieces * 8u + kFlatStageBytes - 1u) / kFlatStageBytes;
}
__host__ __device__ inline FlatLayout flat_layout_mma(uint32_t ncols, uint32_t rpc, uint32_t nparts, uint32_t nst) {
  FlatLayout l;
  const uint32_t ng = ncols / 128u, nb = flat_mma_b_stages(ncols);
  l.x = (nst >= nb ? nst - nb : 0u) * kFlatStageBytes;  // B staging, over the last nb stages
  l.xs = nst * kFlatStageBytes;                // per group: 1 / exponent scale, x sum
  l.wacc = l.xs + ng * 8u;                     // row sums [part][row]
  l.bp = l.wacc + nparts * rpc * 4u;           // [slot][warp][16 rows]
  l.bc = l.bp + kMmaSlots * kFlatConsumerWarps * kMmaRows * 4u;
  l.bars = (l.bc + kMmaSlots * 4u + 15u) & ~15u;
  l.ranges = l.bars + 2 * kFlatMaxStages * 8;
  l.total = l.ranges + kFlatMaxRanges * (uint32_t)sizeof(FlatRange);
  return l;
}

// Shared-memory layout, shared by host (size) and kernel (offsets).  xsm =
// false (column owners: x lives in registers) leaves out x and its chunk sums.
__host__ __device__ inline FlatLayout flat_layout(uint32_t ncols, uint32_t cw, uint32_t rpc, uint32_t nparts,
                                                  uint32_t nst, uint32_t nw = kFlatConsumerWarps,
                                                  bool xsm = true) {
  FlatLayout l;
  const uint32_t nchunks = ncols / cw, slots = xsm ? (nchunks + 31) / 32 : 0u;
  l.x = nst * kFlatStageBytes;
  l.xs = l.x + slots * 32 * cw * 4;
  l.wacc = l.xs + slots * 32 * 4;
  l.bars = (l.wacc + nparts * nw * rpc * 4 + 15) & ~15u;
  l.ranges = l.bars + 2 * kFlatMaxStages * 8;
  l.total = l.ranges + kFlatMaxRanges * (uint32_t)sizeof(FlatRange);
  return l;
}

// Weights per piece: a flat cell, or 16 KiB of a raw stream.
template <int FMT, int KIND>
__host__ __device__ constexpr uint32_t flat_wpp() {
  return KIND == SRC_FLAT ? 32768u : 16384u * 8u / (uint32_t)FmtInfo<FMT>::BITS;
}

// Bounded wait that also gives up once another warp has flagged an error.
CHPE_DEV bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* bad) {
  for (uint32_t i = 0; i < kMaxWaitPolls; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *bad) return false;
  }
  return false;
}
CHPE_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
template <uint32_t NCT>
CHPE_DEV void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

// ALIGNED: flat cells whose rows start at cell boundaries (cols divides
// 32768, as the 72B/9B hidden widths do).  Then every piece is a whole cell of
// rc rows and consumer lane t always decodes the same column chunk t % (cols /
// CW) of rows t / (cols / CW) + k * (256 / (cols / CW)): its x stays in
// registers for the whole launch and shared memory carries only codes.
// ROWBLK: the tensor-core kernel of gemv_rowblk.cuh (same launch record).
// COLOWN8: column owners with eight slots per lane, for FP16 / BF16 rows of
// 1441..3840 chunks (the 72B FP16 down projection, 3696).
enum FlatMode : int { FLAT_STREAM = 0, FLAT_ALIGNED = 1, FLAT_COLOWN = 2, FLAT_MMA = 3, FLAT_ROWBLK = 4, FLAT_COLOWN8 = 5 };

// MMA (aligned 4-bit group-scaled cells of 4096 or 8192 columns, every
// segment a whole number of 16-row blocks): the products go through
// mma.sync.m16n8k32 with the code bytes as the u8 A operand.  A byte
// lo + 16 hi holds the codes of columns 2p and 2p + 1, so
//   lo x0 + hi x1 = lo y + (16 hi) z,   y = x0, z = x1 / 16 (exact),
// and the two MMAs of a k-step take A = the code words & 0x0F0F0F0F and
// & 0xF0F0F0F0 (two LOP3 per 8 weights, the whole decode).  B holds y and z of
// each 128-column group as int8 pieces: scaled by a power of two S_G so that
// the group's largest |y|, |z| lands in [32, 64), then split into 4 pieces
// of 7 bits (value = i0 + i1/128 + i2/128^2 + i3/128^3, columns n = 0..3 of
// B), which keeps about 27 bits of the group's range.  The s32 accumulation
// is exact (|D| < 2^21 by construction), converted with a magic-number add.
// Per group and row: scale * (sum_n D_n 128^-n / S_G - 8 sum x) = scale *
// sum (c - 8) x.  A non-finite x makes 1 / S_G NaN, so the group's rows are
// NaN as the f32 dot product would be.
//
// A block is 16 consecutive rows (16 / rows-per-cell cells); warp w takes the
// 128-column groups w, w + 16, ... (at most four: 8192 columns), their B
// fragments in registers; lane (g, t) (g = lane / 4, t = lane % 4)
// loads 16-byte chunk t of the group for MMA rows g and g + 8, whose four
// words are the A registers of the group's two k-steps.  MMA row m is row
// (m % 8) / 2 (+ 4 for m >= 8 with 8-row cells) of cell m % 2 (+ 2 for m >= 8
// with 4-row cells) of the block: the rows of one quarter-warp (g = 2k, 2k+1)
// then lie in consecutive ring stages, whose offsets differ by 64 modulo 128
// bytes, so their 16-byte loads hit distinct banks (rows of one cell are a
// multiple of 128 bytes apart).  The 16 warps' partial row
// sums of a block meet in a shared slot; the warp that arrives last adds them
// in warp order, so results do not depend on timing.

// COLOWN ("column owner", rows of 384..960 chunks, no fused norm): consumer
// slot u = lane + 480*j (15 consumer warps) owns column chunk u of every row, with that chunk of x
// in registers for the whole launch (read once from global memory, so shared
// memory holds only the ring), and the CTA walks its rows four at a time
// through the ring.  For the 72B and 9B down projections (29568 and 12288
// columns), whose rows do not start at cell boundaries.
template <int FMT, int KIND, int MODE = FLAT_STREAM, int NWT = 16>
__global__ void __launch_bounds__(NWT * 32 + 32, NWT == 8 ? 2 : 1)
    gemv_flat_tma_kernel(const __grid_constant__ FlatTmaLaunch P) {
  constexpr bool ALIGNED = MODE == FLAT_ALIGNED;
  using FI = FmtInfo<FMT>;
  constexpr uint32_t CW = FI::CW, QPC = CW / 4;
  constexpr uint32_t WPP = flat_wpp<FMT, KIND>();
  constexpr uint32_t NCH = WPP / CW;        // chunks in a full piece
  constexpr uint32_t NW = NWT, NCT = NWT * 32;
  constexpr bool COLW = MODE == FLAT_COLOWN || MODE == FLAT_COLOWN8;  // column owners
  static_assert(MODE != FLAT_COLOWN8 || FI::CW <= 8, "eight slots: chunks of 8 weights");
  static_assert(COLW ? NWT == (int)kFlatColownWarps : (NWT == 16 || (NWT == 8 && MODE == FLAT_ALIGNED)),
                "consumer warps: 16; 8 for aligned cells at two CTAs per SM; 15 for column owners");
  static_assert(MODE != FLAT_MMA || (FMT == FMT_W4G && KIND == SRC_FLAT && NWT == (int)kFlatConsumerWarps),
                "MMA mode: 4-bit group-scaled flat cells, 16 consumer warps");
  constexpr uint32_t CPWARP = NCH / NW;     // chunks per consumer warp
  constexpr uint32_t CPL = CPWARP / 32;     // chunks per lane
  static_assert(COLW || (CPL >= 1 && CPWARP % 32 == 0), "piece geometry");
  constexpr bool MMA = MODE == FLAT_MMA;
  constexpr uint32_t NWR = MMA ? 1u : NW;   // per-row partial slots in wacc
  static_assert(NCH * 16 <= 16384, "a piece fits a stage");

  extern __shared__ __align__(128) uint8_t fsm[];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, L = tid & 31;
  const bool swig = P.epi == EPI_SWIGLU;
  const uint32_t nparts = swig ? 2u : 1u;
  const uint32_t C = P.ncols, nst = P.nst;
  constexpr bool XSM = !COLW && !MMA;  // x staged in shared memory as f32
  const FlatLayout lay = MMA ? flat_layout_mma(C, P.rpc, nparts, nst) : flat_layout(C, CW, P.rpc, nparts, nst, NW, XSM);
  float* xsh = reinterpret_cast<float*>(fsm + lay.x);
  float* xsc = reinterpret_cast<float*>(fsm + lay.xs);
  float* wacc = reinterpret_cast<float*>(fsm + lay.wacc);
  uint64_t* full = reinterpret_cast<uint64_t*>(fsm + lay.bars);
  uint64_t* empty = full + kFlatMaxStages;
  FlatRange* rg = reinterpret_cast<FlatRange*>(fsm + lay.ranges);
  __shared__ float sred[NWT];
  __shared__ unsigned long long kbest[NWT];
  __shared__ uint32_t kfin[NWT];
  __shared__ uint32_t s_npieces, s_nranges;
  __shared__ int s_abort, s_is_last;
  __shared__ volatile int s_bad;

  const uint32_t Rt = P.row_start[swig ? 1 : P.nseg];
  // The CTAs split the rows that have weights in the tiles (each segment's
  // covered leading rows, concatenated: "work rows" [cst(g), cst(g + 1)) are
  // rows row_start[g] + ... of segment g), evenly, in whole cells when
  // aligned, whole 16-row blocks in the MMA mode; rows past the tiles have
  // zero sums and are written by the epilogue of every CTA in turn.
  const uint32_t nsg = swig ? 1u : (uint32_t)P.nseg;
  const uint32_t cs1 = P.cov[0], cs2 = cs1 + (nsg > 1u ? P.cov[1] : 0u), cs3 = cs2 + (nsg > 2u ? P.cov[2] : 0u);
  auto cst = [&](uint32_t g) { return g == 0u ? 0u : g == 1u ? cs1 : g == 2u ? cs2 : cs3; };  // (registers)
  const uint32_t Vt = cst(nsg);
  const uint32_t RU = MMA ? kMmaRows : ALIGNED ? P.rc : 1u, Ut = Vt / RU;
  const uint32_t R0 = RU * (uint32_t)((uint64_t)Ut * blockIdx.x / gridDim.x);  // work rows [R0, R1)
  const uint32_t R1 = RU * (uint32_t)((uint64_t)Ut * (blockIdx.x + 1) / gridDim.x);

  if (tid == 0) {
    // this CTA's flat ranges, gate pieces before up pieces for SwiGLU
    uint32_t n = 0, pieces = 0;
    for (uint32_t p = 0; p < nparts; p++) {
      for (uint32_t g = 0; g < nsg; g++) {
        const uint32_t si = swig ? p : g;
        const uint32_t S0 = swig ? 0u : P.row_start[g];
        const uint32_t va = R0 > cst(g) ? R0 : cst(g), vb = R1 < cst(g + 1) ? R1 : cst(g + 1);
        if (va >= vb) continue;
        const uint32_t a = S0 + (va - cst(g)), b = S0 + (vb - cst(g));  // rows of the call
        FlatRange r;
        r.src = si;
        r.part = p;
        const uint32_t row0 = P.src[si].row0;  // tensor row of the call's row 0
        r.fa0 = (a - S0 + row0) * C;
        r.fb0 = (b - S0 + row0) * C;
        // weights past the tiles the call has read as zero (chpe_engine.zig
        // flat loops stop at the available tiles): no pieces there, and rows
        // with nothing left keep a zero sum
        const uint64_t lim = P.src[si].flat_limit;
        if ((uint64_t)r.fb0 > lim) r.fb0 = (uint32_t)lim;
        if (r.fb0 <= r.fa0) continue;
        r.k0 = r.fa0 / WPP;
        r.pstart = pieces;
        r.lrbase = (int32_t)cst(g) - (int32_t)R0 - (int32_t)row0;  // tensor row + lrbase = work row - R0
        r.pad = 0;
        rg[n++] = r;
        pieces += (r.fb0 - 1) / WPP - r.k0 + 1;
      }
    }
    s_nranges = n;
    s_npieces = pieces;
    s_abort = 0;
    s_bad = 0;
    for (uint32_t i = 0; i < nst; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t npieces = s_npieces, nranges = s_nranges;

  // piece i -> (range, tile k, flat range [fa, fb))
  auto locate = [&](uint32_t i, uint32_t& ri, uint32_t& k, uint32_t& fa, uint32_t& fb) {
    while (ri + 1 < nranges && i >= rg[ri + 1].pstart) ri++;
    const FlatRange& r = rg[ri];
    k = r.k0 + (i - r.pstart);
    fa = k * WPP > r.fa0 ? k * WPP : r.fa0;
    fb = (k + 1) * WPP < r.fb0 ? (k + 1) * WPP : r.fb0;
  };

  // ---- producer warp ------------------------------------------------------
  if (warp == NW) {
    uint32_t ri = 0, issued = 0;
    auto issue = [&](uint32_t i) {
      uint32_t k, fa, fb;
      locate(i, ri, k, fa, fb);
      const GemvSrc& s = P.src[rg[ri].src];
      uint8_t* dst = fsm + (i % nst) * kFlatStageBytes;
      const uint32_t bytes = (fb - fa) * FI::BITS / 8;
      const uint8_t* codes;
      const uint8_t* tile = s.arc + s.tile0 + (uint64_t)k * s.stride;
      if constexpr (KIND == SRC_FLAT) codes = tile + (fa - k * WPP) * FI::BITS / 8;
      else codes = s.arc + s.tile0 + (uint64_t)fa * FI::BITS / 8;
      const uint32_t extra = KIND == SRC_FLAT ? kPayloadHead : 0u;
      mbar_expect_tx(&full[i % nst], bytes + extra);
      bulk_g2s(dst, codes, bytes, &full[i % nst]);
      if constexpr (KIND == SRC_FLAT) bulk_g2s(dst + 16384, tile + 16384, kPayloadHead, &full[i % nst]);
    };
    auto drain = [&]() {  // copies in flight complete before the CTA exits
      const uint32_t from = issued > nst ? issued - nst : 0u;
      for (uint32_t i = from; i < issued; i++) mbar_wait(&full[i % nst], (i / nst) & 1u);
    };
    if (L == 0) {
      // (MMA: the last stages hold the B fragments until the consumers' prologue ends)
      uint32_t nfree = MMA ? nst - flat_mma_b_stages(C) : nst;
      if (P.npre && P.npre < nfree) nfree = P.npre;
      const uint32_t npre = npieces < nfree ? npieces : nfree;
      for (; issued < npre; issued++) issue(issued);
    }
    __syncthreads();  // consumers' prologue done: s_abort is final
    if (L != 0) return;
    if (s_abort) { drain(); return; }
    for (; issued < npieces; issued++) {
      const uint32_t i = issued, s = i % nst;
      if (!mbar_wait_or_abort(&empty[s], ((i / nst) - 1u) & 1u, &s_bad)) {
        atomicExch(&P.st->err, 1);
        s_bad = 1;
        break;
      }
      fence_proxy_async_smem();
      issue(i);
    }
    drain();
    return;
  }

  // ---- consumers: x (optionally RMSNorm'ed) into shared memory --------------
  pdl_wait();
  if (tid == 0) {
    int ab = (!P.ignore_stop && P.st->stop) ? 1 : 0;
    if (!ab && !tp_wait(P.tp)) {  // inputs from the other ranks
      atomicExch(&P.st->err, 1);
      ab = 1;
    }
    s_abort = ab;
  }
  consumer_sync<NCT>();
  const bool stop = s_abort != 0;
  float tot = 0.f;
  const uint32_t nq = C / 4;
  const float4* x4 = reinterpret_cast<const float4*>(P.x);
  // x quad q (columns 4q..4q+3) into shared memory: f32 at xpos, or (MMA)
  // the int8 pieces of y and z into the B fragment staging, with the group's
  // exponent and x sum (the 32 lanes of a warp hold the 32 quads of one
  // 128-column group)
  auto put4 = [&](uint32_t q, const float4& o) {
    if constexpr (MMA) {
      mma_b_put_quad(fsm + lay.x, xsc, q, o, L);
    } else {
      *reinterpret_cast<float4*>(&xsh[xpos<CW>(4 * q)]) = o;
    }
  };
  if (!stop) {
    for (uint32_t i = tid; i < nparts * NWR * P.rpc; i += NCT) wacc[i] = 0.f;
    if constexpr (MMA) {
      for (uint32_t i = tid; i < kMmaSlots; i += NCT) reinterpret_cast<uint32_t*>(fsm + lay.bc)[i] = 0u;
    }
    if (COLW) {
      // column owners load their x chunks into registers in the main loop;
      // with the fused RMSNorm the sum of squares of x comes first (every
      // chunk of the row is one lane's slot)
      if (P.norm) {
        float ss = 0.f;
        for (uint32_t q = tid; q < nq; q += NCT) {
          const float4 v = x4[q];
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        ss = warp_sum(ss);
        if (L == 0) sred[warp] = ss;
        consumer_sync<NCT>();
        for (uint32_t w = 0; w < NW; w++) tot += sred[w];
        if (P.check_layer >= 0) {
          // end-of-layer check of the reference's debug block (chpe_engine.zig:1753-1764)
          const int l = P.check_layer;
          const bool cond = l < 3 || (l >= 8 && l <= 16) || !isfinite(P.x[0]);
          if (cond && !isfinite(tot)) {
            if (blockIdx.x == 0 && tid == 0) P.st->stop = 1;
            if (tid == 0) s_abort = 1;
          }
        }
      }
    } else if (!P.norm) {
      // all loads of a batch in flight before any is stored
      for (uint32_t q0 = 0; q0 < nq; q0 += NCT * 8u) {
        float4 v[8];
#pragma unroll
        for (uint32_t u = 0; u < 8; u++) {
          const uint32_t q = q0 + tid + NCT * u;
          if (q < nq) v[u] = x4[q];
        }
#pragma unroll
        for (uint32_t u = 0; u < 8; u++) {
          const uint32_t q = q0 + tid + NCT * u;
          if (q < nq) put4(q, v[u]);
        }
      }
    } else {
      // RMSNorm: x and gamma in one batch (the host sends cols <= 16384 here,
      // <= 8192 to the 8-warp variant)
      constexpr uint32_t XB = ((NWT == 8 ? 8192u : 16384u) / 4u + NCT - 1u) / NCT;
      const float4* g4 = reinterpret_cast<const float4*>(P.gamma);
      float4 v[XB], g[XB];
      float ss = 0.f;
#pragma unroll
      for (uint32_t u = 0; u < XB; u++) {
        const uint32_t q = tid + NCT * u;
        if (q < nq) { v[u] = x4[q]; g[u] = g4[q]; }
      }
#pragma unroll
      for (uint32_t u = 0; u < XB; u++)
        if (tid + NCT * u < nq) ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
      ss = warp_sum(ss);
      if (L == 0) sred[warp] = ss;
      consumer_sync<NCT>();
      for (uint32_t w = 0; w < NW; w++) tot += sred[w];
      if (P.check_layer >= 0) {
        // end-of-layer check of the reference's debug block (chpe_engine.zig:1753-1764)
        const int l = P.check_layer;
        const bool cond = l < 3 || (l >= 8 && l <= 16) || !isfinite(P.x[0]);
        if (cond && !isfinite(tot)) {
          if (blockIdx.x == 0 && tid == 0) P.st->stop = 1;
          if (tid == 0) s_abort = 1;
        }
      }
      const float inv = 1.0f / sqrtf(tot / (float)C + P.eps);
#pragma unroll
      for (uint32_t u = 0; u < XB; u++) {
        const uint32_t q = tid + NCT * u;
        if (q < nq) {
          float4 o;
          o.x = v[u].x * inv * g[u].x;
          o.y = v[u].y * inv * g[u].y;
          o.z = v[u].z * inv * g[u].z;
          o.w = v[u].w * inv * g[u].w;
          put4(q, o);
          if (P.xn_out && blockIdx.x == 0) reinterpret_cast<float4*>(P.xn_out)[q] = o;
        }
      }
    }
  }
  // MMA: each warp's B fragments (its 128-column groups warp + 16 j, lanes
  // g < 4 hold piece g) into registers, before the producer may reuse the
  // stages they were staged in
  uint2 breg[4][4];
  if constexpr (MMA) {
    consumer_sync<NCT>();
    const uint32_t g = L >> 2, t = L & 3u;
    const uint2* bfr = reinterpret_cast<const uint2*>(fsm + lay.x) + t * kMmaPieces + (g < kMmaPieces ? g : 0u);
#pragma unroll
    for (uint32_t j = 0; j < 4; j++) {
      const uint32_t G = warp + NW * j;
#pragma unroll
      for (uint32_t q = 0; q < 4; q++)
        breg[j][q] = (!stop && g < kMmaPieces && G < (C >> 7)) ? bfr[G * (4u * 4u * kMmaPieces) + q * 4u * kMmaPieces]
                                                               : make_uint2(0u, 0u);
    }
  }
  __syncthreads();  // with the producer: abort decision is final
  if (s_abort) {
    if (tid == 0) tp_signal(P.tp, P.tp.signal_sig);  // every CTA arrives once per launch
    return;
  }
  for (uint32_t cc = tid; XSM && cc < C / CW; cc += NCT) {
    float s = 0.f;
#pragma unroll
    for (uint32_t q = 0; q < QPC; q++) {
      const float4 t = xquad<CW>(xsh, cc >> 5, q, cc & 31u);
      s += (t.x + t.y) + (t.z + t.w);
    }
    xsc[cc] = s;
  }
  consumer_sync<NCT>();
  pdl_launch_dependents();

  // ---- main loop, aligned cells ---------------------------------------------
  if constexpr (ALIGNED) {
    const uint32_t NCPR = C / CW;         // column chunks per row (a multiple of 32, <= NCT)
    const uint32_t RG = NCT / NCPR;       // lane groups over the rows of a cell
    const uint32_t cc = tid % NCPR, rgp = tid / NCPR;
    const uint32_t RC = P.rc;             // rows per cell
    constexpr uint32_t CPI = CPL >= 4 ? 1u : 2u;  // cells per iteration
    constexpr uint32_t NV = CPI * CPL;    // values per lane per iteration
    constexpr uint32_t SPAN = 32u / NV;   // lanes per reduced row after the butterfly
    static_assert(NV == 2 || NV == 4, "one or two cells of 1, 2 or 4 chunks per lane");
    f2x xr[CW / 2];
#pragma unroll
    for (uint32_t q = 0; q < QPC; q++) {
      const float4 t = xquad<CW>(xsh, cc >> 5, q, cc & 31u);
      xr[2 * q] = pack2(t.x, t.y);
      xr[2 * q + 1] = pack2(t.z, t.w);
    }
    const float xsm = xsc[cc];
    // this lane's chunks of a cell and their group-scale offsets are fixed
    const uint32_t ci0 = rgp * NCPR + cc, cstep = RG * NCPR;
    uint32_t soff[CPL], coff[CPL];
#pragma unroll
    for (uint32_t kk = 0; kk < CPL; kk++) {
      coff[kk] = 16u * (ci0 + kk * cstep);                                 // code bytes in a stage
      soff[kk] = 16384u + 48u + 2u * (((ci0 + kk * cstep) * CW) >> 7);    // its group scale
    }
    // current range in registers; advanced when the piece index reaches the next one
    uint32_t ri = 0, r_k0 = rg[0].k0, r_ps = rg[0].pstart, r_part = rg[0].part;
    int32_t r_lrb = rg[0].lrbase;
    uint32_t r_end = nranges > 1 ? rg[1].pstart : npieces;
    auto cell_of = [&](uint32_t i, uint32_t& k, uint32_t& part, int32_t& lrb) {
      if (i == r_end) {
        ri++;
        r_k0 = rg[ri].k0;
        r_ps = rg[ri].pstart;
        r_part = rg[ri].part;
        r_lrb = rg[ri].lrbase;
        r_end = ri + 1 < nranges ? rg[ri + 1].pstart : npieces;
      }
      k = r_k0 + (i - r_ps);
      part = r_part;
      lrb = r_lrb;
    };
    uint32_t ss = 0, sph = 0;  // ring slot and phase of piece i
    for (uint32_t i = 0; i < npieces; i += CPI) {
      const bool two = CPI == 2 && i + 1 < npieces;
      const uint32_t sa = ss, sb = ss + 1 < nst ? ss + 1 : 0u, phb = ss + 1 < nst ? sph : sph ^ 1u;
      bool ok = mbar_wait_or_abort(&full[sa], sph, &s_bad);
      if (ok && two) ok = mbar_wait_or_abort(&full[sb], phb, &s_bad);
      ss += CPI;
      if (ss >= nst) {
        ss -= nst;
        sph ^= 1u;
      }
      if (!ok) {
        if (L == 0) { atomicExch(&P.st->err, 1); s_bad = 1; }
        break;
      }
      uint32_t ka, pa, kb = 0, pb = 0;
      int32_t la, lb = 0;
      cell_of(i, ka, pa, la);
      if (two) cell_of(i + 1, kb, pb, lb);
      // an odd last cell is decoded twice (the second copy's sums are dropped):
      // no branches around the loads
      const uint8_t* stg[2] = {fsm + sa * kFlatStageBytes, fsm + (two ? sb : sa) * kFlatStageBytes};
      uint4 vv[NV];
      float sc[NV];
#pragma unroll
      for (uint32_t u = 0; u < NV; u++) {
        const uint32_t c = u / CPL, kk = u % CPL;
        vv[u] = *reinterpret_cast<const uint4*>(stg[c] + coff[kk]);
        if constexpr (FI::GROUPED) sc[u] = ld_f16(stg[c] + soff[kk]);
        else if constexpr (FI::SB) sc[u] = ld_f32(stg[c] + 16384 + 32);
      }
      float v[NV];
#pragma unroll
      for (uint32_t u = 0; u < NV; u++) {
        f2x acc4[4] = {0ull, 0ull, 0ull, 0ull};  // four independent FMA chains per chunk
#pragma unroll
        for (uint32_t q = 0; q < QPC; q++) quad_fma<FMT>(vv[u], (int)q, xr[2 * q], xr[2 * q + 1], acc4[q & 3]);
        if constexpr (QPC > 2) {
          asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc4[0]) : "l"(acc4[2]));
          asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc4[1]) : "l"(acc4[3]));
        }
        const float d = chunk_finish<FMT>(acc4[0], acc4[1], xsm);
        if constexpr (FI::GROUPED) {
          v[u] = d * sc[u];
        } else if constexpr (FI::SB) {
          v[u] = fmaf(ld_f32(stg[u / CPL] + 16384 + 36), xsm, d * sc[u]);
        } else {
          v[u] = d;
        }
      }
      // NV row sums over the warp in one butterfly: afterwards lane u*SPAN
      // holds the sum of value u (cell u / CPL, row rgp + (u % CPL) * RG)
      float bsum;
      if constexpr (NV == 4) {
        const bool h16 = (L & 16u) != 0, h8 = (L & 8u) != 0;
        const float a0 = (h16 ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, h16 ? v[0] : v[2], 16);
        const float a1 = (h16 ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, h16 ? v[1] : v[3], 16);
        bsum = (h8 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, h8 ? a0 : a1, 8);
      } else {
        const bool h16 = (L & 16u) != 0;
        bsum = (h16 ? v[1] : v[0]) + __shfl_xor_sync(0xffffffffu, h16 ? v[0] : v[1], 16);
        bsum += __shfl_xor_sync(0xffffffffu, bsum, 8);
      }
      bsum += __shfl_xor_sync(0xffffffffu, bsum, 4);
      bsum += __shfl_xor_sync(0xffffffffu, bsum, 2);
      bsum += __shfl_xor_sync(0xffffffffu, bsum, 1);
      if ((L & (SPAN - 1u)) == 0u) {
        const uint32_t u = L / SPAN, c = u / CPL, kk = u % CPL;
        if (c == 0 || two) {
          const uint32_t row = (c ? kb : ka) * RC + rgp + kk * RG;  // tensor row
          // each (warp, row) is written once per launch: a plain store
          wacc[((c ? pb : pa) * NW + warp) * P.rpc + (uint32_t)((int32_t)row + (c ? lb : la))] = bsum;
        }
      }
      __syncwarp();
      if (L == 0) {
        mbar_arrive(&empty[sa]);
        if (two) mbar_arrive(&empty[sb]);
      }
    }
  } else if constexpr (MMA) {
    // ---- main loop, 16-row blocks on the tensor cores -------------------------
    const uint32_t RC = P.rc;                  // rows per cell (4 or 8)
    const uint32_t CPB = kMmaRows / RC;        // cells per block
    const uint32_t NG = C >> 7;                // 128-column groups
    const uint32_t g = L >> 2, t = L & 3u;
    const uint32_t rowB = C >> 1;              // code bytes per row
    // MMA rows g and g + 8 -> (cell of the block, row in the cell)
    const uint32_t c1 = g & 1u, r1 = g >> 1;
    const uint32_t c2 = CPB == 4u ? 2u + (g & 1u) : (g & 1u), r2 = CPB == 4u ? (g >> 1) : 4u + (g >> 1);
    const uint32_t off1 = r1 * rowB + t * 16u, off2 = r2 * rowB + t * 16u;
    const uint32_t soff1 = 16384u + 48u + 2u * r1 * NG, soff2 = 16384u + 48u + 2u * r2 * NG;
    // pieces 2t and 2t+1 sit in this lane's two D columns
    const float pw0 = t == 0u ? 1.0f : t == 1u ? 6.103515625e-05f : 0.0f;          // 128^-(2t)
    const float pw1 = t == 0u ? 7.8125e-03f : t == 1u ? 4.76837158203125e-07f : 0.0f;  // 128^-(2t+1)
    const float corr = t == 0u ? 8.0f : 0.0f;  // the x-sum term, once per row (lane t = 0)
    float* bpart = reinterpret_cast<float*>(fsm + lay.bp);
    uint32_t* bcnt = reinterpret_cast<uint32_t*>(fsm + lay.bc);
    uint32_t ri = 0, r_k0 = rg[0].k0, r_ps = rg[0].pstart, r_part = rg[0].part;
    int32_t r_lrb = rg[0].lrbase;
    uint32_t r_end = nranges > 1 ? rg[1].pstart : npieces;
    const uint32_t nblk = npieces / CPB;       // the host sends whole blocks
    uint32_t sb = 0, phb = 0;                  // ring slot and phase of the block's first piece
    // slot of the block's piece c (CPB <= nst)
    auto slot_of = [&](uint32_t c) { return sb + c < nst ? sb + c : sb + c - nst; };
    for (uint32_t blk = 0; blk < nblk; blk++) {
      const uint32_t i0 = blk * CPB;
      bool ok = true;
      for (uint32_t c = 0; c < CPB && ok; c++)
        ok = mbar_wait_or_abort(&full[slot_of(c)], sb + c < nst ? phb : phb ^ 1u, &s_bad);
      if (!ok) {
        if (L == 0) { atomicExch(&P.st->err, 1); s_bad = 1; }
        break;
      }
      if (i0 == r_end) {  // blocks never straddle ranges (whole blocks per segment)
        ri++;
        r_k0 = rg[ri].k0;
        r_ps = rg[ri].pstart;
        r_part = rg[ri].part;
        r_lrb = rg[ri].lrbase;
        r_end = ri + 1 < nranges ? rg[ri + 1].pstart : npieces;
      }
      const uint8_t* st1 = fsm + slot_of(c1) * kFlatStageBytes;
      const uint8_t* st2 = fsm + slot_of(c2) * kFlatStageBytes;
      float acc1 = 0.f, acc2 = 0.f;
#pragma unroll
      for (uint32_t j = 0; j < 4; j++) {
        const uint32_t G = warp + NW * j;
        if (G >= NG) break;
        const uint4 w1 = *reinterpret_cast<const uint4*>(st1 + off1 + G * 64u);
        const uint4 w2 = *reinterpret_cast<const uint4*>(st2 + off2 + G * 64u);
        const float s1 = ld_f16(st1 + soff1 + 2u * G), s2 = ld_f16(st2 + soff2 + 2u * G);
        int d[4] = {0, 0, 0, 0};
#pragma unroll
        for (uint32_t ks = 0; ks < 2; ks++) {
          const uint32_t a0 = word_of(w1, (int)(2 * ks)), a1 = word_of(w2, (int)(2 * ks));
          const uint32_t a2 = word_of(w1, (int)(2 * ks + 1)), a3 = word_of(w2, (int)(2 * ks + 1));
          const uint2 By = breg[j][2 * ks], Bz = breg[j][2 * ks + 1];
          mma_u8s8_16832(d, a0 & 0x0F0F0F0Fu, a1 & 0x0F0F0F0Fu, a2 & 0x0F0F0F0Fu, a3 & 0x0F0F0F0Fu, By.x, By.y);
          mma_u8s8_16832(d, a0 & 0xF0F0F0F0u, a1 & 0xF0F0F0F0u, a2 & 0xF0F0F0F0u, a3 & 0xF0F0F0F0u, Bz.x, Bz.y);
        }
        const float invS = xsc[2 * G], xc = corr * xsc[2 * G + 1];
        const float v1 = fmaf(s32_exact(d[1]), pw1, s32_exact(d[0]) * pw0);
        const float v2 = fmaf(s32_exact(d[3]), pw1, s32_exact(d[2]) * pw0);
        acc1 = fmaf(s1, fmaf(v1, invS, -xc), acc1);
        acc2 = fmaf(s2, fmaf(v2, invS, -xc), acc2);
      }
      // lanes t = 0 and 1 hold the pieces n = 0,1 and n = 2,3; t = 2, 3 hold zeros
      acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
      acc2 += __shfl_xor_sync(0xffffffffu, acc2, 1);
      const uint32_t slot = blk % kMmaSlots;
      float* bp = bpart + slot * (NW * kMmaRows);
      if (t == 0u) {
        bp[warp * kMmaRows + g] = acc1;
        bp[warp * kMmaRows + g + 8u] = acc2;
      }
      __threadfence_block();
      __syncwarp();
      uint32_t last = 0;
      if (L == 0) last = atomicAdd(&bcnt[slot], 1u) == NW - 1u ? 1u : 0u;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        // every warp's partials of this block are in: add them in warp order
        __threadfence_block();
        if (L < kMmaRows) {
          float sum = 0.f;
#pragma unroll
          for (uint32_t w = 0; w < NW; w++) sum += bp[w * kMmaRows + L];
          const uint32_t k0 = r_k0 + (i0 - r_ps);  // first cell of the block
          const uint32_t mc = L < 8u ? (L & 1u) : (CPB == 4u ? 2u + (L & 1u) : (L & 1u));
          const uint32_t mr = L < 8u ? ((L & 7u) >> 1) : (CPB == 4u ? ((L & 7u) >> 1) : 4u + ((L & 7u) >> 1));
          wacc[r_part * P.rpc + (uint32_t)((int32_t)((k0 + mc) * RC + mr) + r_lrb)] = sum;
        }
        if (L == 0) bcnt[slot] = 0u;
        __syncwarp();
      }
      if (L == 0)
        for (uint32_t c = 0; c < CPB; c++) mbar_arrive(&empty[slot_of(c)]);
      sb += CPB;
      if (sb >= nst) {
        sb -= nst;
        phb ^= 1u;
      }
    }
  } else if constexpr (COLW) {
    // ---- main loop, column owners ------------------------------------------
    // One row per group (the host sends rows of 384..960 chunks for 16-byte
    // chunks of 32 weights, 384..480 for 64): every active slot of a lane lies
    // in the row, and four consecutive rows per iteration share one 4-value
    // butterfly.
    const uint32_t NCC = C / CW;                         // chunks per row
    constexpr uint32_t SL = MODE == FLAT_COLOWN8 ? 8u : CW <= 8 ? 3u : CW <= 32 ? 2u : 1u;  // slots per lane
    // rows per iteration: the ring must hold every piece of them at once
    // (two rows of up to 30720 FP16 weights: at most 9 pieces)
    constexpr uint32_t RI = MODE == FLAT_COLOWN8 ? 2u : 4u;
    f2x xr[SL][CW / 2];
    float xsj[SL];
    uint32_t scw[SL];                                     // first column of the slot
    bool act[SL];
    const float inv = P.norm ? 1.0f / sqrtf(tot / (float)C + P.eps) : 1.0f;
#pragma unroll
    for (uint32_t j = 0; j < SL; j++) {
      const uint32_t u = tid + NCT * j;
      act[j] = u < NCC;
      scw[j] = (act[j] ? u : 0u) * CW;
      const float4* xp = reinterpret_cast<const float4*>(P.x + scw[j]);
      float4 t4[QPC];
#pragma unroll
      for (uint32_t q = 0; q < QPC; q++) t4[q] = act[j] ? xp[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (P.norm) {  // x * inv * gamma, as the staged path normalises it
        const float4* gp = reinterpret_cast<const float4*>(P.gamma + scw[j]);
#pragma unroll
        for (uint32_t q = 0; q < QPC; q++) {
          const float4 gm = act[j] ? gp[q] : make_float4(0.f, 0.f, 0.f, 0.f);
          t4[q].x = t4[q].x * inv * gm.x;
          t4[q].y = t4[q].y * inv * gm.y;
          t4[q].z = t4[q].z * inv * gm.z;
          t4[q].w = t4[q].w * inv * gm.w;
          if (P.xn_out && blockIdx.x == 0 && act[j]) reinterpret_cast<float4*>(P.xn_out + scw[j])[q] = t4[q];
        }
      }
      float sx = 0.f;
#pragma unroll
      for (uint32_t q = 0; q < QPC; q++) {
        xr[j][2 * q] = pack2(t4[q].x, t4[q].y);
        xr[j][2 * q + 1] = pack2(t4[q].z, t4[q].w);
        sx += (t4[q].x + t4[q].y) + (t4[q].z + t4[q].w);
      }
      xsj[j] = sx;
    }
    // pieces waited for / released so far, with the ring slot (and phase) of the next one
    uint32_t waited = 0, released = 0, wslot = 0, wph = 0, rslot = 0;
    bool bad = false;
    for (uint32_t r = 0; r < nranges && !bad; r++) {
      const FlatRange rgv = rg[r];
      const uint32_t pend = r + 1 < nranges ? rg[r + 1].pstart : npieces;
      const uint32_t pbase = rgv.pstart - rgv.k0;        // piece of tile k: pbase + k
      const uint32_t ra = rgv.fa0 / C, rb = (rgv.fb0 + C - 1) / C;
      for (uint32_t g0 = ra; g0 < rb; g0 += RI) {
        const uint32_t g1 = g0 + RI < rb ? g0 + RI : rb;
        const uint32_t flo = g0 * C > rgv.fa0 ? g0 * C : rgv.fa0;
        const uint32_t fhi = g1 * C < rgv.fb0 ? g1 * C : rgv.fb0;
        const uint32_t p_lo = pbase + flo / WPP, p_hi = pbase + (fhi - 1u) / WPP;
        for (; waited <= p_hi; waited++) {
          if (!mbar_wait_or_abort(&full[wslot], wph, &s_bad)) { bad = true; break; }
          if (++wslot == nst) {
            wslot = 0;
            wph ^= 1u;
          }
        }
        if (bad) break;
        // every piece before this group's first one has been released
        const uint32_t s_lo = rslot;                     // ring slot of piece p_lo (== released)
        float vrow[RI];
#pragma unroll
        for (uint32_t rr = 0; rr < RI; rr++) vrow[rr] = 0.f;
#pragma unroll
        for (uint32_t j = 0; j < SL; j++) {
          if (warp * 32u + NCT * j >= NCC) continue;  // no active slot j in this warp
          // the slot's chunk of RI rows: every load issued before the decode;
          // a chunk outside the group reads the first piece's bytes and adds 0
          uint4 cv[RI];
          float sc[RI], bi[RI];
          bool ok[RI];
          uint32_t f = g0 * C + scw[j];
#pragma unroll
          for (uint32_t rr = 0; rr < RI; rr++, f += C) {
            ok[rr] = act[j] && g0 + rr < g1 && f >= rgv.fa0 && f < rgv.fb0;
            const uint32_t k = f / WPP, t0 = k * WPP;
            uint32_t sidx = s_lo + (pbase + k - p_lo);
            if (sidx >= nst) sidx -= nst;
            const uint32_t fa_p = t0 > rgv.fa0 ? t0 : rgv.fa0;  // first weight of the piece
            const uint8_t* stg = fsm + (ok[rr] ? sidx : s_lo) * kFlatStageBytes;
            cv[rr] = *reinterpret_cast<const uint4*>(stg + (ok[rr] ? (f - fa_p) * FI::BITS / 8 : 0u));
            if constexpr (FI::GROUPED) sc[rr] = ld_f16(stg + 16384 + 48 + (ok[rr] ? 2 * ((f - t0) >> 7) : 0u));
            else if constexpr (FI::SB) { sc[rr] = ld_f32(stg + 16384 + 32); bi[rr] = ld_f32(stg + 16384 + 36); }
          }
#pragma unroll
          for (uint32_t rr = 0; rr < RI; rr++) {
            f2x acc4[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
            for (uint32_t q = 0; q < QPC; q++) quad_fma<FMT>(cv[rr], (int)q, xr[j][2 * q], xr[j][2 * q + 1], acc4[q & 3]);
            if constexpr (QPC > 2) {
              asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc4[0]) : "l"(acc4[2]));
              asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc4[1]) : "l"(acc4[3]));
            }
            const float d = chunk_finish<FMT>(acc4[0], acc4[1], xsj[j]);
            float t;
            if constexpr (FI::GROUPED) t = d * sc[rr];
            else if constexpr (FI::SB) t = fmaf(bi[rr], xsj[j], d * sc[rr]);
            else t = d;
            vrow[rr] += ok[rr] ? t : 0.f;
          }
          (void)bi;
        }
        // the RI row sums in one butterfly: lane (32 / RI) * rr holds row g0 + rr
        const bool h16 = (L & 16u) != 0, h8 = (L & 8u) != 0;
        float bsum;
        if constexpr (RI == 4) {
          const float a0 = (h16 ? vrow[2] : vrow[0]) + __shfl_xor_sync(0xffffffffu, h16 ? vrow[0] : vrow[2], 16);
          const float a1 = (h16 ? vrow[3] : vrow[1]) + __shfl_xor_sync(0xffffffffu, h16 ? vrow[1] : vrow[3], 16);
          bsum = (h8 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, h8 ? a0 : a1, 8);
        } else {
          (void)h8;
          bsum = (h16 ? vrow[1] : vrow[0]) + __shfl_xor_sync(0xffffffffu, h16 ? vrow[0] : vrow[1], 16);
          bsum += __shfl_xor_sync(0xffffffffu, bsum, 8);
        }
        bsum += __shfl_xor_sync(0xffffffffu, bsum, 4);
        bsum += __shfl_xor_sync(0xffffffffu, bsum, 2);
        bsum += __shfl_xor_sync(0xffffffffu, bsum, 1);
        if ((L & (32u / RI - 1u)) == 0u) {
          const uint32_t row = g0 + L / (32u / RI);
          if (row < g1) wacc[(rgv.part * NW + warp) * P.rpc + (uint32_t)((int32_t)row + rgv.lrbase)] += bsum;
        }
        // pieces wholly before the next group's first weight are done
        const uint32_t fnext = g1 * C;
        const uint32_t p_keep = (g1 < rb && fnext < rgv.fb0) ? pbase + fnext / WPP : pend;
        __syncwarp();
        for (; released < p_keep; released++) {
          if (L == 0) mbar_arrive(&empty[rslot]);
          if (++rslot == nst) rslot = 0;
        }
      }
    }
    if (bad && L == 0) { atomicExch(&P.st->err, 1); s_bad = 1; }
  } else {
  // ---- main loop, any flat stream --------------------------------------------
  const uint32_t NCC = C / CW;  // chunks per row
  const float invC = 1.0f / (float)C;
  uint32_t ri = 0;
  const uint32_t c0 = warp * CPWARP;
  bool failed = false;
  for (uint32_t i = 0; i < npieces; i++) {
    const uint32_t s = i % nst;
    if (!mbar_wait_or_abort(&full[s], (i / nst) & 1u, &s_bad)) {
      if (L == 0) { atomicExch(&P.st->err, 1); s_bad = 1; }
      failed = true;
      break;
    }
    uint32_t k, fa, fb;
    locate(i, ri, k, fa, fb);
    const uint32_t nch = (fb - fa) / CW;
    if (c0 < nch) {
      const uint8_t* stg = fsm + s * kFlatStageBytes;
      const uint8_t* pl = stg + 16384;
      const uint32_t fw = fa + c0 * CW;
      // row of the warp's first chunk: a float quotient corrected to exact
      uint32_t rA = (uint32_t)((float)fw * invC);
      if (rA * C > fw) rA--;
      else if ((rA + 1) * C <= fw) rA++;
      const uint32_t ccA = (fw - rA * C) / CW + L;  // chunk-in-row of this lane's j = 0
      const uint32_t gbase = (KIND == SRC_FLAT ? fa - k * WPP : 0u) + (c0 + L) * CW;  // cell offset, j = 0
      float sA = 0.f, sB = 0.f;
      float psc = 1.f, pbi = 0.f;
      if constexpr (FI::SB) { psc = ld_f32(pl + 32); pbi = ld_f32(pl + 36); }
      bool crossed = false;
      uint4 vv[CPL];  // all of this lane's code loads first
#pragma unroll
      for (uint32_t j = 0; j < CPL; j++) {
        const uint32_t ci = c0 + L + 32u * j;
        vv[j] = ci < nch ? *reinterpret_cast<const uint4*>(stg + 16u * ci) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (uint32_t j = 0; j < CPL; j++) {
        const uint32_t ci = c0 + L + 32u * j;
        if (ci < nch) {
          uint32_t cc = ccA + 32u * j;
          const bool second = cc >= NCC;  // the run wraps into row rA + 1
          cc = second ? cc - NCC : cc;
          crossed |= second;
          const uint4 v = vv[j];
          const ulonglong2* xq = reinterpret_cast<const ulonglong2*>(xsh) + ((cc >> 5) * QPC * 32u + (cc & 31u));
          f2x a0 = 0ull, a1 = 0ull;
#pragma unroll
          for (uint32_t q = 0; q < QPC; q++) {
            const ulonglong2 xv = xq[32u * q];
            quad_fma<FMT>(v, (int)q, xv.x, xv.y, (q & 1) ? a1 : a0);
          }
          const float xsm = xsc[cc];
          const float d = chunk_finish<FMT>(a0, a1, xsm);
          float t;
          if constexpr (FI::GROUPED) t = d * ld_f16(pl + 48 + 2 * ((gbase + 32u * CW * j) >> 7));
          else if constexpr (FI::SB) t = fmaf(pbi, xsm, d * psc);
          else t = d;
          if (second) sB += t; else sA += t;
        }
      }
      // both sums in one butterfly: lanes 0-15 reduce sA, lanes 16-31 sB
      const bool hi = (L & 16u) != 0;
      float keep = hi ? sB : sA;
      keep += __shfl_xor_sync(0xffffffffu, hi ? sA : sB, 16);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
      const bool any2 = __any_sync(0xffffffffu, crossed);
      if (L == 0 || (L == 16 && any2)) {
        const FlatRange& r = rg[ri];
        wacc[(r.part * NW + warp) * P.rpc + (uint32_t)((int32_t)rA + r.lrbase) + (L >> 4)] += keep;
      }
    }
    __syncwarp();
    if (L == 0) mbar_arrive(&empty[s]);
  }
  (void)failed;
  }  // any flat stream
  consumer_sync<NCT>();
  if (s_bad) {
    if (tid == 0) tp_signal(P.tp, P.tp.signal_sig);
    return;
  }

  // ---- epilogue: rows of this CTA -----------------------------------------
  unsigned long long lbest = 0ull;
  uint32_t lfin = 1u;
  // output row gr (of the call) of segment seg from its sums (SwiGLU: gate d0, up d1)
  auto emit = [&](uint32_t seg, uint32_t gr, float d0, float d1) {
    if constexpr (FMT == FMT_I8RAW) {  // raw int8 dot scale (chpe_engine.zig:1236)
      d0 *= 0.00373708f;
      d1 *= 0.00373708f;
    }
    if (swig) {
      tp_put(P.tp, P.out[0], gr, silu_ref(d0) * d1);
      return;
    }
    const uint32_t r = gr - P.row_start[seg];
    const GemvSrc& s = P.src[seg];
    float* y = P.out[seg];
    if (P.epi == EPI_LOGITS) {
      const uint32_t vr = r + s.row0;  // vocabulary index
      if (P.tp.world > 1 && P.st->gather) tp_put(P.tp, y, r, d0);
      else y[r] = d0;
      if (vr == 0 && P.tp.world > 1)
        for (int rr = 0; rr < P.tp.world; rr++) tp_at(P.tp.sh, P.tp, rr)->token0 = d0;
      if (!isfinite(d0)) lfin = 0u;
      if (d0 > -1e30f) {
        const unsigned long long kk = argmax_key(d0, vr);
        lbest = kk > lbest ? kk : lbest;
      }
    } else if (P.epi == EPI_ACCUM) {
      float v = y[r] + d0;
      if (s.bias) v += s.bias[r];
      tp_put(P.tp, y, r, v);
    } else {
      tp_put(P.tp, y, r, s.bias ? d0 + s.bias[r] : d0);
    }
  };
  const uint32_t nrows = R1 - R0;
  for (uint32_t lr = tid; lr < nrows; lr += NCT) {
    float d0 = 0.f, d1 = 0.f;
#pragma unroll
    for (uint32_t w = 0; w < NWR; w++) d0 += wacc[w * P.rpc + lr];
    if (swig) {
#pragma unroll
      for (uint32_t w = 0; w < NWR; w++) d1 += wacc[(NWR + w) * P.rpc + lr];
    }
    const uint32_t v = R0 + lr;
    uint32_t g = 0;
    while (g + 1 < nsg && v >= cst(g + 1)) g++;
    emit(swig ? 0u : g, (swig ? 0u : P.row_start[g]) + (v - cst(g)), d0, d1);
  }
  if (Vt < Rt) {
    // rows past the tiles: zero sums, every CTA a share
    for (uint32_t u = blockIdx.x * NCT + tid; u < Rt - Vt; u += gridDim.x * NCT) {
      uint32_t g = 0, ub = 0;  // uncovered rows before segment g
      for (;;) {
        const uint32_t S0 = swig ? 0u : P.row_start[g], S1 = swig ? Rt : P.row_start[g + 1];
        const uint32_t un = (S1 - S0) - (cst(g + 1) - cst(g));
        if (u < ub + un || g + 1 >= nsg) break;
        ub += un;
        g++;
      }
      const uint32_t S0 = swig ? 0u : P.row_start[g];
      emit(swig ? 0u : g, S0 + (cst(g + 1) - cst(g)) + (u - ub), 0.f, 0.f);
    }
  }
  if (P.epi == EPI_LOGITS) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long ob = __shfl_xor_sync(0xffffffffu, lbest, o);
      lbest = ob > lbest ? ob : lbest;
    }
    lfin = __all_sync(0xffffffffu, lfin != 0u) ? 1u : 0u;
    if (L == 0) { kbest[warp] = lbest; kfin[warp] = lfin; }
    consumer_sync<NCT>();
    if (tid == 0) {
      unsigned long long b = 0ull;
      uint32_t f = 1u;
      for (uint32_t w = 0; w < NW; w++) { b = kbest[w] > b ? kbest[w] : b; f &= kfin[w]; }
      const int nr = P.tp.world > 1 ? P.tp.world : 1;
      for (int rr = 0; rr < nr; rr++) {  // argmax and finiteness on every rank
        StepState* st = nr > 1 ? tp_at(P.st, P.tp, rr) : P.st;
        if (b) atomicMax_system(&st->best, b);
        if (!f) atomicAnd_system(&st->finite, 0u);
      }
      tp_signal(P.tp, P.tp.signal_sig);
      __threadfence();
      s_is_last = atomicAdd(&P.st->done_ctas, 1u) == gridDim.x - 1;
    }
    consumer_sync<NCT>();
    if (s_is_last && tid == 0) {
      float t0;
      if (P.tp.world > 1) {
        // every rank's LM-head CTAs have reported to this rank
        const unsigned long long e = P.tp.sh->epoch;
        if (!tp_wait_count(P.tp, SIG_LM, (e + 1ull) * P.tp.lm_units)) atomicExch(&P.st->err, 1);
        t0 = *reinterpret_cast<volatile float*>(&P.tp.sh->token0);
        P.tp.sh->epoch = (uint32_t)(e + 1ull);
      } else {
        t0 = __ldcg(P.out[0]);
      }
      finalize_logits(P.st, P.res, t0, tot, P.gen_tokens, P.max_gen);
    }
    return;
  }
  consumer_sync<NCT>();
  if (tid == 0) tp_signal(P.tp, P.tp.signal_sig);
}

}  // namespace chpe
