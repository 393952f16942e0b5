// gemv.cuh -- the weight-streaming GEMV family of the decode loop.
//
// One kernel template covers every gemvLinear call site
// (chpe_engine.zig:1396-1489) whose tensor has a uniform format:
//   * raw FP16 / BF16 / INT8 streams            (dotSegment, :1194-1254)
//   * row-tiled cells W2/W4/W8/F16/F32            (gemvTile*, :223-581)
//   * flat 32768-weight W4/W2 cells               (gemvCellFlat, :584-729)
// A warp owns one output row: its lanes stream 16-byte chunks of codes with
// 128-bit non-allocating loads, decode them in registers and FMA against x
// staged once per CTA in shared memory (lane-permuted so each LDS.128 is
// conflict-free), then reduce across the warp.  Epilogues fuse the bias,
// the residual add and SwiGLU; the prologue fuses RMSNorm.
//
// Decode of a 4/2/8-bit code c into a float uses one PRMT: the code byte is
// placed into bits 16..23 of 0x3F000000, giving f = 0.5 + c/256 exactly; a
// chunk's sum over f*x is mapped back to sum over (c - offset)*x with the
// chunk's x-sum, which costs no extra per-weight work.  Pairs of products use
// the packed FFMA2 of sm_100.
#pragma once
#include "device_common.cuh"

namespace chpe {

enum Epi : int32_t { EPI_STORE = 0, EPI_ACCUM = 1, EPI_SWIGLU = 2, EPI_LOGITS = 3 };
enum Outl : uint32_t { OUTL_NONE = 0, OUTL_ADD = 1, OUTL_REPLACE = 2 };

struct GemvLaunch {
  GemvSrc src[3];
  float* out[3];
  uint32_t row_start[4];  // prefix of output rows over segments
  int32_t nseg;
  int32_t epi;
  const float* x;       // input vector when norm == 0
  const float* gamma;   // RMSNorm gains when norm != 0 (x is then `hidden`)
  float eps;
  uint32_t ncols;       // length of x used (= c_total)
  int32_t norm;
  int32_t check_layer;  // layer whose end-of-layer finiteness check runs here, -1 none
  StepState* st;
  float* xn_out;        // optional copy of the staged x (normed) for later passes
  uint64_t prefetch_bytes[3];  // bytes of each segment's weights to prefetch
  const uint8_t* prefetch_base[3];
  int32_t ignore_stop;  // the LM head always runs (the reference only breaks the layer loop)
  StepResult* res;      // EPI_LOGITS: written by the last CTA
  int32_t* gen_tokens;  // EPI_LOGITS: generated-token log (may be null)
  int32_t max_gen;
};

// Ordered key for "first strict maximum": larger logit wins, then lower index.
CHPE_DEV unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t u = __float_as_uint(v);
  uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
CHPE_DEV float key_value(unsigned long long k) {
  uint32_t o = (uint32_t)(k >> 32);
  uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
  return __uint_as_float(u);
}

template <int FMT> struct FmtInfo;
// CW: columns per 16-byte chunk; CELL_ROWS: rows of a full row-tiled cell
// of 2048 columns (the only row-tiled geometry the fast path takes).
template <> struct FmtInfo<FMT_W4G> { static constexpr int CW = 32, BITS = 4, GROUPED = 1, SB = 0, CELL_ROWS = 16; };
template <> struct FmtInfo<FMT_W4SB> { static constexpr int CW = 32, BITS = 4, GROUPED = 0, SB = 1, CELL_ROWS = 16; };
template <> struct FmtInfo<FMT_W2G> { static constexpr int CW = 64, BITS = 2, GROUPED = 1, SB = 0, CELL_ROWS = 16; };
template <> struct FmtInfo<FMT_W2SB> { static constexpr int CW = 64, BITS = 2, GROUPED = 0, SB = 1, CELL_ROWS = 16; };
template <> struct FmtInfo<FMT_W8> { static constexpr int CW = 16, BITS = 8, GROUPED = 0, SB = 0, CELL_ROWS = 8; };
template <> struct FmtInfo<FMT_F16> { static constexpr int CW = 8, BITS = 16, GROUPED = 0, SB = 0, CELL_ROWS = 4; };
template <> struct FmtInfo<FMT_BF16> { static constexpr int CW = 8, BITS = 16, GROUPED = 0, SB = 0, CELL_ROWS = 4; };
template <> struct FmtInfo<FMT_F32> { static constexpr int CW = 4, BITS = 32, GROUPED = 0, SB = 0, CELL_ROWS = 2; };
template <> struct FmtInfo<FMT_I8RAW> { static constexpr int CW = 16, BITS = 8, GROUPED = 0, SB = 0, CELL_ROWS = 1; };

// Shared-memory position of column c for chunk width CW: lane L of slot j
// reads quad q of its chunk at ((j*CW/4 + q)*32 + L)*4.
template <int CW>
CHPE_DEV uint32_t xpos(uint32_t c) {
  uint32_t chunk = c / CW, L = chunk & 31u, j = chunk >> 5, q = (c % CW) >> 2;
  return ((j * (CW / 4) + q) * 32u + L) * 4u + (c & 3u);
}
template <int CW>
CHPE_DEV float4 xquad(const float* xs, uint32_t j, uint32_t q, uint32_t L) {
  return reinterpret_cast<const float4*>(xs)[(j * (CW / 4) + q) * 32u + L];
}

constexpr uint32_t PRMT_HI = 0x3F000000u;  // bytes 4..7 = 00 00 00 3F

CHPE_DEV uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Packed pairs of floats live in 64-bit registers; every product pair is one
// fma.rn.f32x2.  The decoded weights are produced straight into the halves of
// a 64-bit register, so no moves are needed to form the pairs.
typedef unsigned long long f2x;

CHPE_DEV f2x pack2(float a, float b) {
  f2x r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
CHPE_DEV float2 unpack2(f2x v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
CHPE_DEV void fma2x(f2x& acc, f2x a, f2x x) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(x));
}
// Two codes -> (0.5 + c0/256, 0.5 + c1/256) with one PRMT each, then FMA.
CHPE_DEV void code_pair_fma(f2x& acc, uint32_t wa, uint32_t wb, uint32_t sel, f2x x) {
  asm("{\n\t.reg .b32 a, b;\n\t.reg .b64 p;\n\t"
      "prmt.b32 a, %1, %3, %4;\n\tprmt.b32 b, %2, %3, %4;\n\t"
      "mov.b64 p, {a, b};\n\tfma.rn.f32x2 %0, p, %5, %0;\n\t}"
      : "+l"(acc)
      : "r"(wa), "r"(wb), "r"(PRMT_HI), "r"(sel), "l"(x));
}

// Accumulate the 4 columns of quad q (columns 4q..4q+3 of the chunk) of one
// 16-byte chunk against the x quad (x01, x23).  Code formats accumulate
// f(c)*x with f = 0.5 + code/256 (exact), mapped back per chunk in
// chunk_finish.
template <int FMT>
CHPE_DEV void quad_fma(const uint4& v, int q, f2x x01, f2x x23, f2x& acc) {
  if constexpr (FMT == FMT_W4G || FMT == FMT_W4SB) {
    const uint32_t w = word_of(v, q >> 1);
    const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
    const uint32_t s0 = 0x7044u | ((uint32_t)(2 * (q & 1)) << 8), s1 = s0 + 0x100u;
    code_pair_fma(acc, lo, hi, s0, x01);  // columns 4q, 4q+1
    code_pair_fma(acc, lo, hi, s1, x23);  // columns 4q+2, 4q+3
  } else if constexpr (FMT == FMT_W2G || FMT == FMT_W2SB) {
    // codebook {0,1,-2,-1} = (code ^ 2) - 2
    const uint32_t w = word_of(v, q >> 2) ^ 0xAAAAAAAAu;
    const uint32_t sel = 0x7044u | ((uint32_t)(q & 3) << 8);
    const uint32_t m0 = w & 0x03030303u, m1 = (w >> 2) & 0x03030303u;
    const uint32_t m2 = (w >> 4) & 0x03030303u, m3 = (w >> 6) & 0x03030303u;
    code_pair_fma(acc, m0, m1, sel, x01);
    code_pair_fma(acc, m2, m3, sel, x23);
  } else if constexpr (FMT == FMT_W8 || FMT == FMT_I8RAW) {
    // (b ^ 0x80) in the low byte of 2^23 is 2^23 + b + 128; the subtraction is exact
    const uint32_t w = word_of(v, q) ^ 0x80808080u;
    const f2x off = pack2(-8388736.0f, -8388736.0f);
    f2x a = pack2(__uint_as_float(prmt(w, 0x4B000000u, 0x7440u)), __uint_as_float(prmt(w, 0x4B000000u, 0x7441u)));
    f2x b = pack2(__uint_as_float(prmt(w, 0x4B000000u, 0x7442u)), __uint_as_float(prmt(w, 0x4B000000u, 0x7443u)));
    asm("add.rn.f32x2 %0, %0, %1;" : "+l"(a) : "l"(off));
    asm("add.rn.f32x2 %0, %0, %1;" : "+l"(b) : "l"(off));
    fma2x(acc, a, x01);
    fma2x(acc, b, x23);
  } else if constexpr (FMT == FMT_F16) {
    const uint32_t w0 = word_of(v, 2 * q), w1 = word_of(v, 2 * q + 1);
    float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w0));
    float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w1));
    fma2x(acc, pack2(a.x, a.y), x01);
    fma2x(acc, pack2(b.x, b.y), x23);
  } else if constexpr (FMT == FMT_BF16) {
    const uint32_t w0 = word_of(v, 2 * q), w1 = word_of(v, 2 * q + 1);
    fma2x(acc, pack2(__uint_as_float(w0 << 16), __uint_as_float(w0 & 0xFFFF0000u)), x01);
    fma2x(acc, pack2(__uint_as_float(w1 << 16), __uint_as_float(w1 & 0xFFFF0000u)), x23);
  } else {  // F32: the chunk is one quad
    fma2x(acc, pack2(__uint_as_float(v.x), __uint_as_float(v.y)), x01);
    fma2x(acc, pack2(__uint_as_float(v.z), __uint_as_float(v.w)), x23);
  }
}

// D += A * B on the tensor cores, m16n8k32, u8 A, s8 B, s32 accumulate
// (lane = 4g + t).  A registers (four k bytes each): (row g, k 4t..4t+3),
// (row g+8, k 4t..4t+3), (row g, k 4t+16..4t+19), (row g+8, k 4t+16..4t+19);
// B: (k 4t..4t+3, n g), (k 4t+16..4t+19, n g); D: (g, 2t), (g, 2t+1),
// (g+8, 2t), (g+8, 2t+1).
CHPE_DEV void mma_u8s8_16832(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// B operand of the m16n8k32 integer decode: x quad q (columns 4q..4q+3; the
// 32 lanes of a warp hold the 32 quads of one 128-column group) as int8
// pieces.  A code byte lo + 16 hi holds the codes of columns 2p and 2p + 1,
// and lo x0 + hi x1 = lo y + (16 hi) z with y = x0, z = x1 / 16 (exact); y
// and z of the group are scaled by a power of two S that puts the largest
// |y|, |z| in [32, 64) and split into four 7-bit pieces (value = i0 + i1/128
// + i2/128^2 + i3/128^3, B columns n = 0..3).  Staging layout
// [group][k-step][kind y|z][t][piece] x 8 bytes: columns 4q, 4q+1 are code
// byte 2q' of the group (q' = q % 32), 4q+2, 4q+3 byte 2q'+1: word q'/2,
// chunk t = q'/8, k-step and half of the word within the chunk, bytes
// 2(q' % 2) and 2(q' % 2) + 1 of the register.  xsc[2 group] = 1 / S (NaN
// when x holds a non-finite value, whose rows are then NaN as the f32 dot
// product would be), xsc[2 group + 1] = the group's x sum.
constexpr uint32_t kMmaPieces = 4;
CHPE_DEV void mma_b_put_quad(uint8_t* bstage, float* xsc, uint32_t q, const float4& o, uint32_t L) {
  const uint32_t G = q >> 5, qq = q & 31u, t = qq >> 3, wic = (qq >> 1) & 3u;
  const uint32_t s_ = wic >> 1, up = wic & 1u, bi = 2u * (qq & 1u);
  const float y0 = o.x, z0 = o.y * 0.0625f, y1 = o.z, z1 = o.w * 0.0625f;
  float m = fmaxf(fmaxf(fabsf(y0), fabsf(z0)), fmaxf(fabsf(y1), fabsf(z1)));
  if (!(m <= 3.402823466e38f)) m = __int_as_float(0x7f800000);  // NaN -> inf
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, sh));
  float S = 1.0f, invS = 1.0f;
  if (!(m <= 3.402823466e38f)) {
    S = 0.0f;  // pieces 0, rows NaN
    invS = __int_as_float(0x7fc00000);
  } else if (m > 0.0f) {
    int ex;
    frexpf(m, &ex);  // m in [2^(ex-1), 2^ex)
    const int k = 6 - ex < 126 ? 6 - ex : 126;
    S = ldexpf(1.0f, k);
    invS = ldexpf(1.0f, -k);
  }
  uint8_t* bb = bstage + (((G * 2u + s_) * 2u) * 4u + t) * kMmaPieces * 8u + up * 4u + bi;
  float ry0 = y0 * S, ry1 = y1 * S, rz0 = z0 * S, rz1 = z1 * S;
#pragma unroll
  for (uint32_t n = 0; n < kMmaPieces; n++) {
    const float iy0 = rintf(ry0), iy1 = rintf(ry1), iz0 = rintf(rz0), iz1 = rintf(rz1);
    const uint16_t py = (uint16_t)((uint32_t)((int)iy0 & 0xff) | ((uint32_t)((int)iy1 & 0xff) << 8));
    const uint16_t pz = (uint16_t)((uint32_t)((int)iz0 & 0xff) | ((uint32_t)((int)iz1 & 0xff) << 8));
    *reinterpret_cast<uint16_t*>(bb + n * 8u) = py;                         // kind 0: y
    *reinterpret_cast<uint16_t*>(bb + 4u * kMmaPieces * 8u + n * 8u) = pz;   // kind 1: z
    ry0 = (ry0 - iy0) * 128.0f;
    ry1 = (ry1 - iy1) * 128.0f;
    rz0 = (rz0 - iz0) * 128.0f;
    rz1 = (rz1 - iz1) * 128.0f;
  }
  const float sx = warp_sum((o.x + o.y) + (o.z + o.w));
  if (L == 0) {
    xsc[2 * G] = invS;
    xsc[2 * G + 1] = sx;
  }
}

// An int32 of magnitude below 2^22 as a float, exactly: its bits added to
// those of 1.5 * 2^23 give 1.5 * 2^23 + v, from which 1.5 * 2^23 is removed.
CHPE_DEV float s32_exact(int v) { return __int_as_float(v + 0x4B400000) - 12582912.0f; }

// Chunk sum of (weight code value) * x from the quad accumulators.
template <int FMT>
CHPE_DEV float chunk_finish(f2x a0, f2x a1, float xsum) {
  const float2 p = unpack2(a0), r = unpack2(a1);
  const float s = (p.x + r.x) + (p.y + r.y);
  if constexpr (FMT == FMT_W4G || FMT == FMT_W4SB) return 256.0f * s - 136.0f * xsum;  // (c-8) x
  else if constexpr (FMT == FMT_W2G || FMT == FMT_W2SB) return 256.0f * s - 130.0f * xsum;
  else return s;
}

// Address of chunk `ch` of row r and its validity.
template <int FMT, int KIND>
CHPE_DEV const uint8_t* chunk_addr(const GemvSrc& s, uint32_t r, uint32_t ch, bool& ok,
                                   const uint8_t*& payload, uint32_t& grp) {
  using FI = FmtInfo<FMT>;
  if constexpr (KIND == SRC_ROWTILE) {
    uint32_t k = r / s.cell_rows, rin = r - k * s.cell_rows;
    const uint8_t* cell = s.arc + s.tile0 + (uint64_t)k * s.stride;
    payload = cell + 16384;
    grp = rin * (s.cell_cols >> 7) + (ch * FI::CW >> 7);
    ok = r < s.rows_covered;
    return cell + (uint64_t)rin * (s.cell_cols * FI::BITS / 8) + 16u * ch;
  } else if constexpr (KIND == SRC_FLAT) {
    uint64_t f = (uint64_t)r * s.c_total + (uint64_t)FI::CW * ch;
    ok = f < s.flat_limit;
    uint64_t t = f >> 15;
    uint32_t off = (uint32_t)(f & 32767u);
    const uint8_t* cell = s.arc + s.tile0 + t * s.stride;
    payload = cell + 16384;
    grp = off >> 7;
    return cell + off * FI::BITS / 8;
  } else {  // SRC_RAW: tiles are contiguous
    uint64_t f = (uint64_t)r * s.c_total + (uint64_t)FI::CW * ch;
    ok = f < s.flat_limit;
    payload = nullptr;
    grp = 0;
    return s.arc + s.tile0 + f * (FI::BITS / 8);
  }
}

// Rows per warp iteration (NR) and chunk slots loaded per row at a time (UNR)
// for a (format, layout): eight 16-byte loads per lane in flight, except for
// 2-bit rows (one slot each, four rows).  The host sizes grids with the same
// rule (jobs per iteration = NR, or NR/2 gate+up pairs for SwiGLU).
__host__ __device__ constexpr int gemv_nr(int fmt, int kind) {
  return kind == SRC_ROWTILE && (fmt == FMT_W4G || fmt == FMT_W4SB || fmt == FMT_W2G || fmt == FMT_W2SB) ? 4 : 2;
}
__host__ __device__ constexpr int gemv_unr(int fmt, int kind) {
  return kind == SRC_ROWTILE && (fmt == FMT_W2G || fmt == FMT_W2SB) ? 1
         : kind == SRC_ROWTILE && (fmt == FMT_W4G || fmt == FMT_W4SB) ? 2 : 4;
}

// Dot products of NR rows against the staged x.  Every lane first issues the
// 16-byte code loads (and scale loads) of UNR chunk slots of all NR rows,
// then walks the slots quad by quad: each x quad is read from shared memory
// once and applied to all NR rows.  A warp keeps NR*UNR*512 bytes in flight.
//
// Row-tiled tensors (KIND == SRC_ROWTILE) always have 2048 columns and full
// cells here, so no chunk needs a bounds test and the cell geometry is fixed.
template <int FMT, int KIND, int NR, int UNR>
CHPE_DEV void rows_dot(const GemvSrc* const* sp, const uint32_t* rr, const bool* vv, const float* xs,
                       const float* xsum, uint32_t nchunks, uint32_t L, float* acc) {
  using FI = FmtInfo<FMT>;
  constexpr int QPC = FI::CW / 4;
  constexpr bool RT = KIND == SRC_ROWTILE;
#pragma unroll
  for (int n = 0; n < NR; n++) acc[n] = 0.f;
  // row-tiled rows are 2048 columns: a compile-time slot count
  const uint32_t nslots = RT ? (uint32_t)(2048 / (32 * FI::CW)) : (nchunks + 31) >> 5;
  // per-row bases (row-tiled: cell and row inside it, shifts only; rows past
  // the covered range load a covered row and are dropped at the end)
  const uint8_t* rowp[NR];
  const uint8_t* scp[NR];
  bool rok[NR];
#pragma unroll
  for (int n = 0; n < NR; n++) {
    rok[n] = vv[n];
    if constexpr (RT) {
      const GemvSrc& s = *sp[n];
      rok[n] = vv[n] && rr[n] < s.rows_covered;
      const uint32_t r = rok[n] ? rr[n] : 0u;
      const uint32_t k = r / FI::CELL_ROWS, rin = r % FI::CELL_ROWS;
      const uint8_t* cell = s.arc + s.tile0 + (uint64_t)k * s.stride;
      rowp[n] = cell + rin * (2048u * FI::BITS / 8);
      scp[n] = cell + 16384;
      if constexpr (FI::GROUPED) scp[n] += 48 + 2 * rin * 16;
    } else {
      rowp[n] = nullptr;
      scp[n] = nullptr;
    }
  }
  for (uint32_t j0 = 0; j0 < nslots; j0 += UNR) {
    uint4 v[NR][UNR];
    float sc[NR][UNR], bi[NR][UNR];
    bool ok[NR][UNR];
#pragma unroll
    for (int n = 0; n < NR; n++) {
#pragma unroll
      for (int u = 0; u < UNR; u++) {
        const uint32_t ch = L + 32u * (j0 + u);
        sc[n][u] = 1.f;
        bi[n][u] = 0.f;
        if constexpr (RT) {
          ok[n][u] = rok[n];
          v[n][u] = ld_stream(rowp[n] + 16u * ch);
          if constexpr (FI::GROUPED) sc[n][u] = ld_f16(scp[n] + 2 * (ch * FI::CW / 128));
          if constexpr (FI::SB) { sc[n][u] = ld_f32(scp[n] + 32); bi[n][u] = ld_f32(scp[n] + 36); }
        } else {
          ok[n][u] = false;
          v[n][u] = make_uint4(0u, 0u, 0u, 0u);
          if (vv[n] && j0 + u < nslots && ch < nchunks) {
            const uint8_t* pl;
            uint32_t grp;
            bool o;
            const uint8_t* a = chunk_addr<FMT, KIND>(*sp[n], rr[n], ch, o, pl, grp);
            ok[n][u] = o;
            if (o) {
              v[n][u] = ld_stream(a);
              if constexpr (FI::GROUPED) sc[n][u] = ld_f16(pl + 48 + 2 * grp);
              if constexpr (FI::SB) { sc[n][u] = ld_f32(pl + 32); bi[n][u] = ld_f32(pl + 36); }
            }
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < UNR; u++) {
      if (!RT && j0 + u >= nslots) break;
      const uint32_t ch = L + 32u * (j0 + u);
      const bool chv = RT || ch < nchunks;
      f2x a2[NR][2];
#pragma unroll
      for (int n = 0; n < NR; n++) a2[n][0] = a2[n][1] = 0ull;
#pragma unroll
      for (int q = 0; q < QPC; q++) {
        const ulonglong2 xq = reinterpret_cast<const ulonglong2*>(xs)[((j0 + u) * QPC + q) * 32u + L];
#pragma unroll
        for (int n = 0; n < NR; n++) quad_fma<FMT>(v[n][u], q, xq.x, xq.y, a2[n][q & 1]);
      }
      const float xsm = chv ? xsum[chv ? ch : 0] : 0.f;
#pragma unroll
      for (int n = 0; n < NR; n++) {
        const float d = chunk_finish<FMT>(a2[n][0], a2[n][1], xsm);
        float t;
        if constexpr (FI::GROUPED) t = fmaf(d, sc[n][u], acc[n]);
        else if constexpr (FI::SB) t = fmaf(bi[n][u], xsm, fmaf(d, sc[n][u], acc[n]));
        else t = acc[n] + d;
        acc[n] = ok[n][u] ? t : acc[n];
      }
    }
  }
}

// Additive row outliers of W4G/W2G row-tiled cells with 16 rows
// (chpe_engine.zig:244-256, 309-315): lanes 0..7 each add one term.
// With OUTL_REPLACE (tied embedding head, unpackEmbedRowCell :1335-1344,
// :1369-1378) the cell's decoded value at col is replaced instead: lane k adds
// (w_k - decoded)*x unless a later entry names the same column.
CHPE_DEV float outlier_term(const GemvSrc& s, uint32_t r, const float* xs, uint32_t L, int cw) {
  if (L >= 8 || r >= s.rows_covered) return 0.f;
  uint32_t k = r / s.cell_rows, rin = r - k * s.cell_rows;
  const uint8_t* code = s.arc + s.tile0 + (uint64_t)k * s.stride;
  const uint8_t* pl = code + 16384;
  uint32_t col = ld_u16(pl + 816 + 2 * L);
  if (col >= s.x_len) return 0.f;
  float xv = (cw == 32) ? xs[xpos<32>(col)] : xs[xpos<64>(col)];
  float w = ld_f16(pl + 560 + 2 * (rin * 8 + L));
  if (s.outliers == OUTL_ADD) return w * xv;
  for (uint32_t k2 = L + 1; k2 < 8; k2++)
    if (ld_u16(pl + 816 + 2 * k2) == col) return 0.f;
  float sc = ld_f16(pl + 48 + 2 * (rin * (s.cell_cols >> 7) + (col >> 7)));
  float dec;
  if (cw == 32) {
    uint8_t b = code[rin * (s.cell_cols / 2) + col / 2];
    dec = ((float)((col & 1) ? (b >> 4) & 15 : b & 15) - 8.0f) * sc;
  } else {
    const float CB[4] = {0.f, 1.f, -2.f, -1.f};
    uint8_t b = code[rin * (s.cell_cols / 4) + col / 4];
    dec = CB[(b >> (2 * (col & 3))) & 3] * sc;
  }
  return (w - dec) * xv;
}

template <int FMT, int KIND, int THREADS, int NR, int UNR>
__global__ void __launch_bounds__(THREADS, 65536 / (THREADS * 128)) gemv_kernel(const __grid_constant__ GemvLaunch P) {
  using FI = FmtInfo<FMT>;
  extern __shared__ __align__(16) float smem[];
  const uint32_t tid = threadIdx.x, L = tid & 31u, warp = tid >> 5;
  const uint32_t nwarps = THREADS / 32;
  const uint32_t ncols = P.ncols;
  const uint32_t nchunks = (ncols + FI::CW - 1) / FI::CW;
  const uint32_t nslots = (nchunks + 31) >> 5;
  float* xs = smem;
  float* xsum = smem + nslots * 32u * FI::CW;
  __shared__ float red[THREADS / 32];

  // Weight prefetch into L2 before waiting on the predecessor kernel.
  for (int sg = 0; sg < 3; sg++) {
    uint64_t nb = P.prefetch_bytes[sg];
    if (!nb) continue;
    uint64_t per = ((nb + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
    uint64_t b0 = per * blockIdx.x, b1 = b0 + per < nb ? b0 + per : nb;
    for (uint64_t o = b0 + (uint64_t)tid * 16384; o < b1; o += (uint64_t)THREADS * 16384) {
      uint64_t n = b1 - o < 16384 ? b1 - o : 16384;
      n &= ~15ull;
      if (n) prefetch_l2(P.prefetch_base[sg] + o, (uint32_t)n);
    }
  }
  pdl_wait();
  if (!P.ignore_stop && P.st->stop) return;

  // ---- stage x (optionally RMSNorm'ed) into shared memory ----------------
  // Each thread owns float4 quads q = tid + i*THREADS; all loads of a block of
  // XV quads are issued before any is used.  The CW/4 quads of one chunk sit
  // in consecutive lanes, so chunk x-sums are segmented shuffle reductions.
  constexpr int XV = 8;
  constexpr int QPC = FI::CW / 4;  // quads per chunk
  const float* xin = P.x;
  float tot = 0.f;
  const uint32_t nquads = ncols / 4;                      // ncols % 4 == 0
  const uint32_t nquads_pad = nslots * 32u * (uint32_t)QPC;
  const float4* x4 = reinterpret_cast<const float4*>(xin);
  const float4* g4 = reinterpret_cast<const float4*>(P.gamma);
  for (uint32_t q0 = 0; q0 < nquads_pad; q0 += THREADS * XV) {
    float4 v[XV], g[XV];
#pragma unroll
    for (int i = 0; i < XV; i++) {
      uint32_t q = q0 + tid + (uint32_t)i * THREADS;
      v[i] = q < nquads ? x4[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (P.norm) g[i] = q < nquads ? g4[q] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (P.norm) {
      // a norm prologue always fits one block (ncols = hidden_dim <= THREADS*XV*4)
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < XV; i++) ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
      ss = warp_sum(ss);
      if (L == 0) red[warp] = ss;
      __syncthreads();
      for (uint32_t w = 0; w < nwarps; w++) tot += red[w];
      if (P.check_layer >= 0) {
        // end-of-layer check of the reference's debug block (chpe_engine.zig:1753-1764)
        int l = P.check_layer;
        bool cond = l < 3 || (l >= 8 && l <= 16) || !isfinite(xin[0]);
        if (cond && !isfinite(tot)) {
          if (blockIdx.x == 0 && tid == 0) P.st->stop = 1;
          return;
        }
      }
      const float inv = 1.0f / sqrtf(tot / (float)ncols + P.eps);
#pragma unroll
      for (int i = 0; i < XV; i++) {
        v[i].x = v[i].x * inv * g[i].x;
        v[i].y = v[i].y * inv * g[i].y;
        v[i].z = v[i].z * inv * g[i].z;
        v[i].w = v[i].w * inv * g[i].w;
      }
    }
#pragma unroll
    for (int i = 0; i < XV; i++) {
      uint32_t q = q0 + tid + (uint32_t)i * THREADS;
      float qs = (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
      for (int o = 1; o < QPC; o <<= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
      if (q < nquads_pad) {
        *reinterpret_cast<float4*>(&xs[xpos<FI::CW>(q * 4)]) = v[i];
        if ((q % QPC) == 0) xsum[q / QPC] = qs;
        if (P.xn_out && blockIdx.x == 0 && q < nquads) reinterpret_cast<float4*>(P.xn_out)[q] = v[i];
      }
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  // ---- rows --------------------------------------------------------------
  unsigned long long lbest = 0ull;  // EPI_LOGITS per-lane (lane 0) running best
  uint32_t lfin = 1u;
  const bool swig = P.epi == EPI_SWIGLU;
  const uint32_t total = swig ? P.row_start[1] : P.row_start[P.nseg];
  constexpr int JPI_PLAIN = NR;
  const uint32_t jpi = swig ? (uint32_t)(NR / 2) : (uint32_t)JPI_PLAIN;  // jobs per iteration
  for (uint32_t j0 = (blockIdx.x * nwarps + warp) * jpi; j0 < total; j0 += gridDim.x * nwarps * jpi) {
    const GemvSrc* sp[NR];
    uint32_t rr[NR], sg[NR];
    bool vv[NR];
#pragma unroll
    for (int n = 0; n < NR; n++) {
      uint32_t job = j0 + (swig ? (uint32_t)(n >> 1) : (uint32_t)n);
      vv[n] = job < total;
      uint32_t seg = 0, r = job;
      if (swig) {
        seg = (uint32_t)(n & 1);
      } else {
        while ((int)seg + 1 < P.nseg && job >= P.row_start[seg + 1]) seg++;
        r = job - P.row_start[seg];
      }
      sg[n] = seg;
      rr[n] = r;
      sp[n] = &P.src[seg];
    }
    float acc[NR];
    rows_dot<FMT, KIND, NR, UNR>(sp, rr, vv, xs, xsum, nchunks, L, acc);
#pragma unroll
    for (int n = 0; n < NR; n++) {
      if constexpr (KIND == SRC_ROWTILE && FI::GROUPED) {
        if (vv[n] && sp[n]->outliers) acc[n] += outlier_term(*sp[n], rr[n], xs, L, FI::CW);
      }
      acc[n] = warp_sum(acc[n]);
    }
    if (L != 0) continue;
    if (swig) {
#pragma unroll
      for (int n = 0; n + 1 < NR; n += 2)
        if (vv[n]) P.out[0][rr[n]] = silu_ref(acc[n]) * acc[n + 1];
      continue;
    }
#pragma unroll
    for (int n = 0; n < NR; n++) {
      if (!vv[n]) continue;
      float d = acc[n];
      const uint32_t r = rr[n];
      const GemvSrc& s = *sp[n];
      if constexpr (FMT == FMT_I8RAW) d *= 0.00373708f;
      float* y = P.out[sg[n]];
      if (P.epi == EPI_LOGITS) {
        y[r] = d;
        if (!isfinite(d)) lfin = 0u;
        if (d > -1e30f) {
          unsigned long long kk = argmax_key(d, r);
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
  }
  if (P.epi == EPI_LOGITS) {
    // argmax / finiteness over this CTA, then one atomic each; the last CTA
    // to arrive writes the step result (chpe_engine.zig:1775-1802).
    __shared__ unsigned long long kbest[THREADS / 32];
    __shared__ uint32_t kfin[THREADS / 32];
    __shared__ int is_last;
    if (L == 0) { kbest[warp] = lbest; kfin[warp] = lfin; }
    __syncthreads();
    if (tid == 0) {
      unsigned long long b = 0ull;
      uint32_t f = 1u;
      for (uint32_t w = 0; w < nwarps; w++) { b = kbest[w] > b ? kbest[w] : b; f &= kfin[w]; }
      if (b) atomicMax(&P.st->best, b);
      if (!f) atomicAnd(&P.st->finite, 0u);
      __threadfence();
      unsigned prev = atomicAdd(&P.st->done_ctas, 1u);
      is_last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last && tid == 0) {
      __threadfence();
      unsigned long long b = atomicAdd(&P.st->best, 0ull);
      StepResult R;
      R.argmax_token = b ? 0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull) : 0u;
      R.max_logit = b ? key_value(b) : -1e30f;
      R.token0_logit = __ldcg(P.out[0]);
      R.hidden_norm = sqrtf(tot);
      R.all_finite = (int32_t)atomicAdd(&P.st->finite, 0u);
      R.pos = P.st->pos;
      *P.res = R;
      if (P.gen_tokens && P.st->n_gen < P.max_gen) P.gen_tokens[P.st->n_gen] = (int32_t)R.argmax_token;
      P.st->n_gen += 1;
      P.st->pos += 1;
      P.st->best = 0ull;
      P.st->finite = 1u;
      P.st->done_ctas = 0u;
    }
  }
}

// ---- generic exact path (any cell format, per-tile dispatch) --------------
// Restates gemvTilePolymorphic / gemvCellFlat one weight at a time; used for
// archives whose tensors mix formats or geometries.
CHPE_DEV float cell_weight_rowtile(const uint8_t* cell_code, uint32_t qb, uint64_t flags,
                                   float scale, float bias, uint32_t cols, uint32_t rin,
                                   uint32_t c) {
  const uint8_t* pl = cell_code + 16384;
  const bool g128 = (flags & 1u) != 0;
  if (qb == 4) {
    uint8_t b = cell_code[rin * (cols / 2) + c / 2];
    int n = (c & 1) ? (b >> 4) & 15 : b & 15;
    if (g128) return ((float)n - 8.0f) * ld_f16(pl + 48 + 2 * (rin * (cols / 128) + c / 128));
    return (float)(n - 8) * scale + bias;
  } else if (qb == 8) {
    return (float)(int8_t)cell_code[rin * cols + c];
  } else if (qb == 16) {
    uint16_t h = ld_u16(cell_code + 2 * ((uint64_t)rin * cols + c));
    return (flags & 4u) ? h2f(h) : bf2f(h);
  } else if (qb == 32) {
    return ld_f32(cell_code + 4 * ((uint64_t)rin * cols + c));
  }
  const float CB[4] = {0.f, 1.f, -2.f, -1.f};
  uint8_t b = cell_code[rin * (cols / 4) + c / 4];
  float cb = CB[(b >> (2 * (c & 3))) & 3];
  if (g128) return cb * ld_f16(pl + 48 + 2 * (rin * (cols / 128) + c / 128));
  return cb * scale + bias;
}

struct GenLaunch {
  GemvSrc src;
  float* y;
  const float* x;
  int32_t accumulate;
  StepState* st;
};

// Row-tiled cells of any format: one warp per row.
static __global__ void __launch_bounds__(256) gemv_generic_rowtile(const __grid_constant__ GenLaunch P) {
  pdl_wait();
  if (P.st && P.st->stop) return;
  const GemvSrc& s = P.src;
  const uint32_t L = threadIdx.x & 31u;
  for (uint32_t r = blockIdx.x * 8 + (threadIdx.x >> 5); r < s.r_total; r += gridDim.x * 8) {
    uint32_t k = s.row_cell[r];
    if (k == 0xFFFFFFFFu) {  // not covered by any cell: stays 0 (or untouched)
      if (L == 0) {
        float v = P.accumulate ? P.y[r] : 0.f;
        if (s.bias) v += s.bias[r];
        P.y[r] = v;
      }
      continue;
    }
    uint32_t rin = s.row_in_cell[r];
    const uint8_t* code = s.arc + s.tile0 + (uint64_t)k * s.stride;
    const uint8_t* pl = code + 16384;
    uint32_t qb = pl[20];
    uint64_t flags = *reinterpret_cast<const uint64_t*>(pl + 24);
    float scale = ld_f32(pl + 32), bias = ld_f32(pl + 36);
    uint32_t rows = *reinterpret_cast<const uint32_t*>(pl + 40);
    uint32_t cols = *reinterpret_cast<const uint32_t*>(pl + 44);
    bool g128 = (flags & 1u) != 0;
    uint32_t ncols;
    if ((qb == 4 || (qb != 8 && qb != 16 && qb != 32)) && g128)
      ncols = min(cols / 128, s.x_len / 128) * 128;
    else if (qb == 4)
      ncols = min(cols / 2, s.x_len / 2) * 2;
    else if (qb != 8 && qb != 16 && qb != 32)
      ncols = min(cols / 4, s.x_len / 4) * 4;
    else
      ncols = min(cols, s.x_len);
    float acc = 0.f;
    for (uint32_t c = L; c < ncols; c += 32)
      acc = fmaf(cell_weight_rowtile(code, qb, flags, scale, bias, cols, rin, c), P.x[c], acc);
    if ((qb == 4 || (qb != 8 && qb != 16 && qb != 32)) && g128 && rows == 16 && L < 8) {
      uint32_t col = ld_u16(pl + 816 + 2 * L);
      float xv = col < s.x_len ? P.x[col] : 0.f;
      acc = fmaf(ld_f16(pl + 560 + 2 * (rin * 8 + L)), xv, acc);
    }
    acc = warp_sum(acc);
    if (qb == 8) acc = acc * scale + bias;
    if (L == 0) {
      float v = P.accumulate ? P.y[r] + acc : acc;
      if (s.bias) v += s.bias[r];
      P.y[r] = v;
    }
  }
}

// Flat cells of any format: one warp per row, per-chunk tile dispatch.
static __global__ void __launch_bounds__(256) gemv_generic_flat(const __grid_constant__ GenLaunch P) {
  pdl_wait();
  if (P.st && P.st->stop) return;
  const GemvSrc& s = P.src;
  const uint32_t L = threadIdx.x & 31u;
  const float CB[4] = {0.f, 1.f, -2.f, -1.f};
  for (uint32_t r = blockIdx.x * 8 + (threadIdx.x >> 5); r < s.r_total; r += gridDim.x * 8) {
    float acc = 0.f;
    uint64_t f0 = (uint64_t)r * s.c_total;
    for (uint32_t c = L; c < s.c_total; c += 32) {
      uint64_t f = f0 + c;
      if (f >= s.flat_limit) break;
      uint64_t t = f >> 15;
      uint32_t off = (uint32_t)(f & 32767u);
      const uint8_t* code = s.arc + s.tile0 + t * s.stride;
      const uint8_t* pl = code + 16384;
      uint32_t qb = pl[20];
      uint64_t flags = *reinterpret_cast<const uint64_t*>(pl + 24);
      bool g128 = (flags & 1u) != 0;
      float w = 0.f;
      if (qb == 4) {
        uint8_t b = code[off / 2];
        int n = (off & 1) ? (b >> 4) & 15 : b & 15;
        w = g128 ? ((float)n - 8.0f) * ld_f16(pl + 48 + 2 * (off >> 7))
                 : ((float)n - 8.0f) * ld_f32(pl + 32) + ld_f32(pl + 36);
      } else if (qb == 2) {
        uint8_t b = code[off / 4];
        float cb = CB[(b >> (2 * (off & 3))) & 3];
        w = g128 ? cb * ld_f16(pl + 48 + 2 * (off >> 7)) : cb * ld_f32(pl + 32) + ld_f32(pl + 36);
      }
      if (qb == 4 || qb == 2) {
        uint32_t n = ld_u16(pl + 560);
        if (n > 0 && n <= 64) {
          for (uint32_t m = 0; m < n; m++)
            if (ld_u16(pl + 690 + 2 * m) == off) w = ld_f16(pl + 562 + 2 * m);
        }
      }
      acc = fmaf(w, P.x[c], acc);
    }
    acc = warp_sum(acc);
    if (L == 0) {
      float v = P.accumulate ? P.y[r] + acc : acc;
      if (s.bias) v += s.bias[r];
      P.y[r] = v;
    }
  }
}

// down_aux replacements of uniform flat cells: one thread per (tile, entry);
// adds (replacement - decoded) * x to the row it lands in.  Only the last
// entry for a given offset counts (later entries overwrite earlier ones).
struct AuxLaunch {
  GemvSrc src;
  float* y;
  const float* x;
  StepState* st;
};
static __global__ void flat_aux_fix(const __grid_constant__ AuxLaunch P) {
  pdl_wait();
  if (P.st && P.st->stop) return;
  const GemvSrc& s = P.src;
  const float CB[4] = {0.f, 1.f, -2.f, -1.f};
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint64_t t = i >> 6;
  uint32_t m = (uint32_t)(i & 63u);
  if (t >= s.n_tiles) return;
  const uint8_t* code = s.arc + s.tile0 + t * s.stride;
  const uint8_t* pl = code + 16384;
  uint32_t qb = pl[20];
  if (qb != 4 && qb != 2) return;
  uint32_t n = ld_u16(pl + 560);
  if (n == 0 || n > 64 || m >= n) return;
  uint32_t off = ld_u16(pl + 690 + 2 * m);
  if (off >= 32768) return;
  for (uint32_t m2 = m + 1; m2 < n; m2++)
    if (ld_u16(pl + 690 + 2 * m2) == off) return;
  uint64_t f = t * 32768u + off;
  if (f >= s.flat_limit) return;
  uint64_t r = f / s.c_total, c = f % s.c_total;
  if (r >= s.r_total) return;
  uint64_t flags = *reinterpret_cast<const uint64_t*>(pl + 24);
  bool g128 = (flags & 1u) != 0;
  float w;
  if (qb == 4) {
    uint8_t b = code[off / 2];
    int nn = (off & 1) ? (b >> 4) & 15 : b & 15;
    w = g128 ? ((float)nn - 8.0f) * ld_f16(pl + 48 + 2 * (off >> 7))
             : ((float)nn - 8.0f) * ld_f32(pl + 32) + ld_f32(pl + 36);
  } else {
    uint8_t b = code[off / 4];
    float cb = CB[(b >> (2 * (off & 3))) & 3];
    w = g128 ? cb * ld_f16(pl + 48 + 2 * (off >> 7)) : cb * ld_f32(pl + 32) + ld_f32(pl + 36);
  }
  float repl = ld_f16(pl + 562 + 2 * m);
  atomicAdd(&P.y[r], (repl - w) * P.x[c]);
}

}  // namespace chpe
