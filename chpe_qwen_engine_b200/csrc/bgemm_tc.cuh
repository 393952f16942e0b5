// bgemm_tc.cuh -- the batched (small-M) 4-bit GEMM of speculative
// verification and prompt chunks on the 5th-generation tensor cores.
//
// Y[t][r] = sum_c W[r][c] X[t][c] for NT tokens (4 or 8) at once, W a flat
// 4-bit group-128 tensor (gemvCellFlat's weights, chpe_engine.zig:584-729,
// the dequantised value (c - 8) * scale).  Each weight is read from HBM once
// for all NT tokens: at NT = 8 the CUDA-core FMA rate could not keep up with
// the weight stream, so the products run on tcgen05.mma.
//
// Operands (swap-AB: weights are the M = 128 operand, tokens the N one):
// a code byte lo + 16 hi holds the codes of columns 2p and 2p + 1, and
//   lo x0 + hi x1 = lo y + (16 hi) z,   y = x0, z = x1 / 16 (exact),
// so A is the code bytes masked with 0x0F (A_lo) and 0xF0 (A_hi), unsigned
// 8-bit, written by the threads straight from registers into tensor memory
// (one TMEM lane per weight row).  B holds, per 128-column group, y and z of
// every token as int8 pieces: scaled by a power of two S that puts the
// group's largest |y|, |z| in [32, 64), then split into four 7-bit pieces
// (value = i0 + i1/128 + i2/128^2 + i3/128^3), column n = 4 t + piece of B
// (N = 4 NT).  The four K = 32 MMAs of a group (A_lo x B_y and A_hi x B_z,
// two K halves each) accumulate exactly in s32 (|D| < 2^21), and per group
// and row the epilogue forms scale * (sum_n D_n 128^-n / S - 8 sum x) =
// scale * sum (c - 8) x from a tcgen05.ld of the row's D columns.
//
// B is built once per launch by bgemm_prep_kernel (into global memory, in
// the shared-memory layout) and every CTA copies its groups in with one bulk
// copy.
//
// Work split: a CTA takes one block of 128 rows and one range of at most
// kBgMaxGroups groups (split-K); two CTAs share an SM (256 TMEM columns and
// at most 128 registers per thread each), so one's prologue and epilogue
// overlap the other's stream.  Its 256 threads are two warpgroups; each
// processes alternate groups with its own two TMEM stages (A 32 columns,
// D 32 columns each).  Thread r of a warpgroup owns row r: it loads the row's
// 64 code bytes and scale of a group kBgAhead groups ahead (registers), masks
// them into the stage's A columns, and after the warpgroup's named barrier
// its first thread issues the group's MMAs and commits them to the stage's
// mbarrier; the epilogue of a group reads D once that mbarrier completes.
// Split-K partial sums go to a [ksplit][NT][rows] buffer; the last CTA of a
// block (arrival counter, reset by it) sums them in split order and applies
// the epilogue (store + bias, residual add, SwiGLU over the gate and up
// blocks of a pair, or logits with per-token argmax and finiteness).  Every
// sum has a fixed order, so results do not depend on timing.
#pragma once
#include "gemv.cuh"
#include "tc_common.cuh"

namespace chpe {

constexpr uint32_t kBgRows = 128;       // rows per block: the MMA's M
constexpr uint32_t kBgStages = 2;       // TMEM stages per warpgroup
constexpr uint32_t kBgAhead = 3;        // groups whose codes are loaded ahead of use
constexpr uint32_t kBgMaxGroups = 12;   // groups (128 columns) per CTA
constexpr uint32_t kBgThreads = 256;    // two warpgroups
constexpr uint32_t kBgTmemCols = 256;   // 2 warpgroups x 2 stages x (32 A + 32 D)

struct BgemmLaunch {
  GemvSrc src[3];          // FLAT, FMT_W4G segments; rows concatenated in order
  float* out[3];           // per segment [NT][out_stride] (SwiGLU: out[0])
  uint32_t row_start[4];   // prefix of segment rows (multiples of 128)
  int32_t nseg, epi;
  uint32_t C;              // columns (multiple of 128)
  uint32_t ksplit;         // column ranges per block
  uint32_t nunits;         // blocks x ksplit (the grid)
  uint32_t rows_total;     // rows over all segments (width of a partial row)
  uint32_t rows_avail[3];  // per segment: tensor rows (row0 included) whose weights the tiles hold;
                           // later rows contribute nothing (the reference never reaches them)
  const float* x;          // [NT][x_stride]
  uint32_t x_stride, out_stride;
  const float* gamma;      // RMSNorm gain over C (null: x used as is)
  float eps;
  float* part;             // [ksplit][NT][rows_total]
  uint32_t* counters;      // per block (SwiGLU: per gate/up pair), zero between launches
  unsigned long long* best;// EPI_LOGITS: [NT] argmax keys
  uint32_t* finite;        // EPI_LOGITS: [NT] finiteness flags
  int32_t* bad;            // EPI_ACCUM: set when a residual leaves [-1e18, 1e18] or is not finite
  int32_t* err;            // set when a bounded wait gave up
  // RMSNorm factors without re-reading x: an EPI_ACCUM launch writes, per
  // 128-row block, each token's sum of squares of the new rows to
  // ssq_out[block][NT]; a normalising launch with ssq_in sums its ssq_n
  // slots per token in block order (null: it reads x itself).
  float* ssq_out;
  const float* ssq_in;
  uint32_t ssq_n;
  // B pieces and per-(group, token) (1/S, sum x) of every group, written by
  // bgemm_prep_kernel: [G][128 N] bytes in the shared-memory layout of B, and
  // [G][NT][2] floats
  uint8_t* pieces;
  float* pxsc;
  // Timing trace (measurement only; null in the decode paths): per CTA the
  // global timer at entry, after the prologue, after the main loop and at
  // the end, as 4 consecutive u64; then, for CTA 0's first thread, 6 stamps
  // per main-loop iteration for the first 8 iterations (iteration start,
  // epilogue wait done, D read, A stored, warpgroup barrier passed, MMAs
  // issued).
  unsigned long long* trace;
};

CHPE_DEV unsigned long long bg_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct BgSmem {  // dynamic shared memory layout (bytes)
  uint32_t b, xsc, ycomb, total;
};
__host__ __device__ inline BgSmem bg_smem(uint32_t nt, uint32_t ng) {
  BgSmem s;
  const uint32_t n = 4u * nt;
  s.b = 0;                                       // ng x 128 n bytes of B pieces
  s.xsc = s.b + ng * 128u * n;                   // [nt][ng] (1/S, sum x)
  s.ycomb = s.xsc + nt * ng * 8u;                // [128][nt] second warpgroup's sums
  s.total = s.ycomb + kBgRows * nt * 4u;
  s.total = (s.total + 127u) & ~127u;
  return s;
}

// Byte offset of B element (n, k) of a group's lo or hi half: MMA block
// j = k / 32 of N x 32 bytes, K-major no-swizzle core matrices of 8 rows x
// 16 bytes, the two along K 128 bytes apart, row groups 256 bytes apart.
__host__ __device__ inline uint32_t bg_b_off(uint32_t n, uint32_t k, uint32_t N) {
  const uint32_t j = k >> 5, kk = k & 31u;
  return j * N * 32u + (n >> 3) * 256u + (kk >> 4) * 128u + (n & 7u) * 16u + (kk & 15u);
}

// B pieces of one 128-column group for every token, once per launch: CTA g
// = group g, warp t = token t (lane L: columns 4L..4L+3, code bytes 2L and
// 2L + 1).  RMSNorm factors from the sums of squares the last residual
// update left (ssq_in), or from x itself.  It lets the GEMM's CTAs start (and
// prefetch their weights into L2) before it has finished.
template <int NT>
__global__ void __launch_bounds__(NT * 32) bgemm_prep_kernel(const __grid_constant__ BgemmLaunch P) {
  constexpr uint32_t N = 4u * NT;
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t g = blockIdx.x, t = threadIdx.x >> 5, L = threadIdx.x & 31u;
  float inv = 1.0f;
  if (P.gamma) {
    float ss = 0.f;
    if (P.ssq_in) {
      for (uint32_t b = 0; b < P.ssq_n; b++) ss += P.ssq_in[b * NT + t];
    } else {
      const float* xr = P.x + (size_t)t * P.x_stride;
      for (uint32_t c = 4u * L; c < P.C; c += 128u) {
        const float4 v = *reinterpret_cast<const float4*>(xr + c);
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
      }
      ss = warp_sum(ss);
    }
    inv = 1.0f / sqrtf(ss / (float)P.C + P.eps);
  }
  const uint32_t c = g * 128u + 4u * L;
  float4 o = *reinterpret_cast<const float4*>(P.x + (size_t)t * P.x_stride + c);
  if (P.gamma) {
    const float4 gm = *reinterpret_cast<const float4*>(P.gamma + c);
    o.x = o.x * inv * gm.x;
    o.y = o.y * inv * gm.y;
    o.z = o.z * inv * gm.z;
    o.w = o.w * inv * gm.w;
  }
  const float y0 = o.x, z0 = o.y * 0.0625f, y1 = o.z, z1 = o.w * 0.0625f;
  float m = fmaxf(fmaxf(fabsf(y0), fabsf(z0)), fmaxf(fabsf(y1), fabsf(z1)));
  if (!(m <= 3.402823466e38f)) m = __int_as_float(0x7f800000);  // NaN -> inf
  m = warp_max(m);
  float Sc = 1.0f, invS = 1.0f;
  if (!(m <= 3.402823466e38f)) {
    Sc = 0.0f;  // pieces 0, rows NaN
    invS = __int_as_float(0x7fc00000);
  } else if (m > 0.0f) {
    int ex;
    frexpf(m, &ex);  // m in [2^(ex-1), 2^ex)
    const int k = 6 - ex < 126 ? 6 - ex : 126;
    Sc = ldexpf(1.0f, k);
    invS = ldexpf(1.0f, -k);
  }
  uint8_t* gb = P.pieces + (size_t)g * 128u * N;  // lo half, then hi half at + 64 N
  float ry0 = y0 * Sc, ry1 = y1 * Sc, rz0 = z0 * Sc, rz1 = z1 * Sc;
#pragma unroll
  for (uint32_t n = 0; n < 4u; n++) {
    const float iy0 = rintf(ry0), iy1 = rintf(ry1), iz0 = rintf(rz0), iz1 = rintf(rz1);
    const uint16_t py = (uint16_t)((uint32_t)((int)iy0 & 0xff) | ((uint32_t)((int)iy1 & 0xff) << 8));
    const uint16_t pz = (uint16_t)((uint32_t)((int)iz0 & 0xff) | ((uint32_t)((int)iz1 & 0xff) << 8));
    const uint32_t off = bg_b_off(4u * t + n, 2u * L, N);
    *reinterpret_cast<uint16_t*>(gb + off) = py;
    *reinterpret_cast<uint16_t*>(gb + 64u * N + off) = pz;
    ry0 = (ry0 - iy0) * 128.0f;
    ry1 = (ry1 - iy1) * 128.0f;
    rz0 = (rz0 - iz0) * 128.0f;
    rz1 = (rz1 - iz1) * 128.0f;
  }
  const float sx = warp_sum((o.x + o.y) + (o.z + o.w));
  if (L == 0) {
    P.pxsc[2u * (g * NT + t)] = invS;
    P.pxsc[2u * (g * NT + t) + 1u] = sx;
  }
}

template <int NT>
__global__ void __launch_bounds__(kBgThreads, 2) bgemm_w4_kernel(const __grid_constant__ BgemmLaunch P) {
  constexpr uint32_t N = 4u * NT;
  extern __shared__ __align__(1024) uint8_t bsm[];
  __shared__ __align__(8) uint64_t dfull[2][kBgStages];
  __shared__ __align__(8) uint64_t bfull;
  __shared__ uint32_t s_taddr;
  __shared__ float s_red[4 * NT];
  __shared__ int s_last;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, L = tid & 31u;
  const uint32_t wg = tid >> 7, row = tid & 127u;
  if (P.trace && tid == 0) P.trace[4 * blockIdx.x] = bg_now();

  // this CTA's block and column range
  const uint32_t split = blockIdx.x % P.ksplit, blk = blockIdx.x / P.ksplit;
  const uint32_t G = P.C >> 7;
  const uint32_t g0 = split * G / P.ksplit, g1 = (split + 1) * G / P.ksplit, ng = g1 - g0;
  const uint32_t grow0 = blk * kBgRows;  // first row over the concatenated segments
  uint32_t seg = 0;
  while (seg + 1 < (uint32_t)P.nseg && grow0 >= P.row_start[seg + 1]) seg++;
  const GemvSrc& S = P.src[seg];
  const uint32_t lrow0 = grow0 - P.row_start[seg];  // segment-local first row
  const BgSmem lay = bg_smem(NT, ng);

  if (warp == 0) {
    tc::tmem_alloc(&s_taddr, kBgTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int w = 0; w < 2; w++)
      for (uint32_t s = 0; s < kBgStages; s++) mbar_init(&dfull[w][s], 1);
    mbar_init(&bfull, 1);
    fence_mbar_init();
  }
  // where row `row` of this block keeps the codes of group g (64 bytes) and
  // its scale: flat weight index -> (tile, offset)
  const uint64_t rflat = (uint64_t)(S.row0 + lrow0 + row) * P.C;
  const bool have = S.row0 + lrow0 + row < P.rows_avail[seg];
  auto code_ptr = [&](uint32_t g, const uint8_t** sc) -> const uint8_t* {
    const uint64_t idx = rflat + (uint64_t)g * 128u;
    const uint64_t t = idx >> 15, w = idx & 32767u;
    const uint8_t* base = S.arc + S.tile0 + t * S.stride;
    *sc = base + 16384u + 48u + 2u * (uint32_t)(w >> 7);
    return base + (w >> 1);
  };
  if (wg == 0 && have) {  // L2 prefetch of the block's codes in this column range, before the PDL wait
    const uint8_t* sc;
    const uint64_t a = rflat + (uint64_t)g0 * 128u, b = rflat + (uint64_t)g1 * 128u;
    if ((a >> 15) == ((b - 1) >> 15)) {
      prefetch_l2(code_ptr(g0, &sc), (uint32_t)((b - a) >> 1));
    } else {
      const uint32_t gm = (uint32_t)((((a >> 15) + 1) << 15) - rflat) >> 7;  // first group of the next tile
      prefetch_l2(code_ptr(g0, &sc), (gm - g0) * 64u);
      prefetch_l2(code_ptr(gm, &sc), (g1 - gm) * 64u);
    }
  }
  pdl_wait();
  __syncthreads();  // the barriers initialised above are visible to every thread

  // this CTA's groups of B and their (1/S, sum x), prepared by
  // bgemm_prep_kernel, copied in with two bulk copies
  float* xsc = reinterpret_cast<float*>(bsm + lay.xsc);
  {
    const uint32_t nb = ng * 128u * N, nx = ng * (uint32_t)NT * 8u;
    if (tid == 0) {
      mbar_expect_tx(&bfull, nb + nx);
      bulk_g2s(bsm + lay.b, P.pieces + (size_t)g0 * 128u * N, nb, &bfull);
      bulk_g2s(xsc, P.pxsc + (size_t)g0 * NT * 2u, nx, &bfull);
    }
    if (!mbar_wait(&bfull, 0)) {
      if (tid == 0) atomicExch(P.err, 1);
    }
  }
  fence_proxy_async_smem();  // B written by threads, read by the tensor core
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t taddr = s_taddr;
  const uint32_t lane_base = (uint32_t)((warp & 3u) * 32u) << 16;

  if (P.trace && tid == 0) P.trace[4 * blockIdx.x + 1] = bg_now();
  // ---- main loop: this warpgroup's groups gl = wg, wg + 2, ... ----------
  float y[NT];
#pragma unroll
  for (int t = 0; t < NT; t++) y[t] = 0.f;
  const uint32_t nmy = ng > wg ? (ng - wg + 1u) / 2u : 0u;
  // codes of the next kBgAhead (3) groups in a register queue (c0 next), and
  // the scales of the groups in the two TMEM stages (q0 oldest): shifted,
  // never indexed at run time
  static_assert(kBgAhead == 3 && kBgStages == 2, "the register queues below are written for 3 and 2");
  uint4 c0[4], c1[4], c2[4];
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, q0 = 0.f, q1 = 0.f;
  auto load = [&](uint32_t i, uint4 (&cr)[4], float& sc) {
    if (i >= nmy) return;
    if (!have) {  // a row past the tensor's tiles: zero codes and scale
#pragma unroll
      for (int v = 0; v < 4; v++) cr[v] = make_uint4(0u, 0u, 0u, 0u);
      sc = 0.f;
      return;
    }
    const uint8_t* sp;
    const uint8_t* cp = code_ptr(g0 + wg + 2u * i, &sp);
#pragma unroll
    for (int v = 0; v < 4; v++) cr[v] = ld_stream(cp + 16 * v);
    sc = ld_f16(sp);
  };
  load(0, c0, s0);
  load(1, c1, s1);
  load(2, c2, s2);
  bool failed = false;
  const uint32_t idesc = tc::idesc_i8_u8s8(kBgRows, N);
  unsigned long long* tr = (P.trace && blockIdx.x == 0 && tid == 0) ? P.trace + 4u * gridDim.x : nullptr;
  uint32_t it_now = 0;
  auto stamp = [&](uint32_t k) {
    if (tr && it_now < 8u) tr[it_now * 6u + k] = bg_now();
  };
  auto epilogue = [&](uint32_t k, float scale) {
    const uint32_t s = k % kBgStages, gl = wg + 2u * k;
    if (!failed && !mbar_wait(&dfull[wg][s], (k / kBgStages) & 1u)) {
      failed = true;
      if (row == 0) atomicExch(P.err, 1);
    }
    stamp(1);
    tc::fence_after_sync();
    if (failed) return;
    const uint32_t dcol = (wg * kBgStages + s) * 64u + 32u;
    uint32_t d[N];
#pragma unroll
    for (uint32_t cc = 0; cc < N; cc += 16u)
      tc::ld16(taddr + lane_base + dcol + cc, *reinterpret_cast<uint32_t(*)[16]>(&d[cc]));
    tc::ld_wait();
    stamp(2);
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const float d0 = (float)(int32_t)d[4 * t], d1 = (float)(int32_t)d[4 * t + 1];
      const float d2 = (float)(int32_t)d[4 * t + 2], d3 = (float)(int32_t)d[4 * t + 3];
      const float sum = (d0 + d1 * 0.0078125f) + (d2 * 6.103515625e-05f + d3 * 4.76837158203125e-07f);
      const float invS = xsc[2u * (gl * NT + t)], sx = xsc[2u * (gl * NT + t) + 1u];
      y[t] = fmaf(scale, fmaf(sum, invS, -8.0f * sx), y[t]);
    }
  };
  for (uint32_t i = 0; i < nmy; i++) {
    const uint32_t s = i % kBgStages, gl = wg + 2u * i;
    it_now = i;
    stamp(0);
    if (i >= kBgStages) {  // frees stage s
      epilogue(i - kBgStages, q0);
      q0 = q1;
    }
    uint32_t lo[16], hi[16];
#pragma unroll
    for (int v = 0; v < 4; v++) {
      const uint32_t w4[4] = {c0[v].x, c0[v].y, c0[v].z, c0[v].w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        lo[4 * v + e] = w4[e] & 0x0F0F0F0Fu;
        hi[4 * v + e] = w4[e] & 0xF0F0F0F0u;
      }
    }
    if (i == 0) q0 = s0;  // the stages now hold group 0 (q0) ...
    else q1 = s0;         // ... or groups i-1 (q0, after the shift above) and i (q1)
#pragma unroll
    for (int v = 0; v < 4; v++) {
      c0[v] = c1[v];
      c1[v] = c2[v];
    }
    s0 = s1;
    s1 = s2;
    load(i + kBgAhead, c2, s2);
    const uint32_t acol = (wg * kBgStages + s) * 64u;
    tc::st16(taddr + lane_base + acol, lo);
    tc::st16(taddr + lane_base + acol + 16u, hi);
    tc::st_wait();
    stamp(3);
    tc::fence_before_sync();
    asm volatile("bar.sync %0, 128;" ::"r"(1u + wg) : "memory");  // this warpgroup's A is complete
    stamp(4);
    if (row == 0) {
      tc::fence_after_sync();
      const uint8_t* gb = bsm + lay.b + gl * 128u * N;
      const uint32_t dt = taddr + acol + 32u;
#pragma unroll
      for (uint32_t j = 0; j < 2; j++)
        tc::mma_i8_ts(dt, taddr + acol + 8u * j, tc::smem_desc_kmajor(gb + j * N * 32u, 128u, 256u), idesc, j);
#pragma unroll
      for (uint32_t j = 0; j < 2; j++)
        tc::mma_i8_ts(dt, taddr + acol + 16u + 8u * j,
                      tc::smem_desc_kmajor(gb + 64u * N + j * N * 32u, 128u, 256u), idesc, 1u);
      tc::commit(&dfull[wg][s]);
      stamp(5);
    }
  }
  // the groups still in the stages (at most two): oldest first
  if (nmy >= 2) {
    epilogue(nmy - 2, q0);
    epilogue(nmy - 1, q1);
  } else if (nmy == 1) {
    epilogue(0, q0);
  }

  if (P.trace && tid == 0) P.trace[4 * blockIdx.x + 2] = bg_now();
  // ---- the two warpgroups' sums, in a fixed order ------------------------
  float* ycomb = reinterpret_cast<float*>(bsm + lay.ycomb);
  if (wg == 1) {
#pragma unroll
    for (int t = 0; t < NT; t++) ycomb[row * NT + t] = y[t];
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {  // every tcgen05 access of the CTA is complete: free the columns
    tc::fence_after_sync();
    tc::tmem_dealloc(taddr, kBgTmemCols);
  }
  // the next launch's CTAs allocate tensor memory before their dependency
  // wait: release it before letting them start
  __syncthreads();
  pdl_launch_dependents();
  if (wg == 0) {
#pragma unroll
    for (int t = 0; t < NT; t++) y[t] += ycomb[row * NT + t];
  }
  const bool swig = P.epi == EPI_SWIGLU;
  if (wg == 0 && (P.ksplit > 1 || swig)) {
#pragma unroll
    for (int t = 0; t < NT; t++)
      P.part[((size_t)split * NT + t) * P.rows_total + grow0 + row] = y[t];
  }
  const uint32_t nb_half = P.row_start[1] / kBgRows;  // SwiGLU: blocks of the gate half
  const bool partial = P.ksplit > 1 || swig;
  if (partial) {
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const uint32_t ci = swig ? (blk < nb_half ? blk : blk - nb_half) : blk;
      const uint32_t expect = swig ? 2u * P.ksplit : P.ksplit;
      const uint32_t prev = atomicAdd(&P.counters[ci], 1u);
      s_last = prev == expect - 1u;
      if (s_last) P.counters[ci] = 0u;
    }
    __syncthreads();
    if (!s_last) {
      if (P.trace && tid == 0) P.trace[4 * blockIdx.x + 3] = bg_now();
      return;
    }
    __threadfence();
  }
  if (P.trace && tid == 0) P.trace[4 * blockIdx.x + 3] = bg_now();
  if (wg != 0) return;
  // ---- epilogue of the block's rows (thread = row) -----------------------
  if (swig) {
    const uint32_t gb = (blk < nb_half ? blk : blk - nb_half) * kBgRows + row;  // gate row
    const uint32_t F = P.row_start[1];
#pragma unroll
    for (int t = 0; t < NT; t++) {
      float g = 0.f, u = 0.f;
      for (uint32_t j = 0; j < P.ksplit; j++) {
        g += __ldcg(P.part + ((size_t)j * NT + t) * P.rows_total + gb);
        u += __ldcg(P.part + ((size_t)j * NT + t) * P.rows_total + F + gb);
      }
      P.out[0][(size_t)t * P.out_stride + gb] = silu_ref(g) * u;
    }
    return;
  }
  if (P.ksplit > 1) {
#pragma unroll
    for (int t = 0; t < NT; t++) {
      float v = 0.f;
      for (uint32_t j = 0; j < P.ksplit; j++) v += __ldcg(P.part + ((size_t)j * NT + t) * P.rows_total + grow0 + row);
      y[t] = v;
    }
  }
  const uint32_t lr = lrow0 + row;
  float* o = P.out[seg];
  if (P.epi == EPI_STORE) {
    const float b = S.bias ? S.bias[lr] : 0.f;
#pragma unroll
    for (int t = 0; t < NT; t++) o[(size_t)t * P.out_stride + lr] = y[t] + b;
  } else if (P.epi == EPI_ACCUM) {
    bool ok = true;
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const float v = o[(size_t)t * P.out_stride + lr] + y[t];
      o[(size_t)t * P.out_stride + lr] = v;
      ok = ok && fabsf(v) <= 1e18f;
      y[t] = v;
    }
    if (!ok) atomicExch(P.bad, 1);
    if (P.ssq_out) {  // the block's sums of squares per token, in a fixed order
      float* red = s_red;  // [4 warps][NT]
#pragma unroll
      for (int t = 0; t < NT; t++) {
        const float q = warp_sum(y[t] * y[t]);
        if (L == 0) red[(warp & 3u) * NT + t] = q;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (row < (uint32_t)NT)
        P.ssq_out[blk * NT + row] = ((red[row] + red[NT + row]) + red[2 * NT + row]) + red[3 * NT + row];
    }
  } else {  // EPI_LOGITS
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const float v = y[t];
      o[(size_t)t * P.out_stride + lr] = v;
      unsigned long long k = isnan(v) ? 0ull : argmax_key(v, lr);
      uint32_t f = isfinite(v) ? 1u : 0u;
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1) {
        const unsigned long long ok2 = __shfl_xor_sync(0xffffffffu, k, sh);
        k = ok2 > k ? ok2 : k;
        f &= __shfl_xor_sync(0xffffffffu, f, sh);
      }
      if (L == 0) {
        if (k) atomicMax(&P.best[t], k);
        if (!f) atomicAnd(&P.finite[t], 0u);
      }
    }
  }
}

}  // namespace chpe
