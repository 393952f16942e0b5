// attention.cuh -- GQA decode attention over the FP16 KV cache.
//
// Restates the forwardDecode attention block (chpe_engine.zig:1688-1734):
// NeoX rotate-half RoPE on q and k (applyRope, :195-216), append k/v at
// `pos`, then per query head softmax(q.k * 1/sqrt(hd)) over t <= pos and the
// weighted sum of v.  The cache holds FP16 K and V, paged (below).
//
// One CTA per (kv head, split of the positions).  A CTA stages its positions
// in tiles of ATT_TT rows: every thread issues its 16-byte K and V loads of
// the tile at once into shared memory, then warp g (query head kv*G + g)
// scores the tile from shared memory, lane per position, and folds it into an
// online softmax.  The last CTA of a kv head (atomic arrival counter, reset by
// that CTA) merges the splits: lanes over splits for the max and the sum,
// lanes over head_dim for the weighted values.
#pragma once
#include <cstdlib>

#include "device_common.cuh"

namespace chpe {

struct AttnLaunch {
  const float* q;       // [H*HD] un-rotated
  const float* k;       // [KV*HD] un-rotated
  const float* v;       // [KV*HD]
  __half* kc;           // this layer's K cache
  __half* vc;           // this layer's V cache
  float* out;           // [H*HD]
  float* part;          // [KV][nsplit][G][HD + 4]: values, m, l, pad (16-byte records)
  uint32_t* counters;   // [KV], zero between steps
  const float* inv_freq;// [HD/2]
  StepState* st;
  int32_t H, KV, HD, nsplit;  // H, KV: this rank's heads (all of them on one GPU)
  int32_t max_seq;      // cache capacity; a step at pos >= max_seq is skipped
  const uint32_t* pages;  // page table (logical page -> physical page), or nullptr: contiguous
  int32_t page_shift;   // log2(positions per page)
  uint32_t n_pages;     // physical pages in this layer's pool (entries beyond read page 0)
  // Batched steps: token z = blockIdx.z sits at position st->pos + z, its
  // q / out / partials / counters offset by these strides, and the K/V rows
  // of every position it attends to (its own included) are already in the
  // cache (rope_append_kernel), so nothing is appended here.
  int32_t batched;
  uint32_t q_tok, out_tok, part_tok;
  TpLink tp;            // tensor parallel: out lies in the exchange region
};

// Cache row of position t: the physical row in the layer's pool.
CHPE_DEV size_t kv_cache_row(const AttnLaunch& P, int t) {
  if (!P.pages) return (size_t)t;
  uint32_t pg = P.pages[t >> P.page_shift];
  if (pg >= P.n_pages) pg = 0;  // an unmapped entry never addresses outside the pool
  return ((size_t)pg << P.page_shift) + (size_t)(t & ((1 << P.page_shift) - 1));
}

constexpr int ATT_TT = 32;  // positions per staged tile
// Splits of the positions per kv head: between 16 and 64, about two CTAs per
// SM over the kv heads a GPU holds (a CTA needs 23-45 KB of shared memory and
// 256 threads, so two are resident).  The merge keeps one weight per split in
// two registers per lane, so at most 64.
constexpr int kAttnSplits = 16;
constexpr int kAttnMaxSplits = 64;
static_assert(kAttnMaxSplits <= 64, "attention merge holds at most 64 split weights");
inline int attn_splits(int num_sms, int kv_heads, int max_seq) {
  // CHPE_ATTN_SPLITS=n (1..64) fixes the count (measurements)
  if (const char* e = getenv("CHPE_ATTN_SPLITS")) {
    const int f = atoi(e);
    if (f >= 1 && f <= kAttnMaxSplits) return f;
  }
  int n = 2 * num_sms / (kv_heads > 0 ? kv_heads : 1);
  const int tiles = (max_seq + ATT_TT - 1) / ATT_TT;  // more splits than tiles only idle
  if (n > tiles) n = tiles;
  return n < kAttnSplits ? kAttnSplits : (n > kAttnMaxSplits ? kAttnMaxSplits : n);
}

// Returns true on the CTA that reports this kv head to the other ranks: the
// one that merged the splits (and wrote the head's outputs), or split 0 when
// the step is skipped.
template <int HD>
CHPE_DEV bool attention_body(const AttnLaunch& P);

template <int HD>
__global__ void __launch_bounds__(256, 2) attention_kernel(const __grid_constant__ AttnLaunch P) {
  const bool reporter = attention_body<HD>(P);
  if (P.tp.world > 1 && reporter) {  // one arrival per kv head, after its outputs
    __syncthreads();
    if (threadIdx.x == 0) tp_signal(P.tp, P.tp.signal_sig);
  }
}

template <int HD>
CHPE_DEV bool attention_body(const AttnLaunch& P) {
  constexpr int PER = HD / 32;     // head elements per lane
  constexpr int KPAD = HD + 8;     // padded shared V row (halves, 16-byte rows)
  // K rows are read lane-per-row: a 4-byte padding makes the row stride an
  // odd number of words, so the 32 lanes of a score step hit 32 banks
  constexpr int KPADK = HD + 2;
  const int G = P.H / P.KV;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, L = threadIdx.x & 31;
  __shared__ float qs[8][HD];
  __shared__ float kn[HD], vn[HD];
  __shared__ __align__(16) __half ks[ATT_TT][KPADK];
  __shared__ __align__(16) __half vs[ATT_TT][KPAD];
  __shared__ float ps[8][ATT_TT];
  __shared__ int last_flag;

  // Single-token steps start before the dependency wait: the step's position
  // is set before the step begins, and the rows of the positions before it
  // are in the cache from earlier steps (the page table from the host), so
  // the first tile's K/V loads are in flight while the QKV projection
  // finishes.  Batched steps wait first: their candidates' rows come from the
  // preceding rope_append_kernel.
  if (P.batched) pdl_wait();
  const int tok = P.batched ? (int)blockIdx.z : 0;
  const int pos = P.st->pos + tok;
  if (pos < 0 || pos >= P.max_seq) {  // the host never schedules this
    if (!P.batched) pdl_wait();
    return blockIdx.x == 0;
  }
  const float pf = (float)pos;
  float* const part_base = P.part + (size_t)tok * P.part_tok;
  uint32_t* const counters = P.counters + (size_t)tok * P.KV;
  const int n = pos + 1;
  // at least one full tile per split: short contexts use fewer splits (the
  // rest find an empty range and only report -inf to the merge)
  int chunk = (n + P.nsplit - 1) / P.nsplit;
  if (chunk < ATT_TT) chunk = ATT_TT;
  const int t0 = split * chunk, t1 = min(n, t0 + chunk);

  constexpr int VPR = HD / 8;                 // 16-byte vectors per row
  constexpr int MAXV = ATT_TT * VPR / 128;    // vectors per thread (launched with >= 128 threads)
  // The next tile's K/V rows are loaded into registers while the current one
  // is scored from shared memory.  This step's own row (single-token steps)
  // comes from the values computed below, filled in by `own`.
  uint4 kr[MAXV], vr[MAXV];
  auto fetch = [&](int tb) {
    const int nt = min(ATT_TT, t1 - tb);
#pragma unroll
    for (int u = 0; u < MAXV; u++) {
      const int i = threadIdx.x + u * blockDim.x;
      if (i >= nt * VPR) continue;
      const int r = i / VPR, c8 = (i % VPR) * 8, t = tb + r;
      if (t == pos && !P.batched) continue;
      const size_t off = (kv_cache_row(P, t) * P.KV + kvh) * HD + c8;
      kr[u] = *reinterpret_cast<const uint4*>(P.kc + off);
      vr[u] = *reinterpret_cast<const uint4*>(P.vc + off);
    }
  };
  if (t0 < t1) fetch(t0);
  // RoPE angles of this lane's pairs i = L + 32 j (applyRope: cos/sin of pos * inv_freq[i])
  constexpr int NJ = (HD / 2 + 31) / 32;
  float rc[NJ], rs[NJ];
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int i = L + 32 * j;
    const float th = i < HD / 2 ? pf * P.inv_freq[i] : 0.f;
    rc[j] = cosf(th);
    rs[j] = sinf(th);
  }
  if (!P.batched) pdl_wait();
  if (P.st->stop) return blockIdx.x == 0;

  // RoPE on this warp's query head, on the new key; copy of the new value.
  if (warp < G) {
    const float* qh = P.q + (size_t)tok * P.q_tok + (size_t)(kvh * G + warp) * HD;
#pragma unroll
    for (int j = 0; j < NJ; j++) {
      const int i = L + 32 * j;
      if (i >= HD / 2) break;
      const float x0 = qh[i], x1 = qh[i + HD / 2];
      qs[warp][i] = x0 * rc[j] - x1 * rs[j];
      qs[warp][i + HD / 2] = x0 * rs[j] + x1 * rc[j];
    }
  }
  if (!P.batched && (int)threadIdx.x < HD / 2) {  // pair i = threadIdx.x = L + 32 warp
    const float* kh = P.k + (size_t)kvh * HD;
    float c = 0.f, s = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; j++)
      if (j == warp) {
        c = rc[j];
        s = rs[j];
      }
    const int i = threadIdx.x;
    const float x0 = kh[i], x1 = kh[i + HD / 2];
    kn[i] = x0 * c - x1 * s;
    kn[i + HD / 2] = x0 * s + x1 * c;
  }
  for (int i = threadIdx.x; i < HD && !P.batched; i += blockDim.x) vn[i] = P.v[(size_t)kvh * HD + i];
  __syncthreads();
  if (split == 0 && !P.batched) {
    size_t base = (kv_cache_row(P, pos) * P.KV + kvh) * HD;
    for (int i = threadIdx.x; i < HD; i += blockDim.x) {
      P.kc[base + i] = __float2half_rn(kn[i]);
      P.vc[base + i] = __float2half_rn(vn[i]);
    }
  }
  pdl_launch_dependents();

  const float scale = 1.0f / sqrtf((float)HD);
  float m = -INFINITY, l = 0.f, acc[PER];
#pragma unroll
  for (int e = 0; e < PER; e++) acc[e] = 0.f;
  // this step's entry, from the values just computed (rounded as the cache holds them)
  auto own = [&](int tb) {
    const int nt = min(ATT_TT, t1 - tb);
#pragma unroll
    for (int u = 0; u < MAXV; u++) {
      const int i = threadIdx.x + u * blockDim.x;
      if (i >= nt * VPR) continue;
      const int r = i / VPR, c8 = (i % VPR) * 8, t = tb + r;
      if (t != pos || P.batched) continue;
      __half2 hk[4], hv[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        hk[e] = __floats2half2_rn(kn[c8 + 2 * e], kn[c8 + 2 * e + 1]);
        hv[e] = __floats2half2_rn(vn[c8 + 2 * e], vn[c8 + 2 * e + 1]);
      }
      kr[u] = *reinterpret_cast<uint4*>(hk);
      vr[u] = *reinterpret_cast<uint4*>(hv);
    }
  };
  if (t0 < t1) own(t0);
  for (int tb = t0; tb < t1; tb += ATT_TT) {
    const int nt = min(ATT_TT, t1 - tb);
    __syncthreads();  // previous tile consumed
#pragma unroll
    for (int u = 0; u < MAXV; u++) {
      const int i = threadIdx.x + u * blockDim.x;
      if (i >= nt * VPR) continue;
      const int r = i / VPR, c8 = (i % VPR) * 8;
      {
        uint32_t* kd = reinterpret_cast<uint32_t*>(&ks[r][c8]);  // 4-byte aligned rows
        kd[0] = kr[u].x;
        kd[1] = kr[u].y;
        kd[2] = kr[u].z;
        kd[3] = kr[u].w;
      }
      *reinterpret_cast<uint4*>(&vs[r][c8]) = vr[u];
    }
    if (tb + ATT_TT < t1) {
      fetch(tb + ATT_TT);
      own(tb + ATT_TT);
    }
    __syncthreads();
    if (warp < G) {
      float sc = -INFINITY;  // lane = tile row
      if (L < nt) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};  // four independent chains
#pragma unroll 4
        for (int e = 0; e < HD; e += 8) {
#pragma unroll
          for (int h = 0; h < 4; h++) {
            const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(&ks[L][e + 2 * h]));
            d[h] = fmaf(qs[warp][e + 2 * h], kf.x, d[h]);
            d[h] = fmaf(qs[warp][e + 2 * h + 1], kf.y, d[h]);
          }
        }
        sc = ((d[0] + d[1]) + (d[2] + d[3])) * scale;
      }
      const float tmax = warp_max(sc);
      const float mn = fmaxf(m, tmax);
      const float p = (L < nt) ? expf(sc - mn) : 0.f;
      const float corr = expf(m - mn);
      l = l * corr + warp_sum(p);
      ps[warp][L] = p;
      __syncwarp();
#pragma unroll
      for (int e = 0; e < PER; e++) acc[e] *= corr;
      for (int r = 0; r < nt; r++) {
        const float pr = ps[warp][r];
        // this lane's PER contiguous dims: 8-byte shared loads of 4 halves
#pragma unroll
        for (int e4 = 0; e4 < PER; e4 += 4) {
          const uint2 hv = *reinterpret_cast<const uint2*>(&vs[r][PER * L + e4]);
          const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
          const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
          acc[e4] = fmaf(pr, v01.x, acc[e4]);
          acc[e4 + 1] = fmaf(pr, v01.y, acc[e4 + 1]);
          acc[e4 + 2] = fmaf(pr, v23.x, acc[e4 + 2]);
          acc[e4 + 3] = fmaf(pr, v23.y, acc[e4 + 3]);
        }
      }
      m = mn;
      __syncwarp();
    }
  }
  constexpr int PS = HD + 4;  // partial record: HD values, m, l, pad (16-byte records)
  if (warp < G) {
    float* dst = part_base + (((size_t)kvh * P.nsplit + split) * G + warp) * PS;
#pragma unroll
    for (int e4 = 0; e4 < PER; e4 += 4)
      *reinterpret_cast<float4*>(dst + PER * L + e4) = make_float4(acc[e4], acc[e4 + 1], acc[e4 + 2], acc[e4 + 3]);
    if (L == 0) *reinterpret_cast<float2*>(dst + HD) = make_float2(m, l);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned prev = atomicAdd(&counters[kvh], 1u);
    last_flag = (prev == (unsigned)P.nsplit - 1);
  }
  __syncthreads();
  if (!last_flag) return false;
  __threadfence();
  if (warp < G) {
    const float* src = part_base + ((size_t)kvh * P.nsplit * G + warp) * PS;
    const size_t sstride = (size_t)G * PS;
    // (m, l) of splits L and L+32 in one round of loads
    float2 ml[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int s = L + 32 * h;
      ml[h] = s < P.nsplit ? __ldcg(reinterpret_cast<const float2*>(src + s * sstride + HD))
                           : make_float2(-INFINITY, 0.f);
    }
    const float M = warp_max(fmaxf(ml[0].x, ml[1].x));
    float wl[2], den = 0.f;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      wl[h] = ml[h].x == -INFINITY ? 0.f : expf(ml[h].x - M);
      den = fmaf(ml[h].y, wl[h], den);
    }
    den = warp_sum(den);
    // the values in batches of MB splits, every 16-byte load of a batch
    // issued before any is used
    constexpr int MB = PER == 4 ? 16 : 8;
    float o[PER];
#pragma unroll
    for (int e = 0; e < PER; e++) o[e] = 0.f;
    for (int s0 = 0; s0 < P.nsplit; s0 += MB) {
      float4 a[MB][PER / 4];
#pragma unroll
      for (int b = 0; b < MB; b++) {
        const int s = s0 + b;
#pragma unroll
        for (int e4 = 0; e4 < PER / 4; e4++)
          a[b][e4] = s < P.nsplit ? __ldcg(reinterpret_cast<const float4*>(src + s * sstride + PER * L + 4 * e4))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int b = 0; b < MB; b++) {
        const int s = s0 + b;
        const float w = __shfl_sync(0xffffffffu, (s & 32) ? wl[1] : wl[0], s & 31);
#pragma unroll
        for (int e4 = 0; e4 < PER / 4; e4++) {
          o[4 * e4] = fmaf(a[b][e4].x, w, o[4 * e4]);
          o[4 * e4 + 1] = fmaf(a[b][e4].y, w, o[4 * e4 + 1]);
          o[4 * e4 + 2] = fmaf(a[b][e4].z, w, o[4 * e4 + 2]);
          o[4 * e4 + 3] = fmaf(a[b][e4].w, w, o[4 * e4 + 3]);
        }
      }
    }
    const float inv = 1.0f / den;
    float* outp = P.out + (size_t)tok * P.out_tok + (size_t)(kvh * G + warp) * HD;
#pragma unroll
    for (int e = 0; e < PER; e++) tp_put(P.tp, outp, PER * L + e, o[e] * inv);
  }
  if (threadIdx.x == 0) counters[kvh] = 0;
  return true;
}

}  // namespace chpe
