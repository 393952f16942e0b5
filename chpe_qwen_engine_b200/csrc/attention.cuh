// attention.cuh -- GQA decode attention over the FP16 KV cache.
//
// Restates the forwardDecode attention block (chpe_engine.zig:1688-1734):
// NeoX rotate-half RoPE on q and k (applyRope, :195-216), append k/v at
// `pos`, then per query head softmax(q.k * 1/sqrt(hd)) over t <= pos and the
// weighted sum of v.  Layout of the cache: [max_seq][kv_heads][head_dim] FP16
// per layer.  One CTA per (kv head, split of the positions); warp g handles
// query head kv*G + g with an online softmax; the last CTA of a kv head
// (atomic arrival counter, reset by that CTA) merges the splits.
#pragma once
#include "device_common.cuh"

namespace chpe {

struct AttnLaunch {
  const float* q;       // [H*HD] un-rotated
  const float* k;       // [KV*HD] un-rotated
  const float* v;       // [KV*HD]
  __half* kc;           // this layer's K cache
  __half* vc;           // this layer's V cache
  float* out;           // [H*HD]
  float* part;          // [KV][nsplit][G][HD + 2]
  uint32_t* counters;   // [KV], zero between steps
  const float* inv_freq;// [HD/2]
  StepState* st;
  int32_t H, KV, HD, nsplit;
  int32_t max_seq;      // cache capacity; a step at pos >= max_seq is skipped
};

template <int HD>
__global__ void __launch_bounds__(256) attention_kernel(const __grid_constant__ AttnLaunch P) {
  constexpr int PER = HD / 32;  // elements per lane
  const int G = P.H / P.KV;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, L = threadIdx.x & 31;
  __shared__ float qs[8][HD];
  __shared__ float kn[HD], vn[HD];
  __shared__ int last_flag;

  pdl_wait();
  if (P.st->stop) return;
  const int pos = P.st->pos;
  if (pos < 0 || pos >= P.max_seq) return;  // the host never schedules this
  const float pf = (float)pos;

  // RoPE on this warp's query head and (warp 0) on the new key.
  if (warp < G) {
    const float* qh = P.q + (size_t)(kvh * G + warp) * HD;
    for (int i = L; i < HD / 2; i += 32) {
      float th = pf * P.inv_freq[i];
      float c = cosf(th), s = sinf(th);
      float x0 = qh[i], x1 = qh[i + HD / 2];
      qs[warp][i] = x0 * c - x1 * s;
      qs[warp][i + HD / 2] = x0 * s + x1 * c;
    }
  }
  if (threadIdx.x < HD / 2) {
    int i = threadIdx.x;
    const float* kh = P.k + (size_t)kvh * HD;
    float th = pf * P.inv_freq[i];
    float c = cosf(th), s = sinf(th);
    float x0 = kh[i], x1 = kh[i + HD / 2];
    kn[i] = x0 * c - x1 * s;
    kn[i + HD / 2] = x0 * s + x1 * c;
  }
  for (int i = threadIdx.x; i < HD; i += blockDim.x) vn[i] = P.v[(size_t)kvh * HD + i];
  __syncthreads();
  if (split == 0) {
    size_t base = ((size_t)pos * P.KV + kvh) * HD;
    for (int i = threadIdx.x; i < HD; i += blockDim.x) {
      P.kc[base + i] = __float2half_rn(kn[i]);
      P.vc[base + i] = __float2half_rn(vn[i]);
    }
  }
  pdl_launch_dependents();

  const int n = pos + 1;
  const int chunk = (n + P.nsplit - 1) / P.nsplit;
  const int t0 = split * chunk, t1 = min(n, t0 + chunk);
  const float scale = 1.0f / sqrtf((float)HD);
  float m = -INFINITY, l = 0.f, acc[PER];
#pragma unroll
  for (int e = 0; e < PER; e++) acc[e] = 0.f;
  if (warp < G) {
    float qv[PER];
#pragma unroll
    for (int e = 0; e < PER; e++) qv[e] = qs[warp][L + 32 * e];
    for (int t = t0; t < t1; t++) {
      float kv[PER], vv[PER];
      if (t == pos) {
#pragma unroll
        for (int e = 0; e < PER; e++) { kv[e] = kn[L + 32 * e]; vv[e] = vn[L + 32 * e]; }
      } else {
        const __half* kr = P.kc + ((size_t)t * P.KV + kvh) * HD;
        const __half* vr = P.vc + ((size_t)t * P.KV + kvh) * HD;
#pragma unroll
        for (int e = 0; e < PER; e++) {
          kv[e] = __half2float(kr[L + 32 * e]);
          vv[e] = __half2float(vr[L + 32 * e]);
        }
      }
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < PER; e++) d = fmaf(qv[e], kv[e], d);
      float s = warp_sum(d) * scale;
      float mn = fmaxf(m, s);
      float corr = expf(m - mn), p = expf(s - mn);
      l = l * corr + p;
#pragma unroll
      for (int e = 0; e < PER; e++) acc[e] = fmaf(p, vv[e], acc[e] * corr);
      m = mn;
    }
    float* dst = P.part + (((size_t)kvh * P.nsplit + split) * G + warp) * (HD + 2);
#pragma unroll
    for (int e = 0; e < PER; e++) dst[L + 32 * e] = acc[e];
    if (L == 0) { dst[HD] = m; dst[HD + 1] = l; }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned prev = atomicAdd(&P.counters[kvh], 1u);
    last_flag = (prev == (unsigned)P.nsplit - 1);
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  if (warp < G) {
    const float* src = P.part + ((size_t)kvh * P.nsplit * G + warp) * (HD + 2);
    const size_t sstride = (size_t)G * (HD + 2);
    float M = -INFINITY;
    for (int s = 0; s < P.nsplit; s++) M = fmaxf(M, __ldcg(src + s * sstride + HD));
    float den = 0.f, o[PER];
#pragma unroll
    for (int e = 0; e < PER; e++) o[e] = 0.f;
    for (int s = 0; s < P.nsplit; s++) {
      const float* ps = src + s * sstride;
      float ms = __ldcg(ps + HD);
      if (ms == -INFINITY) continue;
      float w = expf(ms - M);
      den = fmaf(__ldcg(ps + HD + 1), w, den);
#pragma unroll
      for (int e = 0; e < PER; e++) o[e] = fmaf(__ldcg(ps + L + 32 * e), w, o[e]);
    }
    float inv = 1.0f / den;
    float* outp = P.out + (size_t)(kvh * G + warp) * HD;
#pragma unroll
    for (int e = 0; e < PER; e++) outp[L + 32 * e] = o[e] * inv;
  }
  if (threadIdx.x == 0) P.counters[kvh] = 0;
}

}  // namespace chpe
