// deltanet.cu -- one decode step of a Qwen3.5 Gated DeltaNet (linear
// attention) layer after its input projections, as a per-value-head kernel.
//
// The reference engine runs the 9B's linear layers as GQA and has no such
// function; the recurrence is the gated delta rule (Yang, Kautz, Hatamizadeh,
// ICLR 2025) wired as Qwen3.5 wires it for one cached token:
//   conv:   u[c] = silu(w[c][0] h[t-3] + w[c][1] h[t-2] + w[c][2] h[t-1] + w[c][3] x[c]),
//           the inputs of positions p kept in a 4-slot circular history (slot p % 4)
//   split:  q = u[0, nk*dk), k = u[nk*dk, 2*nk*dk), v = u[2*nk*dk, ..)
//   gates:  beta = sigmoid(b[h]), decay = exp(-exp(A_log[h]) * softplus(a[h] + dt_bias[h]))
//   norms:  q, k of the key head h / (nv/nk) scaled by 1/sqrt(sum sq + 1e-6); q /= sqrt(dk)
//   state:  S = decay * S;  m = S^T k;  d = (v - m) * beta;  S += k d^T;  o = S^T q
//   output: o / sqrt(mean(o^2) + eps) * norm_w * silu(z)
// with S stored per value head as [j][i] (value j, key i, 128 x 128 f32).
//
// One CTA per value head, 512 threads.  Threads first compute the conv of the
// head's 384 channels (its key head's q and k, its own v); every CTA that
// shares a key head computes the same q/k values and writes the same inputs
// into history slot t % 4, which no CTA reads during this step.  Then warp w
// owns state columns j = 8w..8w+7: each lane keeps keys 4L..4L+3 of every
// column (all eight 16-byte loads issued first), and each column takes two
// warp reductions (S^T k, then S^T q after the update).  The gated RMSNorm
// closes the head.  State traffic: 128 KiB read + written per value head.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/chpe.h"
#include "device_common.cuh"

namespace {

constexpr int kDk = 128, kDv = 128, kThreads = 512;

struct DeltaNetLaunch {
  const float *mixed, *z, *a, *b, *conv_w;
  float* hist;
  uint32_t t;
  const float *a_log, *dt_bias, *norm_w;
  float* state;
  float* out;
  uint32_t nk, nv;
  float eps;
};

__device__ __forceinline__ float sigmoid_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

__global__ void __launch_bounds__(kThreads, 1) deltanet_step_kernel(const DeltaNetLaunch P) {
  const uint32_t h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, L = tid & 31u;
  const uint32_t kh = h / (P.nv / P.nk);
  const uint32_t conv_dim = 2u * P.nk * kDk + P.nv * kDv;
  __shared__ float qs[kDk], ks[kDk], vs[kDv], os[kDv];
  __shared__ float s_qn, s_kn, s_on;

  // ---- conv of this head's channels: q (0..127), k (128..255), v (256..383)
  if (tid < 3u * 128u) {
    const uint32_t part = tid >> 7, i = tid & 127u;
    const uint32_t c = part == 0 ? kh * kDk + i : part == 1 ? P.nk * kDk + kh * kDk + i
                                                            : 2u * P.nk * kDk + h * kDv + i;
    const uint32_t p3 = (P.t + 1u) & 3u, p2 = (P.t + 2u) & 3u, p1 = (P.t + 3u) & 3u, p0 = P.t & 3u;
    const float4 w = *reinterpret_cast<const float4*>(P.conv_w + 4u * c);
    const float x = P.mixed[c];
    float acc = w.x * P.hist[(size_t)p3 * conv_dim + c];
    acc += w.y * P.hist[(size_t)p2 * conv_dim + c];
    acc += w.z * P.hist[(size_t)p1 * conv_dim + c];
    acc += w.w * x;
    const float u = acc * sigmoid_(acc);
    P.hist[(size_t)p0 * conv_dim + c] = x;  // slot of position t (not read this step)
    if (part == 0) qs[i] = u;
    else if (part == 1) ks[i] = u;
    else vs[i] = u;
  }
  __syncthreads();
  // ---- l2 norms of q and k (warps 0 and 1), gates
  if (warp < 2) {
    const float* src = warp == 0 ? qs : ks;
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; e++) ss += src[L + 32 * e] * src[L + 32 * e];
    ss = warp_sum(ss);
    if (L == 0) {
      if (warp == 0) s_qn = 1.0f / sqrtf(ss + 1e-6f) * (1.0f / sqrtf((float)kDk));
      else s_kn = 1.0f / sqrtf(ss + 1e-6f);
    }
  }
  __syncthreads();
  const float beta = sigmoid_(P.b[h]);
  const float decay = expf(-expf(P.a_log[h]) * softplus_(P.a[h] + P.dt_bias[h]));
  float q4[4], k4[4];
#pragma unroll
  for (int e = 0; e < 4; e++) {
    q4[e] = qs[4 * L + e] * s_qn;
    k4[e] = ks[4 * L + e] * s_kn;
  }
  // ---- state columns j = 8*warp .. 8*warp+7
  float* S = P.state + (size_t)h * kDv * kDk;
  float4 col[8];
#pragma unroll
  for (int c = 0; c < 8; c++) col[c] = *reinterpret_cast<const float4*>(S + (size_t)(8 * warp + c) * kDk + 4 * L);
#pragma unroll
  for (int c = 0; c < 8; c++) {
    const uint32_t j = 8 * warp + c;
    float4 s = col[c];
    s.x *= decay;
    s.y *= decay;
    s.z *= decay;
    s.w *= decay;
    float m = s.x * k4[0];
    m += s.y * k4[1];
    m += s.z * k4[2];
    m += s.w * k4[3];
    m = warp_sum(m);
    const float d = (vs[j] - m) * beta;
    s.x += k4[0] * d;
    s.y += k4[1] * d;
    s.z += k4[2] * d;
    s.w += k4[3] * d;
    float o = s.x * q4[0];
    o += s.y * q4[1];
    o += s.z * q4[2];
    o += s.w * q4[3];
    o = warp_sum(o);
    *reinterpret_cast<float4*>(S + (size_t)j * kDk + 4 * L) = s;
    if (L == 0) os[j] = o;
  }
  __syncthreads();
  // ---- gated RMSNorm of the head's 128 outputs
  if (warp == 0) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; e++) ss += os[L + 32 * e] * os[L + 32 * e];
    ss = warp_sum(ss);
    if (L == 0) s_on = 1.0f / sqrtf(ss / (float)kDv + P.eps);
  }
  __syncthreads();
  if (tid < (uint32_t)kDv) {
    const float zz = P.z[(size_t)h * kDv + tid];
    P.out[(size_t)h * kDv + tid] = os[tid] * s_on * P.norm_w[tid] * (zz * sigmoid_(zz));
  }
}

}  // namespace

extern "C" int chpe_deltanet_step(const float* mixed_qkv, const float* z, const float* a, const float* b,
                                  const float* conv_w, float* conv_hist, uint32_t t, const float* a_log,
                                  const float* dt_bias, const float* norm_w, float* state, float* out,
                                  uint32_t num_k_heads, uint32_t num_v_heads, uint32_t k_head_dim,
                                  uint32_t v_head_dim, float eps, void* stream) {
  if (!mixed_qkv || !z || !a || !b || !conv_w || !conv_hist || !a_log || !dt_bias || !norm_w || !state || !out)
    return -1;
  if (k_head_dim != (uint32_t)kDk || v_head_dim != (uint32_t)kDv) return -1;
  if (num_k_heads == 0 || num_v_heads == 0 || num_v_heads % num_k_heads != 0 || num_v_heads > 4096) return -1;
  if ((reinterpret_cast<uintptr_t>(conv_w) | reinterpret_cast<uintptr_t>(state)) & 15u) return -1;
  DeltaNetLaunch P{mixed_qkv, z, a, b, conv_w, conv_hist, t, a_log, dt_bias, norm_w, state, out,
                   num_k_heads, num_v_heads, eps};
  deltanet_step_kernel<<<num_v_heads, kThreads, 0, (cudaStream_t)stream>>>(P);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
