/* deltanet_oracle.c -- CPU restatement of one decode step of a Gated DeltaNet
 * (linear-attention) layer as Qwen3.5 computes it.  TEST INFRASTRUCTURE: only
 * the tests call it, as the checker of the GPU kernel.
 *
 * The reference engine has no such function (its 9B layers run as GQA); the
 * recurrence is the published gated delta rule (Yang, Kautz, Hatamizadeh,
 * "Gated Delta Networks", ICLR 2025) with Qwen3.5's decode-step wiring, which
 * the installed transformers package implements in
 * transformers/models/qwen3_5/modeling_qwen3_5.py (Qwen3_5GatedDeltaNet with
 * torch_causal_conv1d_update, torch_recurrent_gated_delta_rule, l2norm and
 * Qwen3_5RMSNormGated).  tests/golden/gen_deltanet.py runs those functions on
 * seeded inputs and stores the outputs; tests/test_oracle_kats.py pins this
 * restatement against them.
 *
 * One token, after the input projections:
 *   conv:   u[c] = silu(w[c][0] h[t-3] + w[c][1] h[t-2] + w[c][2] h[t-1] + w[c][3] x[c])
 *           over the last three inputs of channel c (zeros before the sequence),
 *           kept in a 4-slot circular history (input of position p in slot p % 4)
 *   split:  q = u[0, nk*dk), k = u[nk*dk, 2*nk*dk), v = u[2*nk*dk, ..)
 *   gates:  beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias)
 *   norms:  q, k of each key head scaled by 1/sqrt(sum sq + 1e-6); q *= 1/sqrt(dk)
 *   state:  value head h uses key head h / (nv/nk);
 *           S = S * exp(g);  m = S^T k;  d = (v - m) * beta;  S += k d^T;  o = S^T q
 *   output: o * (1/sqrt(mean(o^2) + eps)) * norm_w * silu(z)   per value head
 * State layout here and on the GPU: S[h][j][i] (value index j, key index i).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

static float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
static float siluf_(float x) { return x * sigmoidf_(x); }
/* torch.nn.functional.softplus with beta 1, threshold 20 */
static float softplusf_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

void oracle_deltanet_step(const float *mixed_qkv, const float *z, const float *a, const float *b,
                          const float *conv_w, float *conv_hist, uint32_t t, const float *a_log,
                          const float *dt_bias, const float *norm_w, float *state, float *out,
                          uint32_t nk, uint32_t nv, uint32_t dk, uint32_t dv, float eps) {
  const size_t conv_dim = 2 * (size_t)nk * dk + (size_t)nv * dv;
  float u[2 * 16 * 256 + 64 * 256]; /* conv output, sized for <= 16 key / 64 value heads of 256 */
  if (conv_dim > sizeof(u) / sizeof(u[0]) || dk > 256 || dv > 256) return;
  /* circular history of 4 slots: the input of position p lives in slot p % 4;
   * a step reads the slots of t-3, t-2, t-1 and writes slot t % 4 */
  const uint32_t p3 = (t + 1u) % 4u, p2 = (t + 2u) % 4u, p1 = (t + 3u) % 4u, p0 = t % 4u;
  for (size_t c = 0; c < conv_dim; c++) {
    const float *w = conv_w + 4 * c;
    float acc = w[0] * conv_hist[(size_t)p3 * conv_dim + c];
    acc += w[1] * conv_hist[(size_t)p2 * conv_dim + c];
    acc += w[2] * conv_hist[(size_t)p1 * conv_dim + c];
    acc += w[3] * mixed_qkv[c];
    u[c] = siluf_(acc);
  }
  for (size_t c = 0; c < conv_dim; c++) conv_hist[(size_t)p0 * conv_dim + c] = mixed_qkv[c];
  const float *qa = u, *ka = u + (size_t)nk * dk, *va = u + 2 * (size_t)nk * dk;
  const uint32_t rep = nv / nk;
  const float qscale = 1.0f / sqrtf((float)dk);
  for (uint32_t h = 0; h < nv; h++) {
    const uint32_t kh = h / rep;
    float q[256], k[256], o[256];
    float sq = 0.f, sk = 0.f;
    for (uint32_t i = 0; i < dk; i++) {
      sq += qa[(size_t)kh * dk + i] * qa[(size_t)kh * dk + i];
      sk += ka[(size_t)kh * dk + i] * ka[(size_t)kh * dk + i];
    }
    const float iq = 1.0f / sqrtf(sq + 1e-6f), ik = 1.0f / sqrtf(sk + 1e-6f);
    for (uint32_t i = 0; i < dk; i++) {
      q[i] = qa[(size_t)kh * dk + i] * iq * qscale;
      k[i] = ka[(size_t)kh * dk + i] * ik;
    }
    const float beta = sigmoidf_(b[h]);
    const float decay = expf(-expf(a_log[h]) * softplusf_(a[h] + dt_bias[h]));
    float *S = state + (size_t)h * dv * dk;
    for (uint32_t j = 0; j < dv; j++) {
      float *col = S + (size_t)j * dk;
      float m = 0.f;
      for (uint32_t i = 0; i < dk; i++) {
        col[i] *= decay;
        m += col[i] * k[i];
      }
      const float d = (va[(size_t)h * dv + j] - m) * beta;
      float acc = 0.f;
      for (uint32_t i = 0; i < dk; i++) {
        col[i] += k[i] * d;
        acc += col[i] * q[i];
      }
      o[j] = acc;
    }
    float ss = 0.f;
    for (uint32_t j = 0; j < dv; j++) ss += o[j] * o[j];
    const float inv = 1.0f / sqrtf(ss / (float)dv + eps);
    for (uint32_t j = 0; j < dv; j++)
      out[(size_t)h * dv + j] = o[j] * inv * norm_w[j] * siluf_(z[(size_t)h * dv + j]);
  }
}
