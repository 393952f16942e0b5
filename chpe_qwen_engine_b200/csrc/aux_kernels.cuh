// aux_kernels.cuh -- embedding lookup, stand-alone RMSNorm / SwiGLU / argmax
// for decomposed plans, the synthetic-pattern GEMV and the dequant probe.
// The kernels here and in gemv.cuh have internal linkage: every translation
// unit that launches one holds its own copy.
#pragma once
#include "device_common.cuh"
#include "gemv.cuh"

namespace chpe {

enum EmbedMode : int32_t { EMB_PATTERN = 0, EMB_RAW_F16 = 1, EMB_RAW_BF16 = 2, EMB_RAW_I8 = 3, EMB_CELL = 4 };

struct EmbedLaunch {
  const uint8_t* arc;
  uint64_t record_count;
  uint64_t stride;      // bytes between tiles
  uint64_t prefix;      // code area offset inside a record
  int32_t mode;
  uint32_t D;
  float* hidden;
  StepState* st;
  const StepResult* res;
  int32_t use_state;    // 0: token comes from `token` (probe), 1: from the step state,
                        // 2: from tokens[blockIdx.y] into row blockIdx.y of hidden ([y][D])
  uint32_t token;
  const int32_t* tokens;
};

CHPE_DEV float embed_pattern(uint32_t i, uint32_t tok) {
  return 0.05f * (float)((int32_t)((i + tok) % 17u) - 8);
}

// unpackEmbedRow (chpe_engine.zig:1491-1552) and unpackEmbedRowCell
// (:1288-1394); each CTA owns blockDim.x columns of the hidden vector.
static __global__ void embed_kernel(const __grid_constant__ EmbedLaunch P) {
  pdl_wait();
  const uint32_t tok = P.use_state == 2 ? (uint32_t)P.tokens[blockIdx.y]
                       : P.use_state ? (P.st->feed_argmax ? P.res->argmax_token : (uint32_t)P.st->token)
                                     : P.token;
  if (P.use_state == 1 && blockIdx.x == 0 && threadIdx.x == 0) P.st->stop = 0;
  const uint32_t D = P.D;
  float* const hidden = P.hidden + (P.use_state == 2 ? (size_t)blockIdx.y * D : 0);
  const uint32_t c0 = blockIdx.x * blockDim.x, c = c0 + threadIdx.x;
  int mode = P.mode;
  uint64_t tile = 0, row = 0;
  if (mode == EMB_RAW_F16 || mode == EMB_RAW_BF16 || mode == EMB_RAW_I8) {
    uint32_t rpt = (mode == EMB_RAW_I8 ? 16384u : 8192u) / D;
    if (rpt == 0) mode = EMB_PATTERN;
    else { tile = tok / rpt; row = tok % rpt; if (tile >= P.record_count) mode = EMB_PATTERN; }
  } else if (mode == EMB_CELL) {
    tile = tok / 16u; row = tok % 16u;  // for every D (the reference's indexing)
    if (tile >= P.record_count) mode = EMB_PATTERN;
  }
  const uint8_t* code = P.arc + 4096 + tile * P.stride + P.prefix;
  if (mode == EMB_PATTERN) {
    if (c < D) hidden[c] = embed_pattern(c, tok);
    return;
  }
  if (mode == EMB_RAW_F16) {
    if (c < D) hidden[c] = ld_f16(code + 2 * (row * D + c));
    return;
  }
  if (mode == EMB_RAW_BF16) {
    if (c < D) hidden[c] = bf2f(ld_u16(code + 2 * (row * D + c)));
    return;
  }
  if (mode == EMB_RAW_I8) {
    if (c < D) hidden[c] = (float)(int8_t)code[row * D + c] * 0.00373708f;
    return;
  }
  const uint8_t* pl = code + 16384;
  const uint32_t qb = pl[20];
  const uint64_t flags = *reinterpret_cast<const uint64_t*>(pl + 24);
  const bool g128 = (flags & 1u) != 0;
  const uint32_t ng = D / 128;
  bool replace = false;
  if (qb == 8) {
    if (row >= 8) return;  // the row is left as it was
    if (c < ng * 128)
      hidden[c] = (float)(int8_t)code[row * D + c] * ld_f16(pl + 48 + 2 * (row * ng + c / 128));
    return;
  } else if (qb == 2) {
    if (row >= 16) return;
    const float CB[4] = {0.f, 1.f, -2.f, -1.f};
    if (c < ng * 128) {
      uint8_t b = code[row * (D / 4) + c / 4];
      hidden[c] = CB[(b >> (2 * (c & 3))) & 3] * ld_f16(pl + 48 + 2 * (row * ng + c / 128));
    }
    replace = g128;
  } else if (g128 || qb == 4) {
    if (row >= 16) return;
    if (c < ng * 128) {
      uint8_t b = code[row * (D / 2) + c / 2];
      float q = (float)((c & 1) ? (b >> 4) & 15 : b & 15);
      hidden[c] = (q - 8.0f) * ld_f16(pl + 48 + 2 * (row * ng + c / 128));
    }
    replace = g128;
  } else {
    if (c < D) {
      uint8_t b = code[row * (D / 2) + c / 2];
      float q = (float)((c & 1) ? (b >> 4) & 15 : b & 15);
      hidden[c] = __fadd_rn(__fmul_rn(q - 8.0f, ld_f32(pl + 32)), ld_f32(pl + 36));
    }
    return;
  }
  if (replace) {
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int k = 0; k < 8; k++) {
        uint32_t col = ld_u16(pl + 816 + 2 * k);
        if (col < D && col >= c0 && col < c0 + blockDim.x)
          hidden[col] = ld_f16(pl + 560 + 2 * (row * 8 + k));
      }
    }
  }
}

// Stand-alone RMSNorm for decomposed plans: every CTA computes the sum of
// squares, CTA b writes its slice of y.  Carries the end-of-layer check.
struct NormLaunch {
  const float* x;
  const float* gamma;
  float* y;
  uint32_t n;
  float eps;
  int32_t check_layer;
  StepState* st;
  int32_t ignore_stop;
};
static __global__ void __launch_bounds__(256) rmsnorm_kernel(const __grid_constant__ NormLaunch P) {
  __shared__ float red[8];
  pdl_wait();
  if (!P.ignore_stop && P.st->stop) return;
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < P.n; i += 256) ss += P.x[i] * P.x[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < 8; w++) tot += red[w];
  if (P.check_layer >= 0) {
    int l = P.check_layer;
    bool cond = l < 3 || (l >= 8 && l <= 16) || !isfinite(P.x[0]);
    if (cond && !isfinite(tot)) {
      if (blockIdx.x == 0 && threadIdx.x == 0) P.st->stop = 1;
      return;
    }
  }
  pdl_launch_dependents();
  const float inv = 1.0f / sqrtf(tot / (float)P.n + P.eps);
  uint32_t i = blockIdx.x * 256 + threadIdx.x;
  if (i < P.n) P.y[i] = P.x[i] * inv * P.gamma[i];
}

struct SwigluLaunch {
  const float* g;
  const float* u;
  float* out;
  uint32_t n;
  StepState* st;
};
static __global__ void swiglu_kernel(const __grid_constant__ SwigluLaunch P) {
  pdl_wait();
  if (P.st->stop) return;
  uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < P.n) P.out[i] = silu_ref(P.g[i]) * P.u[i];
}

// gemvLinear on an invalid archive or past the last record
// (chpe_engine.zig:1411-1418).
struct PatternLaunch {
  float* y;
  uint32_t n;
  StepState* st;
};
static __global__ void pattern_kernel(const __grid_constant__ PatternLaunch P) {
  pdl_wait();
  if (P.st && P.st->stop) return;
  uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < P.n) P.y[r] = 0.01f * (float)((int32_t)(r % 13u) - 6);
}

// Argmax / finiteness / result for decomposed LM heads and synthetic logits.
struct ArgmaxLaunch {
  float* logits;
  uint32_t V;
  int32_t pattern;        // 1: logits are the reference's synthetic values
  const float* hidden;
  uint32_t D;
  StepState* st;
  StepResult* res;
  int32_t* gen_tokens;
  int32_t max_gen;
};
static __global__ void __launch_bounds__(256) argmax_kernel(const __grid_constant__ ArgmaxLaunch P) {
  __shared__ unsigned long long kb[8];
  __shared__ uint32_t kf[8];
  __shared__ int is_last;
  pdl_wait();
  unsigned long long best = 0ull;
  uint32_t fin = 1u;
  for (uint32_t v = blockIdx.x * 256 + threadIdx.x; v < P.V; v += gridDim.x * 256) {
    float d = P.pattern ? 0.001f * (float)((int32_t)(v % 13u) - 6) : P.logits[v];
    if (P.pattern) P.logits[v] = d;
    if (!isfinite(d)) fin = 0u;
    if (d > -1e30f) {
      unsigned long long k = argmax_key(d, v);
      best = k > best ? k : best;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
    fin &= __shfl_xor_sync(0xffffffffu, fin, o);
  }
  const int w = threadIdx.x >> 5, L = threadIdx.x & 31;
  if (L == 0) { kb[w] = best; kf[w] = fin; }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    uint32_t f = 1u;
    for (int i = 0; i < 8; i++) { b = kb[i] > b ? kb[i] : b; f &= kf[i]; }
    if (b) atomicMax(&P.st->best, b);
    if (!f) atomicAnd(&P.st->finite, 0u);
    __threadfence();
    is_last = atomicAdd(&P.st->done_ctas, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < P.D; i += 256) { float h = __ldcg(P.hidden + i); ss += h * h; }
  ss = warp_sum(ss);
  __shared__ float red[8];
  if (L == 0) red[w] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < 8; i++) tot += red[i];
    unsigned long long b = atomicAdd(&P.st->best, 0ull);
    StepResult R;
    R.argmax_token = b ? 0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull) : 0u;
    R.max_logit = b ? key_value(b) : -1e30f;
    R.token0_logit = __ldcg(P.logits);
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

// Dequantised weights of one cell exactly as the reference materialises them
// (gemvCellFlat's tile_weights for flat cells, the per-weight affine forms
// for row-tiled cells); products are kept unfused so values are bit-exact.
struct DequantLaunch {
  const uint8_t* cell_code;
  int32_t flat;
  float* out;
  uint32_t cap;
};
static __global__ void dequant_kernel(const __grid_constant__ DequantLaunch P) {
  const uint8_t* code = P.cell_code;
  const uint8_t* pl = code + 16384;
  const uint32_t qb = pl[20];
  const uint64_t flags = *reinterpret_cast<const uint64_t*>(pl + 24);
  const bool g128 = (flags & 1u) != 0;
  const float sc = ld_f32(pl + 32), bi = ld_f32(pl + 36);
  const uint32_t rows = *reinterpret_cast<const uint32_t*>(pl + 40);
  const uint32_t cols = *reinterpret_cast<const uint32_t*>(pl + 44);
  const float CB[4] = {0.f, 1.f, -2.f, -1.f};
  if (P.flat) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < 32768 && i < P.cap; i += gridDim.x * blockDim.x) {
      float w = 0.f;
      if (qb == 4) {
        uint8_t b = code[i / 2];
        float q = (float)((i & 1) ? (b >> 4) & 15 : b & 15) - 8.0f;
        w = g128 ? __fmul_rn(q, ld_f16(pl + 48 + 2 * (i / 128))) : __fadd_rn(__fmul_rn(q, sc), bi);
      } else if (qb == 2) {
        uint8_t b = code[i / 4];
        float cb = CB[(b >> (2 * (i & 3))) & 3];
        w = g128 ? __fmul_rn(cb, ld_f16(pl + 48 + 2 * (i / 128))) : __fadd_rn(__fmul_rn(cb, sc), bi);
      }
      if (qb == 4 || qb == 2) {
        uint32_t n = ld_u16(pl + 560);
        if (n > 0 && n <= 64)
          for (uint32_t m = 0; m < n; m++)
            if (ld_u16(pl + 690 + 2 * m) == i) w = ld_f16(pl + 562 + 2 * m);
      }
      P.out[i] = w;
    }
    return;
  }
  const uint64_t total = (uint64_t)rows * cols;
  const uint32_t tg = cols / 128;
  for (uint64_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total && i < P.cap; i += gridDim.x * blockDim.x) {
    uint32_t r = (uint32_t)(i / cols), c = (uint32_t)(i % cols);
    float w;
    if (qb == 4) {
      uint8_t b = code[(uint64_t)r * (cols / 2) + c / 2];
      int n = (c & 1) ? (b >> 4) & 15 : b & 15;
      w = g128 ? __fmul_rn((float)n - 8.0f, ld_f16(pl + 48 + 2 * (r * tg + c / 128)))
               : __fadd_rn(__fmul_rn((float)(n - 8), sc), bi);
    } else if (qb == 8) {
      w = (float)(int8_t)code[(uint64_t)r * cols + c];
    } else if (qb == 16) {
      uint16_t h = ld_u16(code + 2 * i);
      w = (flags & 4u) ? h2f(h) : bf2f(h);
    } else if (qb == 32) {
      w = ld_f32(code + 4 * i);
    } else {
      uint8_t b = code[(uint64_t)r * (cols / 4) + c / 4];
      float cb = CB[(b >> (2 * (c & 3))) & 3];
      w = g128 ? __fmul_rn(cb, ld_f16(pl + 48 + 2 * (r * tg + c / 128))) : __fadd_rn(__fmul_rn(cb, sc), bi);
    }
    P.out[i] = w;
  }
}

// Failure-detection probe: one thread waits, bounded by tp.wait_polls, for an
// arrival on counter `kind` of this rank's exchange counters that nothing
// sends (a slot no exchange uses), then records the timeout in StepState::err
// exactly as a tensor-parallel wait that gave up does.
struct WaitProbeLaunch {
  TpLink tp;
  StepState* st;
  int32_t kind;
};
static __global__ void wait_probe_kernel(const __grid_constant__ WaitProbeLaunch P) {
  if (threadIdx.x != 0) return;
  const unsigned long long target = ld_acquire_sys(&P.tp.sh->sig[P.kind]) + 1ull;
  if (!tp_wait_count(P.tp, P.kind, target)) atomicExch(&P.st->err, 1);
}

}  // namespace chpe
