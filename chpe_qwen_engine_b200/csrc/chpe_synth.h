/* chpe_synth.h -- deterministic synthetic .chpe archives (test/bench inputs).
 *
 * No real weights exist in this environment, so every parity test and bench
 * runs on seeded synthetic archives laid out exactly as the reference's tensor
 * maps expect.  Each tile's bytes are a pure function of (seed, tile index):
 * a SplitMix64 stream (Steele, Lea, Flood 2014) keyed by both, so the output
 * is identical for any thread count and on any host.
 *
 * Values: weights ~ N(0, 0.02) (Irwin-Hall sum of four 16-bit uniforms,
 * rescaled), 4/2-bit codes uniform over their range, per-group-128 FP16 scales
 * |N(0, 0.01)|, RMSNorm gains 1.0, biases 0 (or N(0, 0.02) with
 * CHPE_SYNTH_BIAS).
 */
#ifndef CHPE_SYNTH_H
#define CHPE_SYNTH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  /* Benchmark configs are numbered from 1 in the order the benchmark
   * definition lists them: 1 = 3B FP16, 2 = 3B 4/2-bit, 3 = 9B 4-bit,
   * 4 = 9B verify, 5 = 72B 4-bit and FP16. */
  CHPE_SYNTH_3B_FP16_RAW = 0, /* 376853 raw tiles, FLAG_RAW_FP16 (config 1) */
  CHPE_SYNTH_3B_BF16_RAW = 1, /* 376853 raw tiles, BF16 */
  CHPE_SYNTH_3B_W4 = 2,       /* 94349 cells, 4-bit group-128 (config 2) */
  CHPE_SYNTH_3B_W2 = 3,       /* 94349 cells, 2-bit group-128 (config 2) */
  CHPE_SYNTH_9B_W4 = 4,       /* 546681 cells, 4-bit (configs 3 and 4) */
  CHPE_SYNTH_72B_W4 = 5,      /* 2219153 cells, 4-bit (config 5) */
  CHPE_SYNTH_72B_FP16_RAW = 6,/* 2219153 raw tiles, reference map (config 5) */
  CHPE_SYNTH_9B_I8_RAW = 7,   /* 546681 raw tiles, INT8 (flags 0x08) */
  CHPE_SYNTH_NUM_CONFIGS = 8
};

/* Variant flags */
#define CHPE_SYNTH_STANDARD 0x1u /* 20480-byte records with prefetch labels (cells only) */
#define CHPE_SYNTH_OUTLIERS 0x2u /* non-zero row outliers and down_aux replacements */
#define CHPE_SYNTH_NONGROUP 0x4u /* per-tile scale/bias instead of group-128 scales */
#define CHPE_SYNTH_BIAS 0x8u     /* non-zero q/k/v biases */
#define CHPE_SYNTH_MIXED 0x10u   /* vary the cell format per tensor (W8/F16/BF16/F32 cells) */

/* Archive size in bytes for a config (0 for an unknown config). */
uint64_t chpe_synth_bytes(int config, uint32_t flags);
/* Fill `out` (len >= chpe_synth_bytes) with the archive; 0 on success. */
int chpe_synth_fill(int config, uint32_t flags, uint64_t seed, uint8_t *out,
                    uint64_t len, int threads);
/* Write the archive to `path` (streamed in chunks); 0 on success. */
int chpe_synth_write(int config, uint32_t flags, uint64_t seed, const char *path,
                     int threads);

#ifdef __cplusplus
}
#endif
#endif
