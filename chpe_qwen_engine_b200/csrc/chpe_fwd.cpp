// chpe_fwd.cpp -- the command-line front end of libchpe.so.
//
// Same contract as the reference's `chpe_fwd` (src/main.zig:10-246): the
// flags --archive, --tokens-file (raw little-endian u32 ids), --out-logits
// (raw f32 logits of the last token), --arch, --bench, --max-seq-len and a
// bare archive path; the same receipt lines on stderr, which the reference's
// scripts parse (scripts/eval_lambada_fidelity.py:134-160,
// tests/verify_baseline_parity.sh:58-94); and the result JSON written to
// run/spoke_outbox/metal.chpe_fwd.result.json when that directory exists.
// Every bench iteration runs the prompt from position 0 (chpe_forward_tokens),
// as the reference's loop over forwardDecode does (src/main.zig:157-181).
//
// Extra flag (no reference counterpart): --device N picks the CUDA device.
#include <cuda_runtime.h>
#include <sys/stat.h>
#include <time.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/chpe.h"

namespace {

struct ArchFacts {
  const char* name;
  int layers, hidden, inter, vocab;
};
// chpe_engine.zig:110-145 (the presets the engine reports)
const ArchFacts kArch[3] = {{"Qwen2.5-3B", 36, 2048, 11008, 151936},
                            {"Qwen3.5-9B", 32, 4096, 12288, 248320},
                            {"Qwen2.5-72B", 80, 8192, 29568, 152064}};

double now_ms() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

// src/main.zig:86-106: the override wins; else the archive path decides.
int pick_arch(const char* archive, const char* override_name) {
  if (override_name) {
    if (strstr(override_name, "9b") || strstr(override_name, "9B")) return CHPE_ARCH_QWEN3_5_9B;
    if (strstr(override_name, "72b") || strstr(override_name, "72B")) return CHPE_ARCH_QWEN2_5_72B;
    return CHPE_ARCH_QWEN2_5_3B;
  }
  if (strstr(archive, "9B") || strstr(archive, "9b") || strstr(archive, "qwen35")) return CHPE_ARCH_QWEN3_5_9B;
  if (strstr(archive, "72B") || strstr(archive, "72b")) return CHPE_ARCH_QWEN2_5_72B;
  return CHPE_ARCH_QWEN2_5_3B;
}

void usage() {
  fprintf(stderr,
          "Unified Polymorphic CHPE Forward Engine\n\n"
          "Usage: chpe_fwd [OPTIONS]\n\n"
          "Options:\n"
          "  --archive <path>       Path to .chpe weight archive\n"
          "  --tokens-file <path>   Binary little-endian u32 tokens file\n"
          "  --out-logits <path>    Destination binary file for output float logits\n"
          "  --arch <name>          Model architecture (qwen2_5_3b | qwen3_5_9b | qwen2_5_72b)\n"
          "  --bench <iters>        Benchmark iterations (default: 1)\n"
          "  --max-seq-len <len>    Maximum sequence length (default: 2048)\n"
          "  --device <n>           CUDA device (default: 0)\n"
          "  -h, --help             Display this help message\n");
}

}  // namespace

int main(int argc, char** argv) {
  std::string archive = "models/warc/Qwen2.5-3B-Instruct.bf16.raw.chpe";
  const char* tokens_file = nullptr;
  const char* out_logits = nullptr;
  const char* arch_override = nullptr;
  long bench_iters = 1, max_seq = 2048;
  int device = 0;
  for (int i = 1; i < argc; i++) {
    const char* a = argv[i];
    auto next = [&]() -> const char* { return i + 1 < argc ? argv[++i] : nullptr; };
    if (!strcmp(a, "--archive")) {
      if (const char* v = next()) archive = v;
    } else if (!strcmp(a, "--tokens-file")) {
      tokens_file = next();
    } else if (!strcmp(a, "--out-logits")) {
      out_logits = next();
    } else if (!strcmp(a, "--arch")) {
      arch_override = next();
    } else if (!strcmp(a, "--bench")) {
      if (const char* v = next()) {
        char* end = nullptr;
        bench_iters = strtol(v, &end, 10);
        if (!end || *end || bench_iters < 1) bench_iters = 1;
      }
    } else if (!strcmp(a, "--max-seq-len")) {
      if (const char* v = next()) {
        char* end = nullptr;
        max_seq = strtol(v, &end, 10);
        if (!end || *end || max_seq < 1) max_seq = 2048;
      }
    } else if (!strcmp(a, "--device")) {
      if (const char* v = next()) device = atoi(v);
    } else if (!strcmp(a, "--help") || !strcmp(a, "-h")) {
      usage();
      return 0;
    } else if (strncmp(a, "--", 2) != 0) {
      archive = a;
    }
  }

  const int arch = pick_arch(archive.c_str(), arch_override);
  const ArchFacts& A = kArch[arch];
  fprintf(stderr, "=== [UNIFIED POLYMORPHIC CHPE FORWARD ENGINE] ===\n");
  fprintf(stderr, "Model Arch     : %s (%d layers, D=%d, intermediate=%d, vocab=%d)\n", A.name, A.layers,
          A.hidden, A.inter, A.vocab);
  fprintf(stderr, "Archive Path   : %s\n", archive.c_str());

  struct stat st;
  if (stat(archive.c_str(), &st) != 0) {
    fprintf(stderr, "ERROR: Failed to open weight archive '%s': FileNotFound\n", archive.c_str());
    return 1;
  }

  {
    uint64_t records = 0;  // header record_count (weight_archive.zig:53-86)
    if (FILE* f = fopen(archive.c_str(), "rb")) {
      if (fseek(f, 16, SEEK_SET) != 0 || fread(&records, 8, 1, f) != 1) records = 0;
      fclose(f);
    }
    fprintf(stderr, "Archive Size   : %lld bytes (%.2f GB, %llu tiles)\n", (long long)st.st_size,
            (double)st.st_size / (1024.0 * 1024.0 * 1024.0), (unsigned long long)records);
  }

  std::vector<uint32_t> prompt;
  if (tokens_file) {
    FILE* f = fopen(tokens_file, "rb");
    if (!f) {
      fprintf(stderr, "ERROR: Failed to open tokens file '%s'\n", tokens_file);
      return 1;
    }
    fseek(f, 0, SEEK_END);
    const long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    const size_t n = sz > 0 ? (size_t)sz / 4 : 0;
    if (n == 0) {
      fclose(f);
      fprintf(stderr, "ERROR: EmptyTokensFile\n");
      return 1;
    }
    prompt.resize(n);
    const size_t got = fread(prompt.data(), 4, n, f);
    fclose(f);
    if (got != n) {
      fprintf(stderr, "ERROR: short read of tokens file '%s'\n", tokens_file);
      return 1;
    }
    fprintf(stderr, "Prompt Tokens  : Loaded %zu tokens from '%s'\n", n, tokens_file);
  } else {
    prompt.push_back(151644);  // <|im_start|>, src/main.zig:128
    fprintf(stderr, "Prompt Tokens  : Default single token [%u]\n", prompt[0]);
  }
  if ((long)prompt.size() > max_seq) {
    fprintf(stderr, "ERROR: %zu tokens exceed --max-seq-len %ld\n", prompt.size(), max_seq);
    return 1;
  }

  void* ctx = chpe_init_ex(archive.c_str(), arch, (uint32_t)max_seq, device);
  if (!ctx) {
    fprintf(stderr, "ERROR: Failed to open weight archive '%s': %s\n", archive.c_str(), chpe_last_error(nullptr));
    return 1;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) == cudaSuccess)
    fprintf(stderr, "Hardware Core  : %s (sm_%d%d, %d SMs, CUDA)\n", prop.name, prop.major, prop.minor,
            prop.multiProcessorCount);
  fprintf(stderr, "Execution Loop : Running forward pass over %zu prompt tokens...\n", prompt.size());

  double min_ms = 1e300, max_ms = 0.0, sum_ms = 0.0;
  for (long it = 0; it < bench_iters; it++) {
    const double t0 = now_ms();
    const int r = chpe_forward_tokens(ctx, prompt.data(), prompt.size(), nullptr);
    const double ms = now_ms() - t0;
    if (r < 0) {
      fprintf(stderr, "ERROR: forward pass failed: %s\n", chpe_last_error(ctx));
      chpe_free(ctx);
      return 1;
    }
    if (ms < min_ms) min_ms = ms;
    if (ms > max_ms) max_ms = ms;
    sum_ms += ms;
    if (bench_iters > 1) fprintf(stderr, "  [Iter %ld/%ld] Latency: %.2f ms\n", it + 1, bench_iters, ms);
  }
  const double mean_ms = sum_ms / (double)bench_iters;
  const double tput = (double)prompt.size() / (mean_ms / 1000.0);
  const uint32_t am = chpe_get_last_argmax(ctx);
  const float mx = chpe_get_last_max_logit(ctx), t0l = chpe_get_last_token0_logit(ctx),
              hn = chpe_get_last_hidden_norm(ctx);
  const bool finite = chpe_get_last_all_finite(ctx) != 0;

  fprintf(stderr, "\n=== [PHYSICAL SILICON EXECUTION RECEIPT] ===\n");
  fprintf(stderr, "Argmax Decoded Token ID : %u\n", am);
  fprintf(stderr, "Maximum Vocab Logit     : %.6f\n", mx);
  fprintf(stderr, "Token 0 Logit           : %.6f\n", t0l);
  fprintf(stderr, "Final Hidden Vector Norm: %.6f\n", hn);
  fprintf(stderr, "Mean Latency            : %.2f ms (%.3f s)\n", mean_ms, mean_ms / 1000.0);
  fprintf(stderr, "Throughput              : %.2f tokens/sec\n", tput);
  fprintf(stderr, "Numerical Soundness     : %s\n",
          finite ? "100% FINITE (Zero NaN / Zero Inf)" : "FAILED (NaN or Inf present)");

  if (out_logits) {
    const size_t V = chpe_get_vocab_size(ctx);
    std::vector<float> lg(V);
    FILE* f = chpe_get_last_logits(ctx, lg.data(), V) == V ? fopen(out_logits, "wb") : nullptr;
    if (f) {
      const size_t w = fwrite(lg.data(), 4, V, f);
      fclose(f);
      if (w == V)
        fprintf(stderr, "Exported Logits Binary  : %s (%zu floats, %zu bytes)\n", out_logits, V, V * 4);
    }
  }

  // src/main.zig:211-245: the result JSON, when run/spoke_outbox exists
  const char* spoke = "run/spoke_outbox/metal.chpe_fwd.result.json";
  if (FILE* f = fopen(spoke, "wb")) {
    fprintf(f,
            "{\n  \"benchmark\": \"CHPE Forward Engine\",\n  \"model\": \"%s\",\n  \"archive\": \"%s\",\n"
            "  \"tokens_evaluated\": %zu,\n  \"argmax_token\": %u,\n  \"max_logit\": %.6f,\n"
            "  \"token0_logit\": %.6f,\n  \"hidden_norm\": %.6f,\n  \"mean_latency_ms\": %.2f,\n"
            "  \"throughput_tok_s\": %.2f,\n  \"all_finite\": %s\n}\n",
            A.name, archive.c_str(), prompt.size(), am, mx, t0l, hn, mean_ms, tput, finite ? "true" : "false");
    fclose(f);
    fprintf(stderr, "Recorded Spoke Telemetry: %s\n", spoke);
  }
  chpe_free(ctx);
  return 0;
}
