// chpe_c_api.cpp -- the extern "C" surface of libchpe.so (see include/chpe.h).
// Restates src/chpe_c_api.zig's contract over the B200 engine.
#include "../../include/chpe.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "engine.h"

namespace {

struct Ctx {
  chpe::Engine* engine = nullptr;
  const uint8_t* map = nullptr;  // owned mmap (chpe_init), or nullptr
  size_t map_len = 0;
  int arch = 0;
  std::vector<float> last_logits;
  uint32_t last_argmax = 0;
  float last_max_logit = 0.f, last_token0 = 0.f, last_hidden_norm = 0.f;
  uint64_t last_elapsed_ns = 0;
  int last_finite = 0;
  std::string err;
  std::string name;  // chpe_role_kernel_name result
};

thread_local std::string g_init_error;

// chpe_c_api.zig:29-37: architecture from path substrings.
int arch_from_path(const char* p) {
  if (strstr(p, "9B") || strstr(p, "9b") || strstr(p, "qwen35")) return CHPE_ARCH_QWEN3_5_9B;
  if (strstr(p, "72B") || strstr(p, "72b")) return CHPE_ARCH_QWEN2_5_72B;
  return CHPE_ARCH_QWEN2_5_3B;
}

// weight_archive.zig:152-172
int validate(const uint8_t* b, uint64_t len) {
  if (len < 4096) return 6;
  uint32_t magic, version;
  uint64_t hb, rc, rb, cb, pb;
  memcpy(&magic, b, 4);
  memcpy(&version, b + 4, 4);
  memcpy(&hb, b + 8, 8);
  memcpy(&rc, b + 16, 8);
  memcpy(&rb, b + 32, 8);
  memcpy(&cb, b + 40, 8);
  memcpy(&pb, b + 48, 8);
  if (magic != CHPE_ARCHIVE_MAGIC && magic != CHPE_CHPE_MAGIC) return 1;
  if (version != 1) return 2;
  if (hb != 4096) return 10;
  bool standard = rb == CHPE_RECORD_BYTES && pb == CHPE_PREFETCH_BYTES;
  bool dense = rb == CHPE_CELL_BYTES && pb == 0;
  bool raw = rb == CHPE_TILE_CODE_BYTES && pb == 0;
  if (!standard && !dense && !raw) return 3;
  if (!raw && cb != CHPE_CELL_BYTES) return 3;
  if (raw && cb != CHPE_TILE_CODE_BYTES) return 3;
  if (hb + rc * rb > len) return 4;
  return 0;
}

void* make_ctx(const uint8_t* bytes, uint64_t len, const uint8_t* owned_map, int arch,
               uint32_t max_seq, int device, int tp_rank = 0, int tp_world = 1) {
  Ctx* c = new Ctx();
  try {
    c->engine = new chpe::Engine(bytes, len, arch, max_seq, device, tp_rank, tp_world);
  } catch (const std::exception& e) {
    g_init_error = e.what();
    if (owned_map) munmap(const_cast<uint8_t*>(owned_map), len);
    delete c;
    return nullptr;
  }
  c->map = owned_map;
  c->map_len = owned_map ? len : 0;
  c->arch = arch;
  c->last_logits.assign(c->engine->arch().V, 0.f);
  return c;
}

// WeightArchive.openPosix (weight_archive.zig:184-222): read-only private map.
void* open_path(const char* path, int arch, uint32_t max_seq, int device, int tp_rank = 0,
                int tp_world = 1) {
  if (!path) { g_init_error = "null path"; return nullptr; }
  int fd = open(path, O_RDONLY);
  if (fd < 0) { g_init_error = "cannot open archive"; return nullptr; }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 4096) {
    close(fd);
    g_init_error = "archive too small";
    return nullptr;
  }
  size_t len = (size_t)st.st_size;
  void* m = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) { g_init_error = "mmap failed"; return nullptr; }
  madvise(m, len, MADV_SEQUENTIAL);
  madvise(m, len, MADV_WILLNEED);
  int rc = validate((const uint8_t*)m, len);
  if (rc != 0) {
    munmap(m, len);
    g_init_error = "archive validation failed: " + std::to_string(rc);
    return nullptr;
  }
  if (arch == CHPE_ARCH_BY_PATH) arch = arch_from_path(path);
  return make_ctx((const uint8_t*)m, len, (const uint8_t*)m, arch, max_seq, device, tp_rank, tp_world);
}

void store_result(Ctx* c) {
  const chpe::StepResult& r = c->engine->last_result();
  c->last_argmax = r.argmax_token;
  c->last_max_logit = r.max_logit;
  c->last_token0 = r.token0_logit;
  c->last_hidden_norm = r.hidden_norm;
  c->last_finite = r.all_finite;
  c->last_elapsed_ns = c->engine->last_elapsed_ns();
  c->engine->copy_logits(c->last_logits.data());
}

}  // namespace

void chpe::set_thread_error(const std::string& msg) { g_init_error = msg; }

extern "C" {

void* chpe_init(const char* archive_path) {
  return open_path(archive_path, CHPE_ARCH_BY_PATH, 2048, 0);
}

void* chpe_init_ex(const char* archive_path, int arch, uint32_t max_seq_len, int device) {
  return open_path(archive_path, arch, max_seq_len, device);
}

void* chpe_init_tp(const char* archive_path, int arch, uint32_t max_seq_len, int device, int rank,
                   int world) {
  return open_path(archive_path, arch, max_seq_len, device, rank, world);
}

void* chpe_init_tp_bytes(const void* bytes, uint64_t len, int arch, uint32_t max_seq_len, int device,
                         int rank, int world) {
  if (!bytes) { g_init_error = "null bytes"; return nullptr; }
  return make_ctx((const uint8_t*)bytes, len, nullptr, arch, max_seq_len, device, rank, world);
}

int chpe_tp_export_handle(void* ctx, uint8_t* handle64) {
  if (!ctx || !handle64) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->tp_export(handle64);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_tp_slice(int arch, int rank, int world, uint32_t out[10]) {
  ChpeTpSlice sl;
  if (!out || chpe_tp_slice_of(arch, rank, world, &sl) != 0) return -1;
  const uint32_t v[10] = {sl.hq, sl.h0, sl.kv0, sl.kvl, sl.dl, sl.d0, sl.fl, sl.f0, sl.vl, sl.v0};
  memcpy(out, v, sizeof(v));
  return 0;
}

int chpe_tp_connect(void* ctx, const uint8_t* handles, int world) {
  if (!ctx || !handles) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->tp_connect(handles, world);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

void* chpe_init_bytes(const void* bytes, uint64_t len, int arch, uint32_t max_seq_len, int device) {
  if (!bytes) { g_init_error = "null bytes"; return nullptr; }
  return make_ctx((const uint8_t*)bytes, len, nullptr, arch, max_seq_len, device);
}

int chpe_validate_archive(const void* bytes, uint64_t len) {
  if (!bytes) return 6;
  return validate((const uint8_t*)bytes, len);
}

int chpe_forward_tokens(void* ctx, const uint32_t* tokens, size_t n, float* out_logits) {
  if (!ctx || !tokens || n == 0) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->forward(tokens, n, 0);
    store_result(c);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  if (out_logits) memcpy(out_logits, c->last_logits.data(), c->last_logits.size() * 4);
  return (int)c->last_argmax;
}

int chpe_decode_step(void* ctx, uint32_t token, uint32_t pos, float* out_logits) {
  if (!ctx) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->forward(&token, 1, pos);
    store_result(c);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  if (out_logits) memcpy(out_logits, c->last_logits.data(), c->last_logits.size() * 4);
  return (int)c->last_argmax;
}

int chpe_verify(void* ctx, const uint32_t* toks, size_t m, uint32_t pos, float* out_logits,
                uint32_t* out_argmax) {
  if (!ctx || !toks || m == 0) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->verify(toks, m, pos, out_logits, out_argmax);
    store_result(c);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_profile_verify(void* ctx, size_t m, uint32_t pos, float* role_ms, double* role_bytes, int cap) {
  if (!ctx || !role_ms || !role_bytes || cap < 1) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    return c->engine->profile_verify(m, pos, role_ms, role_bytes, cap);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
}

int chpe_last_verify_batched(void* ctx) {
  return ctx ? ((Ctx*)ctx)->engine->last_verify_batched() : 0;
}

const char* chpe_verify_batched_unavailable(void* ctx, int m) {
  if (!ctx) return "null context";
  Ctx* c = (Ctx*)ctx;
  try {
    c->name = c->engine->batch_unavailable_reason(m <= 4 ? 4 : 8);
  } catch (const std::exception& e) {
    c->name = e.what();
  }
  return c->name.c_str();
}

int chpe_generate(void* ctx, const uint32_t* prompt, size_t n_prompt, size_t n_gen, uint32_t* out) {
  if (!ctx || !prompt || n_prompt == 0 || (n_gen > 0 && !out)) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->generate(prompt, n_prompt, n_gen, out);
    store_result(c);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_speculative_generate(void* ctx, const uint32_t* prompt, size_t n_prompt, size_t n_gen,
                              uint32_t draft_len, uint32_t ngram, uint32_t* out, uint64_t* stats) {
  if (!ctx || !prompt || n_prompt == 0 || (n_gen > 0 && !out)) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->speculative_generate(prompt, n_prompt, n_gen, draft_len, ngram, out, stats);
    store_result(c);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_bench_greedy(void* ctx, size_t n, float* ms) {
  if (!ctx || !ms) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    *ms = c->engine->timed_greedy_steps(n);
    store_result(c);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_bench_host(void* ctx, const uint32_t* toks, size_t n, float* logits, double* ms) {
  if (!ctx || !toks || !logits || !ms) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    *ms = c->engine->timed_host_steps(toks, n, logits);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_bench_kernel(void* ctx, int role, int rounds, float* avg_ms, double* bytes_per_launch,
                      int* launches) {
  if (!ctx || !avg_ms || !bytes_per_launch || !launches || rounds < 1) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->bench_role(role, rounds, avg_ms, bytes_per_launch, launches);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_bench_kernel_cold(void* ctx, int role, int rounds, float* avg_ms, double* bytes_per_launch,
                           int* launches) {
  if (!ctx || !avg_ms || !bytes_per_launch || !launches || rounds < 1) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->bench_role(role, rounds, avg_ms, bytes_per_launch, launches, true);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_profile_step(void* ctx, float* op_ms, int* op_roles, int cap) {
  if (!ctx || cap < 0) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    return c->engine->profile_step(op_ms, op_roles, cap);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
}

double chpe_step_weight_bytes(void* ctx) {
  if (!ctx) return 0.0;
  return ((Ctx*)ctx)->engine->step_weight_bytes();
}

const char* chpe_role_kernel_name(void* ctx, int role) {
  if (!ctx) return "";
  Ctx* c = (Ctx*)ctx;
  try {
    c->name = c->engine->role_kernel_name(role);
  } catch (const std::exception& e) {
    c->err = e.what();
    c->name.clear();
  }
  return c->name.c_str();
}

size_t chpe_get_last_logits(void* ctx, float* out, size_t max_len) {
  if (!ctx || !out) return 0;
  Ctx* c = (Ctx*)ctx;
  if (max_len < c->last_logits.size()) return 0;
  memcpy(out, c->last_logits.data(), c->last_logits.size() * 4);
  return c->last_logits.size();
}

size_t chpe_get_vocab_size(void* ctx) {
  return ctx ? ((Ctx*)ctx)->engine->arch().V : chpe_arch_preset(CHPE_ARCH_3B)->V;
}
size_t chpe_get_hidden_dim(void* ctx) {
  return ctx ? ((Ctx*)ctx)->engine->arch().D : chpe_arch_preset(CHPE_ARCH_3B)->D;
}
size_t chpe_get_num_layers(void* ctx) {
  return ctx ? ((Ctx*)ctx)->engine->arch().L : chpe_arch_preset(CHPE_ARCH_3B)->L;
}
uint64_t chpe_get_last_elapsed_ns(void* ctx) { return ctx ? ((Ctx*)ctx)->last_elapsed_ns : 0; }
uint32_t chpe_get_last_argmax(void* ctx) { return ctx ? ((Ctx*)ctx)->last_argmax : 0; }
float chpe_get_last_max_logit(void* ctx) { return ctx ? ((Ctx*)ctx)->last_max_logit : 0.f; }
float chpe_get_last_token0_logit(void* ctx) { return ctx ? ((Ctx*)ctx)->last_token0 : 0.f; }
float chpe_get_last_hidden_norm(void* ctx) { return ctx ? ((Ctx*)ctx)->last_hidden_norm : 0.f; }
int chpe_get_last_all_finite(void* ctx) { return ctx ? ((Ctx*)ctx)->last_finite : 0; }
int chpe_kernels_per_step(void* ctx) { return ctx ? ((Ctx*)ctx)->engine->kernels_per_step() : 0; }
uint32_t chpe_get_position(void* ctx) { return ctx ? ((Ctx*)ctx)->engine->current_pos() : 0; }
uint64_t chpe_device_archive_bytes(void* ctx) { return ctx ? ((Ctx*)ctx)->engine->device_archive_bytes() : 0; }

const char* chpe_last_error(void* ctx) {
  return ctx ? ((Ctx*)ctx)->err.c_str() : g_init_error.c_str();
}

void chpe_free(void* ctx) {
  if (!ctx) return;
  Ctx* c = (Ctx*)ctx;
  delete c->engine;
  if (c->map) munmap(const_cast<uint8_t*>(c->map), c->map_len);
  delete c;
}

int chpe_kv_load(void* ctx, uint32_t layer, uint32_t pos0, uint32_t n, const float* k, const float* v) {
  if (!ctx || (n > 0 && (!k || !v))) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->kv_load(layer, pos0, n, k, v);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_kv_set_page_order(void* ctx, const uint32_t* order, uint32_t n) {
  if (!ctx || !order) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->kv_set_page_order(order, n);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_kv_page_table(void* ctx, uint32_t* out, uint32_t cap, uint32_t* num_pages) {
  if (!ctx) return -1;
  Ctx* c = (Ctx*)ctx;
  if (num_pages) *num_pages = c->engine->kv_pages();
  return (int)c->engine->kv_page_table(out, out ? cap : 0);
}

uint32_t chpe_kv_page_size(void) { return chpe::Engine::kKvPage; }

int chpe_probe_gemv_linear(void* ctx, uint64_t tile_start, uint64_t num_tiles, const float* x,
                           uint64_t x_len, float* y, uint64_t r_total, uint64_t c_total,
                           int accumulate, int64_t bias_tile) {
  if (!ctx || !x || !y) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->debug_gemv_linear(tile_start, num_tiles, x, x_len, y, r_total, c_total, accumulate,
                                 bias_tile);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_probe_attention(void* ctx, uint32_t layer, uint32_t pos, const float* q, const float* k,
                         const float* v, float* out) {
  if (!ctx || !q || !k || !v || !out) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->debug_attention(layer, pos, q, k, v, out);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_probe_bgemm(void* ctx, uint64_t tile_start, uint64_t num_tiles, const float* x, int nt, float* y,
                     uint64_t r_total, uint64_t c_total, int accumulate) {
  if (!ctx || !x || !y) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->debug_bgemm(tile_start, num_tiles, x, nt, y, r_total, c_total, accumulate);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_probe_wait_timeout(void* ctx, uint32_t polls) {
  if (!ctx) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->debug_wait_timeout(polls);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_probe_embed(void* ctx, uint32_t token, float* out) {
  if (!ctx || !out) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->debug_embed(token, out);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

int chpe_probe_dequant_cell(void* ctx, uint64_t tile, int flat, float* out, uint64_t cap,
                            uint64_t* n_out) {
  if (!ctx || !out || !n_out) return -1;
  Ctx* c = (Ctx*)ctx;
  try {
    c->engine->debug_dequant_cell(tile, flat, out, cap, n_out);
  } catch (const std::exception& e) {
    c->err = e.what();
    return -1;
  }
  return 0;
}

}  // extern "C"
