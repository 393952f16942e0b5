// attention_noalloc.cu -- decode attention for callers that cannot allocate
// device memory.
//
// Some callers of this library must not call cudaMalloc: serving runtimes
// that hand out device memory only from their own pre-sized pools (an
// allocation behind their back can exceed the budget they planned for the
// KV cache and the weights, and cudaMalloc may synchronise the device in the
// middle of their pipelined work), and plugins loaded into a host process that
// owns all allocation on the GPU.  They have their inputs, caches and outputs
// already, but the decode attention kernel also needs scratch: the per-split
// softmax partials, the arrival counters of the split merge, the RoPE inverse
// frequencies and the step's position.  Here that scratch is a file-scope
// static device array of a fixed size (1 MiB), present on every GPU that
// loads the library for as long as the library stays loaded.
//
// Set-up: the first call on a device (with that device current) resolves the
// array's device address with cudaGetSymbolAddress and caches it.  Every call
// shares the array and finds the previous call's contents there, so each call
// clears the counters it relies on and rewrites the position and frequencies;
// calls whose kernels overlap on the GPU (different streams, no ordering
// between them) race on the array and must not be issued.  Each call copies
// its position and RoPE frequencies from host memory with cudaMemcpyAsync
// (the source is staged before the call returns).
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/chpe.h"
#include "attention.cuh"
#include "engine.h"

namespace {

constexpr size_t kScratchBytes = 1u << 20;  // 1 MiB per device
constexpr size_t kStateOff = 0;             // chpe::StepState
constexpr size_t kCounterOff = 256;         // uint32 per kv head (<= 64)
constexpr size_t kInvFreqOff = 1024;        // float per half head (<= 128)
constexpr size_t kPartOff = 4096;           // split partials

__device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// The message is kept for chpe_last_error(NULL) on this thread.
int fail(int code, const std::string& msg) {
  chpe::set_thread_error("chpe_attention_decode_noalloc: " + msg);
  return code;
}

}  // namespace

extern "C" int chpe_attention_decode_noalloc(const float* q, const float* k, const float* v,
                                             void* k_cache, void* v_cache, float* out,
                                             uint32_t pos, uint32_t max_seq_len, uint32_t num_heads,
                                             uint32_t num_kv_heads, uint32_t head_dim,
                                             float rope_theta, void* stream) {
  if (!q || !k || !v || !k_cache || !v_cache || !out) return fail(-1, "null pointer");
  if (num_kv_heads == 0 || num_kv_heads > 64 || num_heads % num_kv_heads != 0)
    return fail(-1, "num_heads must be a multiple of num_kv_heads (<= 64)");
  const uint32_t G = num_heads / num_kv_heads;
  if (G > 8) return fail(-1, "more than 8 query heads per kv head");
  if (head_dim != 128 && head_dim != 256) return fail(-1, "head_dim must be 128 or 256");
  if (pos >= max_seq_len) return fail(-1, "pos must be below max_seq_len");
  const uint32_t nsplit = chpe::kAttnSplits;
  const size_t need = kPartOff + (size_t)num_kv_heads * nsplit * G * (head_dim + 4) * sizeof(float);
  if (need > kScratchBytes)
    return fail(-2, "needs " + std::to_string(need) + " bytes of scratch; the limit is " +
                        std::to_string(kScratchBytes));

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(-3, "no current CUDA device");
  unsigned char* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
      if (e != cudaSuccess) return fail(-3, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      g_scratch_ptr[dev] = p;
    }
    base = static_cast<unsigned char*>(g_scratch_ptr[dev]);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // step state (this position, no early exit) and RoPE frequencies, computed
  // as applyRope does (chpe_engine.zig:200-202); pageable sources are staged
  // by cudaMemcpyAsync before it returns
  chpe::StepState st;
  memset(&st, 0, sizeof(st));
  st.pos = (int32_t)pos;
  st.finite = 1;
  float invf[128];
  for (uint32_t i = 0; i < head_dim / 2; i++) invf[i] = 1.0f / powf(rope_theta, 2.0f * (float)i / (float)head_dim);
  if (cudaMemcpyAsync(base + kStateOff, &st, sizeof(st), cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaMemcpyAsync(base + kInvFreqOff, invf, head_dim / 2 * sizeof(float), cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaMemsetAsync(base + kCounterOff, 0, num_kv_heads * sizeof(uint32_t), s) != cudaSuccess)
    return fail(-3, "scratch initialisation failed");

  chpe::AttnLaunch P{};
  P.q = q;
  P.k = k;
  P.v = v;
  P.kc = static_cast<__half*>(k_cache);
  P.vc = static_cast<__half*>(v_cache);
  P.out = out;
  P.part = reinterpret_cast<float*>(base + kPartOff);
  P.counters = reinterpret_cast<uint32_t*>(base + kCounterOff);
  P.inv_freq = reinterpret_cast<const float*>(base + kInvFreqOff);
  P.st = reinterpret_cast<chpe::StepState*>(base + kStateOff);
  P.H = (int32_t)num_heads;
  P.KV = (int32_t)num_kv_heads;
  P.HD = (int32_t)head_dim;
  P.nsplit = (int32_t)nsplit;
  P.max_seq = (int32_t)max_seq_len;
  int threads = (int)G * 32;
  if (threads < (int)head_dim / 2) threads = (int)head_dim / 2;
  if (threads < 128) threads = 128;  // the kernel's tile loads assume at least 128 threads
  dim3 grid(nsplit, num_kv_heads);
  if (head_dim == 128) chpe::attention_kernel<128><<<grid, threads, 0, s>>>(P);
  else chpe::attention_kernel<256><<<grid, threads, 0, s>>>(P);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(-3, std::string("launch: ") + cudaGetErrorString(e));
  chpe::set_thread_error("");
  return 0;
}
