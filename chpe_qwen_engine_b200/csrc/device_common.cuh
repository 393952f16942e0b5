// device_common.cuh -- shared device helpers for the sm_100a decode kernels.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "engine_types.h"

#define CHPE_DEV __device__ __forceinline__

// ---- programmatic dependent launch (PDL) ----------------------------------
// Each kernel may run its weight prefetch before pdl_wait(); everything that
// reads a predecessor's output comes after it.
CHPE_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CHPE_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Bulk prefetch of a global byte range into L2 (no data dependency).
CHPE_DEV void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Streaming 128-bit load of weights: read once, do not keep in L1.
CHPE_DEV uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

CHPE_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

CHPE_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
CHPE_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

CHPE_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
CHPE_DEV float bf2f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
CHPE_DEV uint16_t ld_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
CHPE_DEV float ld_f16(const uint8_t* p) { return h2f(ld_u16(p)); }
CHPE_DEV float ld_f32(const uint8_t* p) { return *reinterpret_cast<const float*>(p); }

CHPE_DEV float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// The reference's silu (chpe_engine.zig:159).
CHPE_DEV float silu_ref(float z) { return z / (1.0f + expf(-z)); }

// ---- shared-memory barriers and bulk copies (TMA, non-tensor) -------------
CHPE_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
CHPE_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
CHPE_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
CHPE_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
CHPE_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Bulk copy global -> this CTA's shared memory, completing on `bar`.  Both
// addresses 16-byte aligned, size a multiple of 16.
CHPE_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
CHPE_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Every wait is bounded: try_wait suspends for a bounded time per call, and
// after this many calls the caller records a device timeout and gives up.
constexpr uint32_t kMaxWaitPolls = 1u << 22;
CHPE_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMaxWaitPolls; i++)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ---- tensor-parallel exchange over peer memory ------------------------------
template <class T>
CHPE_DEV T* tp_at(T* p, const chpe::TpLink& t, int r) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(p) + t.delta[r]);
}
CHPE_DEV unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
CHPE_DEV void red_add_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("red.relaxed.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Bounded wait until this rank's counter `kind` reaches `target`: at most
// t.wait_polls polls (kMaxWaitPolls when 0), each followed by a short sleep.
CHPE_DEV bool tp_wait_count(const chpe::TpLink& t, int kind, unsigned long long target) {
  const uint32_t limit = t.wait_polls ? t.wait_polls : kMaxWaitPolls;
  for (uint32_t i = 0; i < limit; i++) {
    if (ld_acquire_sys(&t.sh->sig[kind]) >= target) return true;
    if ((i & 1023u) == 0u && t.err && *reinterpret_cast<volatile const int32_t*>(t.err)) return false;
    __nanosleep(64);
  }
  return false;
}
// The wait a kernel does before reading its input (no-op on one GPU).
CHPE_DEV bool tp_wait(const chpe::TpLink& t) {
  if (t.world <= 1 || t.wait_sig < 0) return true;
  const unsigned long long e = *reinterpret_cast<volatile const uint32_t*>(&t.sh->epoch);
  return tp_wait_count(t, t.wait_sig, (e * t.wait_per_step + t.wait_index) * t.wait_units);
}
// One arrival on every rank; call after this CTA's output stores (and a
// barrier over the threads that made them).  One system-scope fence, then
// relaxed additions: the fence orders every earlier store of the CTA (made
// visible to this thread by the barrier) before each addition (release
// pattern), without a fence per rank.
CHPE_DEV void tp_signal(const chpe::TpLink& t, int kind) {
  if (t.world <= 1 || kind < 0) return;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int r = 0; r < t.world; r++) red_add_relaxed_sys(&tp_at(t.sh, t, r)->sig[kind], 1ull);
}
// n arrivals at once (a CTA that writes the outputs of n CTAs)
CHPE_DEV void tp_signal_n(const chpe::TpLink& t, int kind, uint32_t n) {
  if (t.world <= 1 || kind < 0) return;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int r = 0; r < t.world; r++) red_add_relaxed_sys(&tp_at(t.sh, t, r)->sig[kind], (unsigned long long)n);
}
// Store v at y[i] on this rank, or on every rank when the output is exchanged.
CHPE_DEV void tp_put(const chpe::TpLink& t, float* y, uint32_t i, float v) {
  if (t.bcast && t.world > 1) {
    for (int r = 0; r < t.world; r++) tp_at(y, t, r)[i] = v;
  } else {
    y[i] = v;
  }
}
