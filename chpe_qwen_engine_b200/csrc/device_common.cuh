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

// Bounded spin helpers never needed here: every cross-CTA hand-off in these
// kernels is an atomic counter checked once by the last arriving CTA.
