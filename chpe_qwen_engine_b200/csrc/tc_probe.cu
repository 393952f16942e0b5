// tc_probe.cu -- a self-checking probe of the tcgen05 integer MMA path the
// batched verify GEMM uses: A (128 x 64 unsigned bytes) written to tensor
// memory with tcgen05.st, B (N x 64 signed bytes) in shared memory in the
// K-major no-swizzle layout, two K=32 MMAs accumulating into an s32 tile in
// tensor memory, read back with tcgen05.ld.  The parity suite compares the
// result with an exact integer product on the host.
#include <cuda_runtime.h>

#include <string>

#include "../../include/chpe.h"
#include "engine.h"
#include "tc_common.cuh"

namespace {

constexpr int kProbeMaxN = 32;

// B element (n, k) of MMA block j = k / 32 in the K-major no-swizzle layout:
// core matrices of 8 rows x 16 bytes; the two along K 128 bytes apart, the
// row groups 256 bytes apart; a block holds N x 32 bytes.
__host__ __device__ inline uint32_t b_offset(uint32_t n, uint32_t k, uint32_t N) {
  const uint32_t j = k >> 5, kk = k & 31u;
  return j * N * 32u + (n >> 3) * 256u + (kk >> 4) * 128u + (n & 7u) * 16u + (kk & 15u);
}

__global__ void __launch_bounds__(128, 1)
    tc_probe_kernel(const uint8_t* A, const int8_t* B, int N, int32_t* D, int32_t* status) {
  __shared__ __align__(1024) int8_t bsm[2 * kProbeMaxN * 32];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t s_taddr;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) {
    chpe::tc::tmem_alloc(&s_taddr, 64);
    chpe::tc::tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  for (int i = tid; i < N * 64; i += blockDim.x) {
    const int n = i >> 6, k = i & 63;
    bsm[b_offset((uint32_t)n, (uint32_t)k, (uint32_t)N)] = B[n * 64 + k];
  }
  fence_proxy_async_smem();  // generic stores -> visible to the tensor core
  chpe::tc::fence_before_sync();
  __syncthreads();
  chpe::tc::fence_after_sync();
  const uint32_t taddr = s_taddr;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  {
    uint32_t v[16];
    const uint32_t* row = reinterpret_cast<const uint32_t*>(A + tid * 64);
#pragma unroll
    for (int w = 0; w < 16; w++) v[w] = row[w];
    chpe::tc::st16(taddr + lane_base, v);  // columns 0..15: K bytes 0..63 of row tid
    chpe::tc::st_wait();
  }
  chpe::tc::fence_before_sync();
  __syncthreads();
  if (tid == 0) {
    chpe::tc::fence_after_sync();
    const uint32_t idesc = chpe::tc::idesc_i8_u8s8(128, (uint32_t)N);
#pragma unroll
    for (uint32_t j = 0; j < 2; j++)
      chpe::tc::mma_i8_ts(taddr + 32u, taddr + 8u * j,
                          chpe::tc::smem_desc_kmajor(bsm + j * (uint32_t)N * 32u, 128u, 256u), idesc, j);
    chpe::tc::commit(&bar);
  }
  const bool ok = mbar_wait(&bar, 0);
  chpe::tc::fence_after_sync();
  if (ok) {
    for (int c0 = 0; c0 < N; c0 += 16) {
      uint32_t d[16];
      chpe::tc::ld16(taddr + lane_base + 32u + (uint32_t)c0, d);
      chpe::tc::ld_wait();
#pragma unroll
      for (int i = 0; i < 16; i++) D[tid * N + c0 + i] = (int32_t)d[i];
    }
  } else if (tid == 0) {
    *status = 1;
  }
  chpe::tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    chpe::tc::fence_after_sync();
    chpe::tc::tmem_dealloc(taddr, 64);
  }
}

}  // namespace

extern "C" int chpe_probe_tc_i8(const uint8_t* a, const int8_t* b, int n, int32_t* d, int device) {
  if (!a || !b || !d || (n != 16 && n != 32)) {
    chpe::set_thread_error("chpe_probe_tc_i8: bad arguments (n must be 16 or 32)");
    return -1;
  }
  uint8_t* da = nullptr;
  int8_t* db = nullptr;
  int32_t *dd = nullptr, *ds = nullptr;
  int rc = 0;
  auto ck = [&](cudaError_t e) {
    if (e != cudaSuccess && rc == 0) {
      chpe::set_thread_error(std::string("chpe_probe_tc_i8: ") + cudaGetErrorString(e));
      rc = -1;
    }
    return e == cudaSuccess;
  };
  if (ck(cudaSetDevice(device)) && ck(cudaMalloc(&da, 128 * 64)) && ck(cudaMalloc(&db, n * 64)) &&
      ck(cudaMalloc(&dd, 128 * n * 4)) && ck(cudaMalloc(&ds, 4)) && ck(cudaMemset(ds, 0, 4)) &&
      ck(cudaMemcpy(da, a, 128 * 64, cudaMemcpyHostToDevice)) &&
      ck(cudaMemcpy(db, b, n * 64, cudaMemcpyHostToDevice))) {
    tc_probe_kernel<<<1, 128>>>(da, db, n, dd, ds);
    int32_t st = 0;
    if (ck(cudaGetLastError()) && ck(cudaDeviceSynchronize()) &&
        ck(cudaMemcpy(d, dd, 128 * n * 4, cudaMemcpyDeviceToHost)) &&
        ck(cudaMemcpy(&st, ds, 4, cudaMemcpyDeviceToHost)) && st != 0) {
      chpe::set_thread_error("chpe_probe_tc_i8: the MMA completion wait timed out");
      rc = -1;
    }
  }
  cudaFree(da);
  cudaFree(db);
  cudaFree(dd);
  cudaFree(ds);
  return rc;
}
