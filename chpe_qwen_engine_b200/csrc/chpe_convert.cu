// chpe_convert.cu -- archive format converters (the reference's
// convertToDensePosix, convertToRawContiguousPosix and
// convertToRawFp16ContiguousPosix, src/weight_archive.zig:617-776).
//
// Dense and raw conversions are byte copies (cells without the 3072-byte
// prefetch labels; the 16384 code bytes of each tile) done on the host.  The
// FP16 conversion turns the BF16 weights of every 2-D tile into IEEE half on
// the GPU, in chunks of tiles staged through pinned memory; tiles that hold
// 1-D data (norms, biases: the 3B raw layout's fixed positions, or cells
// whose quant_bits is 32) are copied verbatim, as the reference does.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/chpe.h"
#include "chpe_maps.h"
#include "engine.h"

namespace {

// BF16 bits -> FP16 bits: the f32 value the BF16 denotes, rounded to the
// nearest FP16 (ties to even), overflow to infinity, underflow through the
// subnormals to zero; a NaN stays a NaN with its sign, the quiet bit set and
// the top payload bits kept.
__host__ __device__ inline uint16_t bf16_to_f16_bits(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  const uint32_t exp = (u >> 23) & 0xFFu, mant = u & 0x7FFFFFu;
  if (exp == 0xFFu) return mant ? (uint16_t)(sign | 0x7E00u | (mant >> 13)) : (uint16_t)(sign | 0x7C00u);
  if (exp == 0u) return sign;  // f32 zero or subnormal: far below FP16's smallest subnormal
  const uint32_t m = mant | 0x800000u;  // 24-bit significand, value m * 2^(exp - 150)
  int e16 = (int)exp - 112;             // FP16 biased exponent of the same leading bit
  if (e16 >= 1) {
    uint32_t r = m >> 13;
    const uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    if (r == 0x800u) {  // the rounding carried into the next binade
      r = 0x400u;
      e16++;
    }
    if (e16 >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)e16 << 10) | (r & 0x3FFu));
  }
  const int shift = 14 - e16;  // 13 + (1 - e16): subnormal result
  if (shift > 24) return sign;  // below half the smallest subnormal
  uint32_t r = m >> shift;
  const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
  if (rem > half || (rem == half && (r & 1u))) r++;
  return (uint16_t)(sign | r);  // r == 0x400 encodes the smallest normal
}

__global__ void bf16_to_f16_tiles(uint16_t* data, const uint8_t* convert, uint32_t ntiles) {
  const uint32_t t = blockIdx.x;
  if (t >= ntiles || !convert[t]) return;
  uint4* p = reinterpret_cast<uint4*>(data + (size_t)t * 8192);
  for (uint32_t i = threadIdx.x; i < 1024; i += blockDim.x) {
    uint4 v = p[i];
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++)
      w[j] = (uint32_t)bf16_to_f16_bits((uint16_t)(w[j] & 0xFFFFu)) |
             ((uint32_t)bf16_to_f16_bits((uint16_t)(w[j] >> 16)) << 16);
    p[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

struct Map {
  const uint8_t* p = nullptr;
  size_t len = 0;
  ~Map() {
    if (p) munmap(const_cast<uint8_t*>(p), len);
  }
};

int fail(const std::string& msg) {
  chpe::set_thread_error("chpe_convert_archive: " + msg);
  return -1;
}

uint64_t rd64(const uint8_t* p) {
  uint64_t v;
  memcpy(&v, p, 8);
  return v;
}

}  // namespace

extern "C" int chpe_convert_archive(const char* src_path, const char* dst_path, int mode, int device) {
  if (!src_path || !dst_path) return fail("null path");
  if (mode != CHPE_CONVERT_DENSE && mode != CHPE_CONVERT_RAW && mode != CHPE_CONVERT_RAW_FP16)
    return fail("unknown mode");
  Map src;
  {
    int fd = open(src_path, O_RDONLY);
    if (fd < 0) return fail("cannot open the source archive");
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 4096) {
      close(fd);
      return fail("source archive too small");
    }
    void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return fail("mmap of the source failed");
    src.p = (const uint8_t*)m;
    src.len = (size_t)st.st_size;
    madvise(m, src.len, MADV_SEQUENTIAL);
  }
  const int rc = chpe_validate_archive(src.p, src.len);
  if (rc != 0) return fail("source validation failed: " + std::to_string(rc));
  const uint64_t count = rd64(src.p + 16), rb = rd64(src.p + 32), pb = rd64(src.p + 48);
  const bool src_raw = rb == CHPE_TILE_CODE_BYTES && pb == 0, src_dense = pb == 0;
  if (mode == CHPE_CONVERT_DENSE && src_raw) return fail("a raw archive holds no cells to keep");
  const uint64_t out_stride = mode == CHPE_CONVERT_DENSE ? CHPE_CELL_BYTES : CHPE_TILE_CODE_BYTES;
  const uint64_t out_len = CHPE_HEADER_BYTES + count * out_stride;

  int fd = open(dst_path, O_RDWR | O_CREAT | O_TRUNC, 0644);
  if (fd < 0) return fail("cannot create the destination");
  if (ftruncate(fd, (off_t)out_len) != 0) {
    close(fd);
    return fail("cannot size the destination");
  }
  void* dm = mmap(nullptr, out_len, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (dm == MAP_FAILED) return fail("mmap of the destination failed");
  uint8_t* dst = (uint8_t*)dm;

  // header: the source's 64-byte header with the new geometry, rest zero
  memset(dst, 0, CHPE_HEADER_BYTES);
  memcpy(dst, src.p, 64);
  uint64_t v;
  if (mode == CHPE_CONVERT_DENSE) {
    v = CHPE_CELL_BYTES;
    memcpy(dst + 32, &v, 8);
    v = 0;
    memcpy(dst + 48, &v, 8);
  } else {
    v = CHPE_TILE_CODE_BYTES;
    memcpy(dst + 32, &v, 8);
    memcpy(dst + 40, &v, 8);
    v = 0;
    memcpy(dst + 48, &v, 8);
    if (mode == CHPE_CONVERT_RAW_FP16) {
      v = rd64(src.p + 56) | CHPE_FLAG_RAW_FP16;
      memcpy(dst + 56, &v, 8);
    }
  }
  // source offsets (weight_archive.zig:301-334: getCellDirect, getTileU16Direct)
  auto cell_at = [&](uint64_t i) { return src.p + CHPE_HEADER_BYTES + i * rb + pb; };
  auto tile_at = [&](uint64_t i) {
    if (src_raw) return src.p + CHPE_HEADER_BYTES + i * CHPE_TILE_CODE_BYTES;
    if (src_dense) return src.p + CHPE_HEADER_BYTES + i * CHPE_CELL_BYTES + CHPE_CELL_HEADER_BYTES;
    return src.p + CHPE_HEADER_BYTES + i * CHPE_RECORD_BYTES + CHPE_PREFETCH_BYTES + CHPE_CELL_HEADER_BYTES;
  };
  int result = 0;
  if (mode == CHPE_CONVERT_DENSE) {
    for (uint64_t i = 0; i < count; i++)
      memcpy(dst + CHPE_HEADER_BYTES + i * CHPE_CELL_BYTES, cell_at(i), CHPE_CELL_BYTES);
  } else if (mode == CHPE_CONVERT_RAW) {
    for (uint64_t i = 0; i < count; i++)
      memcpy(dst + CHPE_HEADER_BYTES + i * CHPE_TILE_CODE_BYTES, tile_at(i), CHPE_TILE_CODE_BYTES);
  } else {
    // 1-D tiles (weight_archive.zig:751-765): the 3B raw layout's norm and
    // bias positions, or cells holding f32 data
    auto is_1d = [&](uint64_t i) -> bool {
      if (count == 376853) {
        if (i == 376852) return true;
        if (i < 37984) return false;
        const uint64_t rel = (i - 37984) % 9413;
        if (rel == 0 || rel == 513 || rel == 578 || rel == 643 || rel == 1156) return true;
      }
      if (!src_raw) return cell_at(i)[CHPE_PAYLOAD_OFF + 20] == 32;
      return false;
    };
    const uint64_t chunk = 4096;  // tiles per round trip (64 MiB)
    uint8_t *h_buf = nullptr, *h_conv = nullptr, *d_conv = nullptr;
    uint16_t* d_buf = nullptr;
    cudaStream_t s = nullptr;
    auto ck = [&](cudaError_t e, const char* what) {
      if (e != cudaSuccess && result == 0) {
        result = fail(std::string(what) + ": " + cudaGetErrorString(e));
      }
      return e == cudaSuccess;
    };
    if (ck(cudaSetDevice(device), "cudaSetDevice") &&
        ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream") &&
        ck(cudaMallocHost(&h_buf, chunk * CHPE_TILE_CODE_BYTES), "pinned buffer") &&
        ck(cudaMallocHost(&h_conv, chunk), "pinned flags") &&
        ck(cudaMalloc(&d_buf, chunk * CHPE_TILE_CODE_BYTES), "device buffer") &&
        ck(cudaMalloc(&d_conv, chunk), "device flags")) {
      for (uint64_t t0 = 0; t0 < count && result == 0; t0 += chunk) {
        const uint64_t n = count - t0 < chunk ? count - t0 : chunk;
        for (uint64_t j = 0; j < n; j++) {
          memcpy(h_buf + j * CHPE_TILE_CODE_BYTES, tile_at(t0 + j), CHPE_TILE_CODE_BYTES);
          h_conv[j] = is_1d(t0 + j) ? 0 : 1;
        }
        if (!ck(cudaMemcpyAsync(d_buf, h_buf, n * CHPE_TILE_CODE_BYTES, cudaMemcpyHostToDevice, s), "H2D") ||
            !ck(cudaMemcpyAsync(d_conv, h_conv, n, cudaMemcpyHostToDevice, s), "H2D"))
          break;
        bf16_to_f16_tiles<<<(unsigned)n, 256, 0, s>>>(d_buf, d_conv, (uint32_t)n);
        if (!ck(cudaGetLastError(), "kernel launch") ||
            !ck(cudaMemcpyAsync(h_buf, d_buf, n * CHPE_TILE_CODE_BYTES, cudaMemcpyDeviceToHost, s), "D2H") ||
            !ck(cudaStreamSynchronize(s), "conversion"))
          break;
        memcpy(dst + CHPE_HEADER_BYTES + t0 * CHPE_TILE_CODE_BYTES, h_buf, n * CHPE_TILE_CODE_BYTES);
      }
    }
    if (d_buf) cudaFree(d_buf);
    if (d_conv) cudaFree(d_conv);
    if (h_buf) cudaFreeHost(h_buf);
    if (h_conv) cudaFreeHost(h_conv);
    if (s) cudaStreamDestroy(s);
  }
  if (msync(dm, out_len, MS_SYNC) != 0 && result == 0) result = fail("msync of the destination failed");
  munmap(dm, out_len);
  if (result == 0) chpe::set_thread_error("");
  return result;
}
