// Shared definitions of the forge_b200 CUDA library (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "../../include/forge_b200.h"

namespace fg {

// Internal failures travel as exceptions and become a status code plus a
// thread-local message at the C-ABI boundary (capi.cu).
struct Error : std::runtime_error {
  int status;
  Error(int s, const std::string &m) : std::runtime_error(m), status(s) {}
};

[[noreturn]] inline void raise(int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  throw Error(status, buf);
}

// Sticky CUDA errors poison the context: they map to DeviceLost, the rest to
// InternalGPU (the reference maps WebGPU "internal" scopes the same way,
// graphExecutor.ts:1877-1933).
inline bool cuda_error_is_sticky(cudaError_t e) {
  switch (e) {
    case cudaErrorIllegalAddress:
    case cudaErrorIllegalInstruction:
    case cudaErrorMisalignedAddress:
    case cudaErrorInvalidAddressSpace:
    case cudaErrorInvalidPc:
    case cudaErrorLaunchFailure:
    case cudaErrorHardwareStackError:
    case cudaErrorAssert:
    case cudaErrorLaunchTimeout:
    case cudaErrorECCUncorrectable:
    case cudaErrorDevicesUnavailable:
      return true;
    default:
      return false;
  }
}

[[noreturn]] inline void raise_cuda(cudaError_t e, const char *what, const char *file, int line) {
  int st = e == cudaErrorMemoryAllocation ? FG_ERR_OUT_OF_MEMORY
           : cuda_error_is_sticky(e)      ? FG_ERR_DEVICE_LOST
           : (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) ? FG_ERR_UNAVAILABLE
                                                                          : FG_ERR_INTERNAL_GPU;
  raise(st, "%s failed: %s (%s:%d)", what, cudaGetErrorString(e), file, line);
}

#define FG_CUDA(call)                                                      \
  do {                                                                     \
    cudaError_t fg_e_ = (call);                                            \
    if (fg_e_ != cudaSuccess) ::fg::raise_cuda(fg_e_, #call, __FILE__, __LINE__); \
  } while (0)

#define FG_LAUNCH_CHECK() FG_CUDA(cudaGetLastError())

#define FG_REQUIRE(cond, status, ...)          \
  do {                                         \
    if (!(cond)) ::fg::raise(status, __VA_ARGS__); \
  } while (0)

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline uint64_t align_up(uint64_t a, uint64_t b) { return (a + b - 1) / b * b; }

// ---------------------------------------------------------------- generator
// splitmix64 counter generator + 4-term central-limit normal.  Every float
// step is one explicitly rounded IEEE operation, so host and device agree bit
// for bit with the CPU oracle's recipe.
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;
constexpr float kClt4Scale = 0x1.bb67aep-16f;  // 1/sqrt(4 (2^32 - 1) / 12)

__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t splitmix64(uint64_t seed, uint64_t i) { return mix64(seed + (i + 1) * kGolden); }

__device__ inline float normal01(uint64_t seed, uint64_t i) {
  uint64_t u = splitmix64(seed, i);
  uint32_t s = (uint32_t)(u & 0xFFFF) + (uint32_t)((u >> 16) & 0xFFFF) + (uint32_t)((u >> 32) & 0xFFFF) +
               (uint32_t)(u >> 48);
  return __fmul_rn(__fsub_rn((float)s, 131070.0f), kClt4Scale);
}

// ---------------------------------------------------------------- quant layout
// A quantized [N, K] matrix lives in one allocation.
//
// Q8_0 -- qs: the reference unpack packing (unpack_quant.wgsl.ts:44-51), byte
//   i%4 of u32 word i/4 of a row holds q + 128 for element i; d: fp16 scale
//   per 32-element block, [N][ldd] after qs (256-byte aligned), rows padded to
//   a multiple of 8 scales (16 bytes) for the TMA row pitch.
//
// Q4_0 -- row strips of 16 rows, so that one GEMV worker owns whole output
//   rows (no cross-CTA reduction).  A strip stores its blocks in quads of 4
//   (blocks past K/32, up to a multiple of 4, are zero; rows past N are
//   zero); quad Q of strip s is 1152 bytes at (s * quads_per_strip + Q) * 1152:
//     bytes [0, 1024): codes (q + 8), u32 word (r * 4 + t) * 4 + i = lane-word
//       t of block 4Q + i of row 16s + r.  Lane-word t of a block is GGUF
//       bytes 4t..4t+3 of its qs: the low nibble of byte i holds element
//       4t + i and the high nibble element 16 + 4t + i (q4_elem) -- the k
//       order of the int8 A fragments of mma.sync m16n8k32 (a0/a1: k =
//       4t..4t+3, a2/a3: k = 16+4t..16+4t+3), so a mask (and a shift) turns
//       a word into two fragment registers, and the lane (row g, word t) of
//       an MMA reads one 16-byte word group of 4 blocks;
//     bytes [1024, 1152): fp16 scales, [16 rows][4 blocks].
//   The GEMV streams a strip as tiles of up to 16 quads (18,432 bytes), each
//   one contiguous bulk copy.
constexpr int kQ4StripRows = 16, kQ4QuadBytes = 1152, kQ4TileQuads = 16;
constexpr int kQ4QuadCodeBytes = 1024;
constexpr int kQ4TileBytes = kQ4TileQuads * kQ4QuadBytes;
struct QMat {
  const uint32_t *qs;
  const __half *d;    // Q4_0: the allocation base (scales sit inside the quads)
  int32_t qtype;      // FG_Q4_0 / FG_Q8_0
  int64_t N, K;
  int64_t ldd;        // Q8_0: scales per d row (K/32 rounded up to 8)
  int64_t row_words;  // Q8_0: u32 words per qs row; Q4_0: quads per strip
};
__host__ __device__ inline int64_t qmat_ldd(int64_t K) { return (K / 32 + 7) / 8 * 8; }
__host__ __device__ inline int64_t q4_quads(int64_t K) { return (K / 32 + 3) / 4; }
__host__ __device__ inline int64_t q4_strips(int64_t N) { return (N + kQ4StripRows - 1) / kQ4StripRows; }
__host__ __device__ inline int64_t q4_tiles(int64_t K) { return (q4_quads(K) + kQ4TileQuads - 1) / kQ4TileQuads; }
__host__ __device__ inline int64_t qmat_row_words(int qtype, int64_t K) {
  return qtype == FG_Q4_0 ? q4_quads(K) : K / 4;
}
// Block element held by nibble p of lane-word t (Q4_0 device packing).
__host__ __device__ inline int q4_elem(int t, int p) { return 4 * t + (p >> 1) + 16 * (p & 1); }
// Q4_0: byte offset of quad Q of the strip holding row n.
__host__ __device__ inline int64_t q4_quad_off(const QMat &w, int64_t n, int64_t Q) {
  return ((n / kQ4StripRows) * w.row_words + Q) * kQ4QuadBytes;
}
// Q4_0: u32 index (from qs) of lane-word t of block b of row n.
__host__ __device__ inline int64_t q4_word_at(const QMat &w, int64_t n, int64_t b, int t) {
  return (q4_quad_off(w, n, b >> 2) + ((n % kQ4StripRows) * 4 + t) * 16 + (b & 3) * 4) / 4;
}
// fp16 scale index (from d) of block b of row n, both layouts.
__host__ __device__ inline int64_t qmat_scale_at(const QMat &w, int64_t n, int64_t b) {
  if (w.qtype != FG_Q4_0) return n * w.ldd + b;
  return (q4_quad_off(w, n, b >> 2) + kQ4QuadCodeBytes + ((n % kQ4StripRows) * 4 + (b & 3)) * 2) / 2;
}
inline uint64_t qmat_qs_bytes(int qtype, int64_t N, int64_t K) {
  if (qtype == FG_Q4_0) return (uint64_t)q4_strips(N) * (uint64_t)q4_quads(K) * kQ4QuadBytes;
  return (uint64_t)N * (uint64_t)qmat_row_words(qtype, K) * 4;
}
inline uint64_t qmat_d_offset(int qtype, int64_t N, int64_t K) { return align_up(qmat_qs_bytes(qtype, N, K), 256); }
inline uint64_t qmat_bytes(int qtype, int64_t N, int64_t K) {
  if (qtype == FG_Q4_0) return qmat_qs_bytes(qtype, N, K);
  return qmat_d_offset(qtype, N, K) + (uint64_t)N * (uint64_t)qmat_ldd(K) * 2;
}
inline QMat qmat_at(void *base, int qtype, int64_t N, int64_t K) {
  QMat q;
  q.qtype = qtype;
  q.N = N;
  q.K = K;
  q.ldd = qtype == FG_Q4_0 ? 0 : qmat_ldd(K);
  q.row_words = qmat_row_words(qtype, K);
  q.qs = (const uint32_t *)base;
  q.d = qtype == FG_Q4_0 ? (const __half *)base : (const __half *)((const char *)base + qmat_d_offset(qtype, N, K));
  return q;
}
inline int gguf_block_bytes(int qtype) { return qtype == FG_Q4_0 ? 18 : 34; }

// ---------------------------------------------------------------- device helpers
__device__ inline float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ inline float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streaming 128-bit load that bypasses L1 allocation (weights are read once).
__device__ inline uint4 ld_stream_u4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace fg
