// GGUF k-quants (Q4_K, Q6_K): dequantisation and the fused dequant-GEMV / GEMM.
//
// Q4_K is the super-block format of llama.cpp's Q4_K_M files (ggml's
// published block_q4_K; the reference's quant path stops at its 4/8-bit
// unpack, so this extends it): 256 values in 8 sub-blocks of 32, 144 bytes =
// fp16 d, fp16 dmin, 12 bytes of 6-bit (scale, min) pairs, 128 bytes of
// nibbles; bytes 32c..32c+31 of the nibbles hold sub-block 2c (low nibbles)
// and 2c+1 (high nibbles).  value = (d * scale) * q - (dmin * min), two fp32
// products and one subtraction, rounded separately (no contraction), so the
// dequantised values are bit-identical to the CPU restatement.
//
// On the device the blocks stay in their GGUF order, row-major [N][K / 256]
// (144 = 9 x 16 bytes: every block starts 16-byte aligned).
//
// GEMV (M <= 8 activation rows): one warp per weight row.  Lane l takes the
// 4-byte nibble word l of each super-block -- sub-blocks 2(l/8) and
// 2(l/8) + 1, positions 4(l % 8) .. +3 -- so a warp reads the 128 nibble
// bytes as one coalesced 128-byte line plus the 16-byte header; the scale
// and min apply per lane before the one warp reduction at the end of the
// row.  Each warp streams its row through a 4-stage shared-memory ring of 8
// super-blocks per stage (16-byte cp.async copies), so ~3.4 KB per warp are
// in flight without holding registers.  HBM-bound: 144 bytes per 256 weights.  Larger M dequantises the
// matrix once and runs the fp32 GEMM.
#include "epilogue.cuh"
#include "runtime.cuh"
#include "tma.cuh"

namespace fg {
namespace {

__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *s, int &sc, int &m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// One thread per (super-block, nibble byte): two values.
__global__ void k_dequant_q4k(const uint8_t *__restrict__ blocks, int64_t n_blocks, float *__restrict__ out) {
  const int64_t n = n_blocks * 128;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t >> 7;
    const int byte = (int)(t & 127), c = byte >> 5, l = byte & 31;
    const uint8_t *blk = blocks + b * 144;
    const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(blk[2] | (blk[3] << 8))));
    int s0, m0, s1, m1;
    q4k_scale_min(2 * c, blk + 4, s0, m0);
    q4k_scale_min(2 * c + 1, blk + 4, s1, m1);
    const uint8_t q = blk[16 + byte];
    float *o = out + b * 256 + 64 * c + l;
    o[0] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s0), (float)(q & 0xF)), __fmul_rn(dmin, (float)m0));
    o[32] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s1), (float)(q >> 4)), __fmul_rn(dmin, (float)m1));
  }
}

// (scale, min) of sub-blocks 2c and 2c+1 from the header words y, z, w (scale bytes 0-3, 4-7, 8-11),
// packed as two bytes each (sc = sc(2c) | sc(2c+1) << 8, m likewise), by byte permutes: for c < 2 the
// 6 low bits of bytes 2c, 2c+1 (scales) and 2c+4, 2c+5 (mins); for c >= 2 bytes 2c+4, 2c+5 give the
// low 4 bits (scale: low nibble, min: high nibble) and the top 2 bits of bytes 2c-4, 2c-3 (scale) and
// 2c, 2c+1 (min) go above them.  A lane's c is fixed, so the selectors are loop-invariant.
__device__ __forceinline__ void q4k_pair(const uint4 &h, int c, uint32_t &sc, uint32_t &m) {
  const uint32_t cc = (uint32_t)c & 1;
  const uint32_t x = __byte_perm(h.y, h.z, (2 * cc) | ((2 * cc + 1) << 4) | ((4 + 2 * cc) << 8) | ((5 + 2 * cc) << 12));
  if (c < 2) {
    sc = x & 0x3F3Fu;
    m = (x >> 16) & 0x3F3Fu;
  } else {
    const uint32_t y = __byte_perm(h.w, 0u, (2 * cc) | ((2 * cc + 1) << 4));
    sc = (y & 0x0F0Fu) | ((x >> 2) & 0x3030u);
    m = ((y >> 4) & 0x0F0Fu) | ((x >> 18) & 0x3030u);
  }
}

// 4 warps (rows) per block: 4096-row matrices make ~7 blocks per SM, a smaller tail than 8-warp blocks
// (measured 6 % faster at b1, 16 % at b4 for 4096 x 11008).
constexpr int kQ4kWarps = 4;

// Per-warp shared-memory ring of the Q4_K GEMV: kQ4kStages stages of kQ4kU super-blocks, filled with
// 16-byte cp.async copies (no registers held for bytes in flight).
constexpr int kQ4kU = 8, kQ4kStages = 4;
constexpr int kQ4kStageBytes = kQ4kU * 144;                              // 1152
constexpr int kQ4kSmem = kQ4kWarps * kQ4kStages * kQ4kStageBytes;        // 18 KB per block

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int M>
__global__ void __launch_bounds__(kQ4kWarps * 32) k_gemv_q4k(const uint8_t *__restrict__ w, int64_t N, int64_t K,
                                                             const float *__restrict__ x, int64_t ldx,
                                                             float *__restrict__ y, int64_t ldy) {
  extern __shared__ __align__(16) unsigned char q4k_ring[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = (int64_t)blockIdx.x * kQ4kWarps + warp;
  if (row >= N) return;  // warps are independent: no block barrier follows
  const int64_t nb = K / 256;
  const uint8_t *wr = w + row * nb * 144;
  unsigned char *ring = q4k_ring + warp * kQ4kStages * kQ4kStageBytes;
  const int c = lane >> 3, p = 4 * (lane & 7);
  // stage s <- super-blocks [b0, b0 + kQ4kU) of the row: 9 chunks of 16 bytes each
  const auto issue = [&](int st, int64_t b0) {
    const int chunks = (int)(nb - b0 < kQ4kU ? nb - b0 : kQ4kU) * 9;
    for (int ch = lane; ch < chunks; ch += 32)
      cp_async16(ring + st * kQ4kStageBytes + ch * 16, wr + b0 * 144 + ch * 16);
  };
  float acc[M];
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = 0.0f;
#pragma unroll
  for (int st = 0; st < kQ4kStages - 1; ++st) {
    if ((int64_t)st * kQ4kU < nb) issue(st, (int64_t)st * kQ4kU);
    cp_async_commit();
  }
  int it = 0;
  for (int64_t b0 = 0; b0 < nb; b0 += kQ4kU, ++it) {
    const int64_t bn = b0 + (int64_t)(kQ4kStages - 1) * kQ4kU;
    if (bn < nb) issue((it + kQ4kStages - 1) % kQ4kStages, bn);
    cp_async_commit();
    cp_async_wait<kQ4kStages - 1>();  // this thread's copies of stage `it` have landed
    __syncwarp();                      // ... and every lane's
    const unsigned char *stg = ring + (it % kQ4kStages) * kQ4kStageBytes;
    const int nu = (int)(nb - b0 < kQ4kU ? nb - b0 : kQ4kU);
    for (int u = 0; u < nu; ++u) {
      const int64_t b = b0 + u;
      const uint4 hdr = *reinterpret_cast<const uint4 *>(stg + u * 144);
      const uint32_t qw = reinterpret_cast<const uint32_t *>(stg + u * 144 + 16)[lane];
      const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFF)));
      const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
      uint32_t scp, mp;
      q4k_pair(hdr, c, scp, mp);
      const int s0 = (int)(scp & 0xFF), s1 = (int)(scp >> 8), m0 = (int)(mp & 0xFF), m1 = (int)(mp >> 8);
      const float d0 = d * (float)s0, mm0 = dmin * (float)m0, d1 = d * (float)s1, mm1 = dmin * (float)m1;
      float lo[4], hi[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        lo[e] = (float)((qw >> (8 * e)) & 0xF);
        hi[e] = (float)((qw >> (8 * e + 4)) & 0xF);
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float *xb = x + m * ldx + b * 256 + 64 * c + p;
        const float4 xa = __ldg(reinterpret_cast<const float4 *>(xb));
        const float4 xc = __ldg(reinterpret_cast<const float4 *>(xb + 32));
        const float qa = lo[0] * xa.x + lo[1] * xa.y + lo[2] * xa.z + lo[3] * xa.w;
        const float sa = xa.x + xa.y + xa.z + xa.w;
        const float qc = hi[0] * xc.x + hi[1] * xc.y + hi[2] * xc.z + hi[3] * xc.w;
        const float sc = xc.x + xc.y + xc.z + xc.w;
        acc[m] += (d0 * qa - mm0 * sa) + (d1 * qc - mm1 * sc);
      }
    }
    __syncwarp();  // every lane is done with this stage before a later issue refills it
  }
  cp_async_wait<0>();
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const float v = warp_sum(acc[m]);
    if (lane == 0) y[m * ldy + row] = v;
  }
}

template <int M>
void gemv_q4k_launch(const uint8_t *w, int64_t N, int64_t K, const float *x, float *y, cudaStream_t s) {
  k_gemv_q4k<M><<<(unsigned)ceil_div(N, kQ4kWarps), kQ4kWarps * 32, kQ4kSmem, s>>>(w, N, K, x, K, y, N);
  FG_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ Q6_K
// 256 values in 210 bytes: ql[128] (low 4 bits), qh[64] (high 2 bits), int8
// scales[16], fp16 d.  Half h uses ql[64h..], qh[32h..], scales[8h..]; value
// l (+32, +64, +96) of a half takes the low nibble of ql[l] (low of ql[l+32],
// high of ql[l], high of ql[l+32]) with qh[l] bits 0-1 (2-3, 4-5, 6-7) on top,
// minus 32, times d * scales[l/16] (+2, +4, +6): two fp32 products.  Blocks
// stay in GGUF order (2-byte aligned); the GEMV reads them with 16-bit loads.
__device__ __forceinline__ float q6k_d(const uint8_t *blk) {
  return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short *>(blk + 208))));
}

// One thread per (super-block, half, l): four values.
__global__ void k_dequant_q6k(const uint8_t *__restrict__ blocks, int64_t n_blocks, float *__restrict__ out) {
  const int64_t n = n_blocks * 64;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t >> 6;
    const int h = (int)((t >> 5) & 1), l = (int)(t & 31), is = l >> 4;
    const uint8_t *blk = blocks + b * 210;
    const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
    const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * h);
    const float d = q6k_d(blk);
    const int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
    const int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
    const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
    const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
    float *o = out + b * 256 + 128 * h + l;
    o[0] = __fmul_rn(__fmul_rn(d, (float)sc[is]), (float)q1);
    o[32] = __fmul_rn(__fmul_rn(d, (float)sc[is + 2]), (float)q2);
    o[64] = __fmul_rn(__fmul_rn(d, (float)sc[is + 4]), (float)q3);
    o[96] = __fmul_rn(__fmul_rn(d, (float)sc[is + 6]), (float)q4);
  }
}

// GEMV: one warp per weight row; lane = (half h = lane / 16, positions 2 (lane % 16) and +1 of each
// quarter of the half), so a warp's 16-bit loads of ql and qh cover the block's 192 code bytes.
template <int M, int kU>
__global__ void __launch_bounds__(kQ4kWarps * 32) k_gemv_q6k(const uint8_t *__restrict__ w, int64_t N, int64_t K,
                                                             const float *__restrict__ x, int64_t ldx,
                                                             float *__restrict__ y, int64_t ldy) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kQ4kWarps + (threadIdx.x >> 5);
  if (row >= N) return;
  const int64_t nb = K / 256;
  const uint8_t *wr = w + row * nb * 210;
  const int h = lane >> 4, lp = 2 * (lane & 15), is = lp >> 4;
  float acc[M];
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = 0.0f;
  for (int64_t b0 = 0; b0 < nb; b0 += kU) {
    uint32_t qa[kU], qb[kU], qc[kU], sw[kU];
    float dd[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (b0 + u < nb) {
        const uint8_t *blk = wr + (b0 + u) * 210;
        qa[u] = __ldg(reinterpret_cast<const unsigned short *>(blk + 64 * h + lp));
        qb[u] = __ldg(reinterpret_cast<const unsigned short *>(blk + 64 * h + 32 + lp));
        qc[u] = __ldg(reinterpret_cast<const unsigned short *>(blk + 128 + 32 * h + lp));
        const uint8_t *sp = blk + 192 + 8 * h + is;
        sw[u] = (uint32_t)__ldg(sp) | ((uint32_t)__ldg(sp + 2) << 8) | ((uint32_t)__ldg(sp + 4) << 16) |
                ((uint32_t)__ldg(sp + 6) << 24);
        dd[u] = q6k_d(blk);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (b0 + u >= nb) break;
      const int64_t b = b0 + u;
      // the 6-bit codes of both positions at once, one per byte: quarter k takes the low (k = 0, 1) or
      // high (k = 2, 3) nibbles of ql word a (k even) or b (k odd), and bits 2k, 2k+1 of each qh byte
      // moved to bits 4, 5
      const uint32_t v[4] = {(qa[u] & 0x0F0Fu) | ((qc[u] << 4) & 0x3030u), (qb[u] & 0x0F0Fu) | ((qc[u] << 2) & 0x3030u),
                             ((qa[u] >> 4) & 0x0F0Fu) | (qc[u] & 0x3030u),
                             ((qb[u] >> 4) & 0x0F0Fu) | ((qc[u] >> 2) & 0x3030u)};
      float q[4][2];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        q[k][0] = (float)((int)(v[k] & 0xFF) - 32);
        q[k][1] = (float)((int)(v[k] >> 8) - 32);
      }
      float scf[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) scf[k] = (float)(int8_t)((sw[u] >> (8 * k)) & 0xFF);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float *xb = x + m * ldx + b * 256 + 128 * h + lp;
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 xv = __ldg(reinterpret_cast<const float2 *>(xb + 32 * k));
          sum = fmaf(scf[k], q[k][0] * xv.x + q[k][1] * xv.y, sum);
        }
        acc[m] = fmaf(dd[u], sum, acc[m]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const float v = warp_sum(acc[m]);
    if (lane == 0) y[m * ldy + row] = v;
  }
}

// kU = super-blocks whose loads are issued before any is used: 8 for rows of >= 32 super-blocks
// (K >= 8192; 4096 x 11008: 37.2 -> 33.0 us), 4 for shorter rows (11008 x 4096: 28.9 us vs 34.6 with 8).
template <int M>
void gemv_q6k_launch(const uint8_t *w, int64_t N, int64_t K, const float *x, float *y, cudaStream_t s) {
  const unsigned grid = (unsigned)ceil_div(N, kQ4kWarps);
  if (K / 256 >= 32)
    k_gemv_q6k<M, 8><<<grid, kQ4kWarps * 32, 0, s>>>(w, N, K, x, K, y, N);
  else
    k_gemv_q6k<M, 4><<<grid, kQ4kWarps * 32, 0, s>>>(w, N, K, x, K, y, N);
  FG_LAUNCH_CHECK();
}

}  // namespace

void launch_dequant_q6k(const void *blocks, int64_t n_blocks, float *out, cudaStream_t s) {
  if (n_blocks == 0) return;
  const int64_t n = n_blocks * 64;
  k_dequant_q6k<<<(unsigned)std::min<int64_t>(ceil_div(n, 256), 148 * 32), 256, 0, s>>>((const uint8_t *)blocks,
                                                                                        n_blocks, out);
  FG_LAUNCH_CHECK();
}

// y[M, N] = x[M, K] W^T, W Q6_K [N, K]; `scratch` (N K floats) is used when M > 8.
void launch_qmatmul_q6k(const void *w, int64_t N, int64_t K, const float *x, int64_t M, float *y, float *scratch,
                        cudaStream_t s) {
  if (M == 0 || N == 0) return;
  const uint8_t *wb = (const uint8_t *)w;
  switch (M) {
    case 1: return gemv_q6k_launch<1>(wb, N, K, x, y, s);
    case 2: return gemv_q6k_launch<2>(wb, N, K, x, y, s);
    case 3: return gemv_q6k_launch<3>(wb, N, K, x, y, s);
    case 4: return gemv_q6k_launch<4>(wb, N, K, x, y, s);
    case 5: return gemv_q6k_launch<5>(wb, N, K, x, y, s);
    case 6: return gemv_q6k_launch<6>(wb, N, K, x, y, s);
    case 7: return gemv_q6k_launch<7>(wb, N, K, x, y, s);
    case 8: return gemv_q6k_launch<8>(wb, N, K, x, y, s);
    default:
      launch_dequant_q6k(w, N * K / 256, scratch, s);
      launch_matmul_f32(x, scratch, y, M, K, N, s, /*b_trans=*/true);
  }
}

void launch_dequant_q4k(const void *blocks, int64_t n_blocks, float *out, cudaStream_t s) {
  if (n_blocks == 0) return;
  const int64_t n = n_blocks * 128;
  k_dequant_q4k<<<(unsigned)std::min<int64_t>(ceil_div(n, 256), 148 * 32), 256, 0, s>>>((const uint8_t *)blocks,
                                                                                        n_blocks, out);
  FG_LAUNCH_CHECK();
}

// y[M, N] = x[M, K] W^T, W Q4_K [N, K]; `scratch` (N K floats) is used when M > 8.
void launch_qmatmul_q4k(const void *w, int64_t N, int64_t K, const float *x, int64_t M, float *y, float *scratch,
                        cudaStream_t s) {
  if (M == 0 || N == 0) return;
  const uint8_t *wb = (const uint8_t *)w;
  switch (M) {
    case 1: return gemv_q4k_launch<1>(wb, N, K, x, y, s);
    case 2: return gemv_q4k_launch<2>(wb, N, K, x, y, s);
    case 3: return gemv_q4k_launch<3>(wb, N, K, x, y, s);
    case 4: return gemv_q4k_launch<4>(wb, N, K, x, y, s);
    case 5: return gemv_q4k_launch<5>(wb, N, K, x, y, s);
    case 6: return gemv_q4k_launch<6>(wb, N, K, x, y, s);
    case 7: return gemv_q4k_launch<7>(wb, N, K, x, y, s);
    case 8: return gemv_q4k_launch<8>(wb, N, K, x, y, s);
    default:
      launch_dequant_q4k(w, N * K / 256, scratch, s);
      launch_matmul_f32(x, scratch, y, M, K, N, s, /*b_trans=*/true);
  }
}

// ---------------------------------------------------------------------------
// Epilogue pass of a k-quant model layer.  The k-quant GEMVs write plain
// [M][N] outputs, so RoPE + fp16 KV append, SwiGLU and the residual add run
// as a second pass through the same epi_store_pair the fused Q4_0 kernels
// call, on the pair (v0, v1) of output columns (n, n + 1):
//  * QKV: columns [0, n0) of s0 (q), [n0, n0 + n1) of s1 (k), then s2 (v);
//  * interleave: pair p is (s0[m][p], s1[m][p]) at column 2p (gate, up);
//  * plain: columns of s0.
// ---------------------------------------------------------------------------
__global__ void k_kq_post(Epilogue ep, int M, int64_t npairs, const float *s0, int64_t n0, const float *s1,
                          int64_t n1, const float *s2, int mode) {
  const int64_t total = (int64_t)M * npairs;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / npairs);
    const int64_t p = i % npairs;
    float v0, v1;
    int64_t n;
    if (mode == 1) {  // interleave
      v0 = s0[(int64_t)m * npairs + p];
      v1 = s1[(int64_t)m * npairs + p];
      n = 2 * p;
    } else {
      n = 2 * p;
      const float *src;
      int64_t col, ld;
      if (mode == 0 && n >= n0 + n1) {
        src = s2, col = n - n0 - n1, ld = n1;
      } else if (mode == 0 && n >= n0) {
        src = s1, col = n - n0, ld = n1;
      } else {
        src = s0, col = n, ld = mode == 0 ? n0 : 2 * npairs;
      }
      v0 = src[(int64_t)m * ld + col];
      v1 = src[(int64_t)m * ld + col + 1];
    }
    epi_store_pair(ep, n, m, v0, v1);
  }
}

void launch_kq_post(const Epilogue &ep, int M, int64_t npairs, const float *s0, int64_t n0, const float *s1,
                    int64_t n1, const float *s2, int mode, cudaStream_t s) {
  const int64_t total = (int64_t)M * npairs;
  if (total == 0) return;
  const int grid = (int)std::min<int64_t>(ceil_div(total, 256), 148 * 16);
  k_kq_post<<<grid, 256, 0, s>>>(ep, M, npairs, s0, n0, s1, n1, s2, mode);
  FG_LAUNCH_CHECK();
}

}  // namespace fg
