// Quantized-weight kernels: the reference unpack, GGUF block repacking, exact
// dequantisation and the seeded synthetic generators.  All are HBM-bound
// byte/integer work: coalesced 128-bit accesses, grids sized from the SM count.
#include "runtime.cuh"

namespace fg {

// Q4_0 device packing (common.cuh): codes of one 32-element block <-> its 4
// lane words.
__device__ __forceinline__ void q4_pack(const uint8_t code[32], uint32_t w[4]) {
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    uint32_t v = 0;
#pragma unroll
    for (int p = 0; p < 8; ++p) v |= (uint32_t)(code[q4_elem(t, p)] & 0xF) << (4 * p);
    w[t] = v;
  }
}
__device__ __forceinline__ void q4_unpack(const uint32_t w[4], uint8_t code[32]) {
#pragma unroll
  for (int t = 0; t < 4; ++t)
#pragma unroll
    for (int p = 0; p < 8; ++p) code[q4_elem(t, p)] = (w[t] >> (4 * p)) & 0xF;
}

// ---------------------------------------------------------------------------
// UNPACK_QUANT_WGSL main (packages/forge/src/tensor/kernels/unpack_quant.wgsl.ts:
// 25-62) with the graph path's dispatch (graphExecutor.ts:1313-1323):
// out[i] = (f32(code_i) - zero[i/gs]) * scale[i/gs].  One thread per u32 word
// (8 nibbles or 4 bytes), subtract and multiply rounded separately so the
// result is bit-identical to the reference arithmetic.
// ---------------------------------------------------------------------------
__global__ void k_unpack_quant(const uint32_t *__restrict__ packed, const float *__restrict__ scales,
                               const float *__restrict__ zeros, int bits, int64_t gs, int64_t n,
                               float *__restrict__ out) {
  const int per = bits == 4 ? 8 : 4;
  const int64_t words = (n + per - 1) / per;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < words; w += (int64_t)gridDim.x * blockDim.x) {
    uint32_t word = packed[w];
    int64_t i0 = w * per;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k >= per) break;
      int64_t i = i0 + k;
      if (i >= n) break;
      uint32_t code = bits == 4 ? (word >> (4 * k)) & 0xFu : (word >> (8 * k)) & 0xFFu;
      int64_t g = i / gs;
      out[i] = __fmul_rn(__fsub_rn((float)code, zeros[g]), scales[g]);
    }
  }
}

void launch_unpack_quant(const uint32_t *packed, const float *scales, const float *zeros, int bits, int64_t gs,
                         int64_t n, float *out, cudaStream_t s) {
  if (n <= 0) return;
  int64_t words = ceil_div(n, bits == 4 ? 8 : 4);
  int grid = (int)std::min<int64_t>(ceil_div(words, 256), 148 * 16);
  k_unpack_quant<<<grid, 256, 0, s>>>(packed, scales, zeros, bits, gs, n, out);
  FG_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// GGUF blocks <-> device layout.  GGUF Q4_0 block: fp16 d, then 16 bytes where
// byte j holds value j (low nibble) and value j+16 (high nibble).  Q8_0: fp16
// d then 32 int8.  Q8_0 on the device keeps the reference packing (element i
// in byte i%4 of word i/4, codes offset to unsigned) with a scale plane;
// Q4_0 goes into the tiled layout (common.cuh), whose lane-words are the GGUF
// qs words themselves.  One thread per block; the 18/34-byte source blocks
// are read bytewise.
// ---------------------------------------------------------------------------
__global__ void k_gguf_to_device(const uint8_t *__restrict__ src, QMat w, int64_t nblocks, int64_t nbr,
                                 int64_t dst_rs, int64_t dst_ro) {
  uint32_t *qs = const_cast<uint32_t *>(w.qs);
  __half *d = const_cast<__half *>(w.d);
  for (int64_t sb = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; sb < nblocks; sb += (int64_t)gridDim.x * blockDim.x) {
    // source block sb = (row r, column block cb); destination row r * dst_rs + dst_ro
    const int64_t drow = (sb / nbr) * dst_rs + dst_ro, cb = sb % nbr;
    const int64_t b = drow * nbr + cb;      // Q8_0 qs block index
    const int64_t db = qmat_scale_at(w, drow, cb);
    const int64_t src_b = sb;
    if (w.qtype == FG_Q4_0) {
      const uint8_t *blk = src + 18 * src_b;
      uint8_t code[32];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        code[j] = blk[2 + j] & 0xF;
        code[j + 16] = blk[2 + j] >> 4;
      }
      uint32_t ws[4];
      q4_pack(code, ws);
#pragma unroll
      for (int t = 0; t < 4; ++t) qs[q4_word_at(w, drow, cb, t)] = ws[t];
      d[db] = __ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8)));
    } else {
      const uint8_t *blk = src + 34 * src_b;
      uint32_t ws[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) word |= (uint32_t)(uint8_t)(blk[2 + 4 * t + k] ^ 0x80u) << (8 * k);
        ws[t] = word;
      }
      uint4 *o = reinterpret_cast<uint4 *>(qs) + 2 * b;
      o[0] = make_uint4(ws[0], ws[1], ws[2], ws[3]);
      o[1] = make_uint4(ws[4], ws[5], ws[6], ws[7]);
      d[db] = __ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8)));
    }
  }
}

void launch_gguf_to_device(const uint8_t *blocks, int qtype, int64_t N, int64_t K, const QMat &dst, int64_t dst_rs,
                           int64_t dst_ro, cudaStream_t s) {
  const int64_t nb = N * (K / 32);
  if (nb == 0) return;
  FG_REQUIRE(dst.K == K && dst.qtype == qtype && (N - 1) * dst_rs + dst_ro < dst.N, FG_ERR_SHAPE,
             "quant repack: destination does not fit");
  int grid = (int)std::min<int64_t>(ceil_div(nb, 256), 148 * 16);
  k_gguf_to_device<<<grid, 256, 0, s>>>(blocks, dst, nb, K / 32, dst_rs, dst_ro);
  FG_LAUNCH_CHECK();
}

__global__ void k_device_to_gguf(QMat w, int64_t nblocks, int64_t nbr, uint8_t *__restrict__ dst) {
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nblocks; b += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = b / nbr, cb = b % nbr;
    unsigned short dh = __half_as_ushort(w.d[qmat_scale_at(w, r, cb)]);
    if (w.qtype == FG_Q4_0) {
      uint8_t *blk = dst + 18 * b;
      blk[0] = dh & 0xFF;
      blk[1] = dh >> 8;
      uint32_t ws[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) ws[t] = w.qs[q4_word_at(w, r, cb, t)];
      uint8_t code[32];
      q4_unpack(ws, code);
#pragma unroll
      for (int j = 0; j < 16; ++j) blk[2 + j] = (uint8_t)(code[j] | (code[j + 16] << 4));
    } else {
      uint8_t *blk = dst + 34 * b;
      blk[0] = dh & 0xFF;
      blk[1] = dh >> 8;
      const uint32_t *q = w.qs + 8 * b;
#pragma unroll
      for (int j = 0; j < 32; ++j) blk[2 + j] = (uint8_t)(((q[j / 4] >> (8 * (j % 4))) & 0xFFu) ^ 0x80u);
    }
  }
}

void launch_device_to_gguf(const QMat &w, uint8_t *blocks, cudaStream_t s) {
  int64_t nb = w.N * (w.K / 32);
  if (nb == 0) return;
  int grid = (int)std::min<int64_t>(ceil_div(nb, 256), 148 * 16);
  k_device_to_gguf<<<grid, 256, 0, s>>>(w, nb, w.K / 32, blocks);
  FG_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// Exact dequantisation to fp32 [N, K]: (code - zero) * f32(d) with the same two
// roundings as the reference unpack on the mapped operands (zero 8 / 128).
// One thread per 32-value block; 8 x 16-byte stores.
// ---------------------------------------------------------------------------
__global__ void k_dequant(QMat w, int64_t nblocks, int64_t nbr, float *__restrict__ out) {
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nblocks; b += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = b / nbr, cb = b % nbr;
    const float sc = __half2float(w.d[qmat_scale_at(w, r, cb)]);
    float v[32];
    if (w.qtype == FG_Q4_0) {
      uint32_t ws[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) ws[t] = w.qs[q4_word_at(w, r, cb, t)];
      uint8_t code[32];
      q4_unpack(ws, code);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(__fsub_rn((float)code[j], 8.0f), sc);
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const uint32_t q = w.qs[r * w.row_words + cb * 8 + t];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[4 * t + k] = __fmul_rn(__fsub_rn((float)((q >> (8 * k)) & 0xFFu), 128.0f), sc);
      }
    }
    float4 *o = reinterpret_cast<float4 *>(out + 32 * b);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

void launch_dequant(const QMat &w, float *out, cudaStream_t s) {
  const int64_t nb = w.N * (w.K / 32);
  if (nb == 0) return;
  int grid = (int)std::min<int64_t>(ceil_div(nb, 128), 148 * 16);
  k_dequant<<<grid, 128, 0, s>>>(w, nb, w.K / 32, out);
  FG_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// Seeded synthetic data.
// ---------------------------------------------------------------------------
__global__ void k_synth_normal(uint64_t seed, uint64_t offset, int64_t n, float mean, float stdv, int f16,
                               void *out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float z = __fadd_rn(__fmul_rn(normal01(seed, offset + (uint64_t)i), stdv), mean);
    if (f16)
      ((__half *)out)[i] = __float2half_rn(z);
    else
      ((float *)out)[i] = z;
  }
}

void launch_synth_normal(uint64_t seed, uint64_t offset, int64_t n, float mean, float stdv, int dtype, void *out,
                         cudaStream_t s) {
  if (n <= 0) return;
  int grid = (int)std::min<int64_t>(ceil_div(n, 256), 148 * 32);
  k_synth_normal<<<grid, 256, 0, s>>>(seed, offset, n, mean, stdv, dtype == FG_F16, out);
  FG_LAUNCH_CHECK();
}

// ggml block recipe, one thread per 32-value block (value (r, c) = std *
// N01(seed, (row0 + r) * K + c)).  Q4_0: d = v_absmax / -8, code =
// min(15, trunc(v / d + 8.5)); Q8_0: d = absmax / 127, q = round(v / d).
__global__ void k_synth_quant(int qtype, int64_t N, int64_t K, uint64_t seed, int64_t row0, int64_t col0,
                              int64_t k_full, float stdv, int64_t dst_rs, int64_t dst_ro, QMat dst) {
  uint32_t *qs = const_cast<uint32_t *>(dst.qs);
  __half *dsc = const_cast<__half *>(dst.d);
  const int64_t nbr = K / 32;
  const int64_t nb = N * nbr;
  for (int64_t sb = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; sb < nb; sb += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = sb / nbr, cb = sb % nbr;
    const int64_t drow = r * dst_rs + dst_ro;
    const int64_t db = qmat_scale_at(dst, drow, cb);
    const uint64_t base = (uint64_t)(row0 + r) * (uint64_t)k_full + (uint64_t)col0 + (uint64_t)cb * 32;
    float v[32];
    float amax = 0.0f, vmax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      v[j] = __fmul_rn(normal01(seed, base + j), stdv);
      float a = fabsf(v[j]);
      if (a > amax) {
        amax = a;
        vmax = v[j];
      }
    }
    if (qtype == FG_Q4_0) {
      float dd = __fdiv_rn(vmax, -8.0f);
      float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
      uint8_t code[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        int c = __float2int_rz(__fadd_rn(__fmul_rn(v[j], id), 8.5f));
        code[j] = (uint8_t)(c > 15 ? 15 : c);
      }
      uint32_t w[4];
      q4_pack(code, w);
#pragma unroll
      for (int t = 0; t < 4; ++t) qs[q4_word_at(dst, drow, cb, t)] = w[t];
      dsc[db] = __float2half_rn(dd);
    } else {
      float dd = __fdiv_rn(amax, 127.0f);
      float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
      uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        int q = (int)roundf(__fmul_rn(v[j], id));
        w[j / 4] |= (uint32_t)(uint8_t)(q + 128) << (8 * (j % 4));
      }
      uint4 *o = reinterpret_cast<uint4 *>(qs + drow * dst.row_words) + 2 * cb;
      o[0] = make_uint4(w[0], w[1], w[2], w[3]);
      o[1] = make_uint4(w[4], w[5], w[6], w[7]);
      dsc[db] = __float2half_rn(dd);
    }
  }
}

void launch_synth_quant(int qtype, int64_t N, int64_t K, uint64_t seed, int64_t row0, int64_t col0, int64_t k_full,
                        float stdv, const QMat &dst, int64_t dst_rs, int64_t dst_ro, cudaStream_t s) {
  const int64_t nb = N * (K / 32);
  if (nb == 0) return;
  FG_REQUIRE(dst.K == K && dst.qtype == qtype && (N - 1) * dst_rs + dst_ro < dst.N, FG_ERR_SHAPE,
             "synthetic quant: destination does not fit");
  int grid = (int)std::min<int64_t>(ceil_div(nb, 128), 148 * 16);
  k_synth_quant<<<grid, 128, 0, s>>>(qtype, N, K, seed, row0, col0, k_full, stdv, dst_rs, dst_ro, dst);
  FG_LAUNCH_CHECK();
}

}  // namespace fg
