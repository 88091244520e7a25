/*
 * forge_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, CPU restatement of AMEVA-Forge's quantized-LLM inference path
 * (uno-km/ameva-forge).  It is the parity checker for the CUDA library and
 * the timed CPU baseline; the product never links, loads or calls it.
 *
 * Each function cites the reference code whose arithmetic it restates
 * (paths relative to the reference project root).  Accumulations that the
 * reference performs in fp32 are carried in double here, so the oracle is
 * the "exact" side of every tolerance check.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).  Contraction
 * must stay off: the quantizers and the unpack are checked bit for bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define FO_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* Seeded synthetic data: splitmix64 counter generator + 4-term CLT normal.  */
/* The same integer recipe runs on the GPU (forge_b200 synth kernels); all   */
/* float steps are single IEEE operations, so both sides agree bit for bit.  */
/* ------------------------------------------------------------------------ */
#define FO_GOLDEN 0x9E3779B97F4A7C15ull
/* 1/sqrt(4 * (65536^2 - 1) / 12): unit variance for a sum of 4 uniforms.   */
#define FO_CLT4_SCALE 0x1.bb67aep-16f

static inline uint64_t fo_mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

FO_EXPORT uint64_t fo_splitmix64(uint64_t seed, uint64_t i) {
  return fo_mix64(seed + (i + 1) * FO_GOLDEN);
}

FO_EXPORT float fo_normal(uint64_t seed, uint64_t i) {
  uint64_t u = fo_splitmix64(seed, i);
  uint32_t s = (uint32_t)(u & 0xFFFF) + (uint32_t)((u >> 16) & 0xFFFF) +
               (uint32_t)((u >> 32) & 0xFFFF) + (uint32_t)(u >> 48);
  return ((float)s - 131070.0f) * FO_CLT4_SCALE;
}

/* out[i] = mean + std * normal(seed, offset + i) */
FO_EXPORT void fo_fill_normal(uint64_t seed, uint64_t offset, int64_t n, float mean,
                              float stdv, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    float z = fo_normal(seed, offset + (uint64_t)i) * stdv;
    out[i] = z + mean;
  }
}

/* ------------------------------------------------------------------------ */
/* IEEE binary16 <-> binary32, round to nearest even.                       */
/* ------------------------------------------------------------------------ */
FO_EXPORT uint16_t fo_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7FFFFFFFu;
  if (absx >= 0x7F800000u) { /* inf or nan */
    return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u | ((absx >> 13) & 0x3FFu) : 0u));
  }
  if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520 -> inf */
  if (absx < 0x38800000u) {                                  /* result is subnormal or zero */
    if (absx < 0x33000000u) return (uint16_t)sign;             /* < 2^-25 rounds to zero */
    uint32_t e = absx >> 23;
    uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126u - e; /* 14..24: value = m * 2^(e-150), unit = 2^-24 */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (absx >> 23) - 112u; /* rebias 127 -> 15 */
  uint32_t m = absx & 0x7FFFFFu;
  uint32_t h = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

FO_EXPORT float fo_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else { /* subnormal: normalise */
      e = 113;
      while (!(m & 0x400u)) { m <<= 1; e--; }
      x = sign | (e << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    x = sign | 0x7F800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

FO_EXPORT void fo_f32_to_f16_array(const float *in, int64_t n, uint16_t *out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = fo_f32_to_f16(in[i]);
}
FO_EXPORT void fo_f16_to_f32_array(const uint16_t *in, int64_t n, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = fo_f16_to_f32(in[i]);
}

/* ------------------------------------------------------------------------ */
/* GGUF block quantizers (ggml's published Q4_0 / Q8_0 reference recipe,    */
/* restated from its format description; ggml is not vendored by the        */
/* reference).  Block = 32 consecutive values of one row.                    */
/*   Q4_0: 18 B = fp16 d, 16 B qs; value j<16 in low nibble of qs[j], value  */
/*         j+16 in the high nibble; x ~= (code - 8) * d, d = signed absmax/-8.*/
/*   Q8_0: 34 B = fp16 d, 32 int8 q; x ~= q * d, d = absmax/127.             */
/* ------------------------------------------------------------------------ */
FO_EXPORT void fo_quantize_q4_0(const float *x, int64_t n_blocks, uint8_t *out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < n_blocks; ++b) {
    const float *v = x + 32 * b;
    uint8_t *blk = out + 18 * b;
    float amax = 0.0f, vmax = 0.0f;
    for (int j = 0; j < 32; ++j) {
      float a = fabsf(v[j]);
      if (a > amax) { amax = a; vmax = v[j]; }
    }
    float d = vmax / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = fo_f32_to_f16(d);
    blk[0] = (uint8_t)(dh & 0xFF);
    blk[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 16; ++j) {
      float t0 = v[j] * id;
      float t1 = v[j + 16] * id;
      t0 = t0 + 8.5f;
      t1 = t1 + 8.5f;
      int c0 = (int)(int8_t)t0; /* truncation, as the int8 cast of the recipe */
      int c1 = (int)(int8_t)t1;
      if (c0 > 15) c0 = 15;
      if (c1 > 15) c1 = 15;
      blk[2 + j] = (uint8_t)(c0 | (c1 << 4));
    }
  }
}

FO_EXPORT void fo_quantize_q8_0(const float *x, int64_t n_blocks, uint8_t *out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < n_blocks; ++b) {
    const float *v = x + 32 * b;
    uint8_t *blk = out + 34 * b;
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
      float a = fabsf(v[j]);
      if (a > amax) amax = a;
    }
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = fo_f32_to_f16(d);
    blk[0] = (uint8_t)(dh & 0xFF);
    blk[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 32; ++j) {
      float t = v[j] * id;
      blk[2 + j] = (uint8_t)(int8_t)roundf(t);
    }
  }
}

/* Code of value j (0..31) inside a Q4_0 block. */
static inline int fo_q4_code(const uint8_t *blk, int j) {
  return j < 16 ? (blk[2 + j] & 0xF) : (blk[2 + j - 16] >> 4);
}
static inline float fo_blk_scale(const uint8_t *blk) {
  return fo_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
}

/*
 * GGUF blocks -> the reference's generic unpack operands (packed u32 words,
 * per-group fp32 scales and zeros), the mapping under which
 * unpack_quant.wgsl.ts reproduces GGUF dequantisation exactly:
 *   Q4_0: bits 4, group 32, zero 8,   code i in nibble i%8 of word i/8;
 *   Q8_0: bits 8, group 32, zero 128, byte q+128 in byte i%4 of word i/4.
 */
FO_EXPORT void fo_gguf_to_ref(int qtype, const uint8_t *blocks, int64_t n_blocks,
                              uint32_t *packed, float *scales, float *zeros) {
  if (qtype == 4) {
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < n_blocks; ++b) {
      const uint8_t *blk = blocks + 18 * b;
      scales[b] = fo_blk_scale(blk);
      zeros[b] = 8.0f;
      for (int w = 0; w < 4; ++w) {
        uint32_t word = 0;
        for (int k = 0; k < 8; ++k) word |= (uint32_t)fo_q4_code(blk, 8 * w + k) << (4 * k);
        packed[4 * b + w] = word;
      }
    }
  } else {
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < n_blocks; ++b) {
      const uint8_t *blk = blocks + 34 * b;
      scales[b] = fo_blk_scale(blk);
      zeros[b] = 128.0f;
      for (int w = 0; w < 8; ++w) {
        uint32_t word = 0;
        for (int k = 0; k < 4; ++k)
          word |= (uint32_t)(uint8_t)((int)(int8_t)blk[2 + 4 * w + k] + 128) << (8 * k);
        packed[8 * b + w] = word;
      }
    }
  }
}

/*
 * Reference unpack: UNPACK_QUANT_WGSL main (packages/forge/src/tensor/
 * kernels/unpack_quant.wgsl.ts:25-62), graph dispatch graphExecutor.ts:
 * 1313-1323.  out[i] = (f32(code_i) - zero[g]) * scale[g], g = i / gs.
 */
FO_EXPORT void fo_unpack_quant(const uint32_t *packed, const float *scales, const float *zeros,
                               int bits, int64_t group_size, int64_t n, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    int64_t g = i / group_size;
    float raw = 0.0f;
    if (bits == 4) {
      raw = (float)((packed[i / 8] >> (4 * (i % 8))) & 0xFu);
    } else if (bits == 8) {
      raw = (float)((packed[i / 4] >> (8 * (i % 4))) & 0xFFu);
    }
    float t = raw - zeros[g];
    out[i] = t * scales[g];
  }
}

/* One GGUF block to 32 fp32 values: (code - 8) * d or q * d, one multiply. */
static inline void fo_dequant_block(int qtype, const uint8_t *blk, float *out) {
  float d = fo_blk_scale(blk);
  if (qtype == 4) {
    for (int j = 0; j < 32; ++j) out[j] = (float)(fo_q4_code(blk, j) - 8) * d;
  } else {
    for (int j = 0; j < 32; ++j) out[j] = (float)(int8_t)blk[2 + j] * d;
  }
}

/* GGUF dequantisation to fp32 (row-major, n_blocks*32 values). */
FO_EXPORT void fo_dequant(int qtype, const uint8_t *blocks, int64_t n_blocks, float *out) {
  int64_t bsz = qtype == 4 ? 18 : 34;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < n_blocks; ++b) fo_dequant_block(qtype, blocks + bsz * b, out + 32 * b);
}

/*
 * Quantized Linear, y[m, n] = sum_k x[m, k] * W[n, k] with W dequantised
 * exactly as above: nn.Linear.forward (packages/forge-py/src/forge/nn.py:
 * 248-259, x @ W^T) over the unpack_quant output.  Double accumulation.
 */
FO_EXPORT void fo_qmatmul(int qtype, const uint8_t *blocks, int64_t N, int64_t K, const float *x,
                          int64_t M, float *y) {
  int64_t nb = K / 32;
  int64_t bsz = qtype == 4 ? 18 : 34;
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t n = 0; n < N; ++n) {
    float wrow[32];
    double acc[16];
    for (int64_t m0 = 0; m0 < M; m0 += 16) {
      int64_t mc = M - m0 < 16 ? M - m0 : 16;
      for (int64_t m = 0; m < mc; ++m) acc[m] = 0.0;
      for (int64_t b = 0; b < nb; ++b) {
        fo_dequant_block(qtype, blocks + (n * nb + b) * bsz, wrow);
        for (int64_t m = 0; m < mc; ++m) {
          const float *xr = x + (m0 + m) * K + 32 * b;
          double s = 0.0;
          for (int j = 0; j < 32; ++j) s += (double)xr[j] * (double)wrow[j];
          acc[m] += s;
        }
      }
      for (int64_t m = 0; m < mc; ++m) y[(m0 + m) * N + n] = (float)acc[m];
    }
  }
}

/*
 * GGUF Q4_K super-block (the published ggml block_q4_K layout of llama.cpp's
 * Q4_K_M files; no counterpart in the reference, whose quant path is the
 * 4/8-bit unpack): 256 values in 8 sub-blocks of 32, 144 bytes = fp16 d,
 * fp16 dmin, 12 bytes of 6-bit (scale, min) pairs, 128 bytes of nibbles.
 * Bytes 32c..32c+31 of the nibbles hold sub-block 2c (low nibbles) and 2c+1
 * (high nibbles).  Pair j < 4: scale = s[j] & 63, min = s[j+4] & 63; j >= 4:
 * scale = (s[j+4] & 15) | (s[j-4] >> 6) << 4, min = (s[j+4] >> 4) | (s[j] >> 6) << 4.
 * value = (d * scale) * q - (dmin * min): two fp32 products, one subtraction.
 */
static inline void fo_q4k_scale_min(int j, const uint8_t *s, int *sc, int *m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

static inline void fo_dequant_q4k_block(const uint8_t *blk, float *out) {
  const float d = fo_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
  const float dmin = fo_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
  const uint8_t *sc = blk + 4, *qs = blk + 16;
  for (int c = 0; c < 4; ++c) {
    int s0, m0, s1, m1;
    fo_q4k_scale_min(2 * c, sc, &s0, &m0);
    fo_q4k_scale_min(2 * c + 1, sc, &s1, &m1);
    const float d0 = d * (float)s0, mm0 = dmin * (float)m0, d1 = d * (float)s1, mm1 = dmin * (float)m1;
    for (int l = 0; l < 32; ++l) {
      out[64 * c + l] = d0 * (float)(qs[32 * c + l] & 0xF) - mm0;
      out[64 * c + 32 + l] = d1 * (float)(qs[32 * c + l] >> 4) - mm1;
    }
  }
}

FO_EXPORT void fo_dequant_q4k(const uint8_t *blocks, int64_t n_blocks, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < n_blocks; ++b) fo_dequant_q4k_block(blocks + 144 * b, out + 256 * b);
}

/* y[m, n] = sum_k x[m, k] W[n, k], W Q4_K [N, K] dequantised as above; double accumulation. */
FO_EXPORT void fo_qmatmul_q4k(const uint8_t *blocks, int64_t N, int64_t K, const float *x, int64_t M, float *y) {
  const int64_t nb = K / 256;
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t n = 0; n < N; ++n) {
    float wrow[256];
    for (int64_t m = 0; m < M; ++m) {
      double acc = 0.0;
      for (int64_t b = 0; b < nb; ++b) {
        fo_dequant_q4k_block(blocks + (n * nb + b) * 144, wrow);
        const float *xr = x + m * K + 256 * b;
        for (int j = 0; j < 256; ++j) acc += (double)xr[j] * (double)wrow[j];
      }
      y[m * N + n] = (float)acc;
    }
  }
}

/*
 * GGUF Q6_K super-block (the published ggml block_q6_K layout, the other
 * k-quant of llama.cpp's Q4_K_M files): 256 values, 210 bytes = ql[128]
 * (low 4 bits), qh[64] (high 2 bits), int8 scales[16], fp16 d.  Half h of the
 * block (values 128h..128h+127) uses ql[64h..], qh[32h..], scales[8h..]; for
 * l < 32, values l, l+32, l+64, l+96 of the half take the low nibble of
 * ql[l], the low nibble of ql[l+32], the high nibble of ql[l], the high
 * nibble of ql[l+32], each with 2 bits of qh[l] (bits 0-1, 2-3, 4-5, 6-7) on
 * top, minus 32, and scales[l/16], [l/16+2], [l/16+4], [l/16+6].
 * value = (d * scale) * q: two fp32 products.
 */
static inline void fo_dequant_q6k_block(const uint8_t *blk, float *out) {
  const uint8_t *ql = blk, *qh = blk + 128;
  const int8_t *sc = (const int8_t *)(blk + 192);
  const float d = fo_f16_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
  for (int h = 0; h < 2; ++h) {
    for (int l = 0; l < 32; ++l) {
      const int is = l / 16;
      const int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
      const int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
      const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
      const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
      out[128 * h + l] = d * (float)sc[is] * (float)q1;
      out[128 * h + l + 32] = d * (float)sc[is + 2] * (float)q2;
      out[128 * h + l + 64] = d * (float)sc[is + 4] * (float)q3;
      out[128 * h + l + 96] = d * (float)sc[is + 6] * (float)q4;
    }
    ql += 64;
    qh += 32;
    sc += 8;
  }
}

FO_EXPORT void fo_dequant_q6k(const uint8_t *blocks, int64_t n_blocks, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < n_blocks; ++b) fo_dequant_q6k_block(blocks + 210 * b, out + 256 * b);
}

/* y[m, n] = sum_k x[m, k] W[n, k], W Q6_K [N, K] dequantised as above; double accumulation. */
FO_EXPORT void fo_qmatmul_q6k(const uint8_t *blocks, int64_t N, int64_t K, const float *x, int64_t M, float *y) {
  const int64_t nb = K / 256;
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t n = 0; n < N; ++n) {
    float wrow[256];
    for (int64_t m = 0; m < M; ++m) {
      double acc = 0.0;
      for (int64_t b = 0; b < nb; ++b) {
        fo_dequant_q6k_block(blocks + (n * nb + b) * 210, wrow);
        const float *xr = x + m * K + 256 * b;
        for (int j = 0; j < 256; ++j) acc += (double)xr[j] * (double)wrow[j];
      }
      y[m * N + n] = (float)acc;
    }
  }
}

/* Dense fp32 matmul C[M,N] = A[M,K] B[K,N]: cpuMatMul of
 * packages/forge/tests/matmul_tiled.test.ts:20 (double accumulation). */
FO_EXPORT void fo_matmul(const float *A, const float *B, int64_t M, int64_t K, int64_t N, float *C) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      double s = 0.0;
      for (int64_t k = 0; k < K; ++k) s += (double)A[m * K + k] * (double)B[k * N + n];
      C[m * N + n] = (float)s;
    }
  }
}

/*
 * Scaled dot-product attention with the reference's flash-attention
 * semantics (packages/forge/src/tensor/kernels/flash_attention.wgsl.ts:
 * 13-178; golden formula standardAttention in packages/forge/tests/
 * flash_attention.test.ts:18-76):
 *   GQA: kv_head = h / (H / H_kv)                          (wgsl :58-59)
 *   causal: key j visible iff j < N_kv - N_q + i + 1       (wgsl :92-96)
 *   out = sum_j p_j v_j / max(sum_j p_j, 1e-12)            (wgsl :160)
 * Q [B,H,Nq,d], K/V [B,Hkv,Nkv,d] (row strides given in elements so that a
 * KV cache with capacity > Nkv can be read in place), O [B,H,Nq,d].
 */
FO_EXPORT void fo_attention(const float *Q, const float *K, const float *V, float *O, int64_t B,
                            int64_t H, int64_t Hkv, int64_t Nq, int64_t Nkv, int64_t d,
                            int64_t kv_head_stride, float scale, int causal) {
  int64_t group = H / Hkv;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t h = 0; h < H; ++h) {
      int64_t kvh = h / group;
      const float *kb = K + (b * Hkv + kvh) * kv_head_stride;
      const float *vb = V + (b * Hkv + kvh) * kv_head_stride;
      double *s = (double *)malloc(sizeof(double) * (size_t)(Nkv > 0 ? Nkv : 1));
      double *acc = (double *)malloc(sizeof(double) * (size_t)d);
      for (int64_t i = 0; i < Nq; ++i) {
        const float *q = Q + ((b * H + h) * Nq + i) * d;
        int64_t lim = Nkv;
        if (causal) {
          int64_t c = Nkv - Nq + i + 1;
          lim = c < Nkv ? c : Nkv;
          if (lim < 0) lim = 0;
        }
        double mx = -1e30;
        for (int64_t j = 0; j < lim; ++j) {
          double dot = 0.0;
          for (int64_t c = 0; c < d; ++c) dot += (double)q[c] * (double)kb[j * d + c];
          s[j] = dot * (double)scale;
          if (s[j] > mx) mx = s[j];
        }
        double l = 0.0;
        for (int64_t c = 0; c < d; ++c) acc[c] = 0.0;
        for (int64_t j = 0; j < lim; ++j) {
          double p = exp(s[j] - mx);
          l += p;
          for (int64_t c = 0; c < d; ++c) acc[c] += p * (double)vb[j * d + c];
        }
        double inv = 1.0 / (l > 1e-12 ? l : 1e-12);
        float *o = O + ((b * H + h) * Nq + i) * d;
        for (int64_t c = 0; c < d; ++c) o[c] = (float)(acc[c] * inv);
      }
      free(s);
      free(acc);
    }
  }
}

/* RMSNorm: RMSNORM_WGSL (packages/forge/src/tensor/kernels/rmsnorm.wgsl.ts:
 * 10-74), cpuRMSNorm (packages/forge/tests/llm_generation_primitives.test.ts:
 * 56-75).  out = x / sqrt(mean(x^2) + eps) * gamma (gamma optional). */
FO_EXPORT void fo_rmsnorm(const float *x, const float *gamma, int64_t tokens, int64_t dim, float eps,
                          float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < tokens; ++t) {
    const float *r = x + t * dim;
    double ss = 0.0;
    for (int64_t i = 0; i < dim; ++i) ss += (double)r[i] * (double)r[i];
    double inv = 1.0 / sqrt(ss / (double)dim + (double)eps);
    for (int64_t i = 0; i < dim; ++i) {
      double v = (double)r[i] * inv;
      if (gamma) v *= (double)gamma[i];
      out[t * dim + i] = (float)v;
    }
  }
}

/* Inverse frequencies of the interleaved RoPE, base^(-2p/d), rounded to fp32
 * (the reference evaluates theta in fp32: rope.wgsl.ts:46-47). */
FO_EXPORT void fo_rope_inv_freq(float base, int64_t d, float *inv_freq) {
  for (int64_t p = 0; p < d / 2; ++p)
    inv_freq[p] = (float)pow((double)base, -2.0 * (double)p / (double)d);
}

/* Interleaved-pair RoPE: ROPE_WGSL (packages/forge/src/tensor/kernels/
 * rope.wgsl.ts:11-62), F.rope CPU branch (packages/forge-py/src/forge/
 * functional.py:839-861).  Pair p rotates elements (2p, 2p+1) by
 * theta = fp32(inv_freq[p] * (n + offset)).  x is [rows, N, d] with rows = B*H. */
FO_EXPORT void fo_rope(const float *x, int64_t rows, int64_t N, int64_t d, float base,
                       int64_t offset, float *out) {
  float inv_freq[512];
  fo_rope_inv_freq(base, d, inv_freq);
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t n = 0; n < N; ++n) {
      float pos = (float)(n + offset);
      const float *v = x + (r * N + n) * d;
      float *o = out + (r * N + n) * d;
      for (int64_t p = 0; p < d / 2; ++p) {
        float theta = inv_freq[p] * pos;
        double c = cos((double)theta), s = sin((double)theta);
        double v0 = v[2 * p], v1 = v[2 * p + 1];
        o[2 * p] = (float)(v0 * c - v1 * s);
        o[2 * p + 1] = (float)(v1 * c + v0 * s);
      }
    }
  }
}

/* SwiGLU: SWIGLU_WGSL (packages/forge/src/tensor/kernels/swiglu.wgsl.ts:
 * 11-42): out = gate / (1 + exp(-gate)) * up. */
FO_EXPORT void fo_swiglu(const float *gate, const float *up, int64_t n, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    double g = gate[i];
    out[i] = (float)(g / (1.0 + exp(-g)) * (double)up[i]);
  }
}

/* Embedding gather: EMBEDDING_WGSL (packages/forge/src/tensor/kernels/
 * embedding.wgsl.ts:20-63); an id outside [0, vocab) yields a zero row. */
FO_EXPORT void fo_embedding(const float *table, int64_t vocab, int64_t dim, const int32_t *ids,
                            int64_t n, float *out) {
  for (int64_t t = 0; t < n; ++t) {
    int32_t id = ids[t];
    if (id < 0 || id >= vocab) {
      memset(out + t * dim, 0, sizeof(float) * (size_t)dim);
    } else {
      memcpy(out + t * dim, table + (int64_t)id * dim, sizeof(float) * (size_t)dim);
    }
  }
}

/* Greedy pick: LLMSampler.sample temperature<=1e-5 branch (packages/forge/
 * src/tensor/sampling.ts:45-55): first index of the maximum (strict >). */
FO_EXPORT int64_t fo_argmax(const float *logits, int64_t n) {
  int64_t best = 0;
  float v = logits[0];
  for (int64_t i = 1; i < n; ++i) {
    if (logits[i] > v) { v = logits[i]; best = i; }
  }
  return best;
}

FO_EXPORT int fo_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
