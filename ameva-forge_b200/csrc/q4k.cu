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
#include <cstdlib>

#include "q4_gemv.cuh"
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


// ---------------------------------------------------------------------------
// Q4_K GEMV on integer tensor cores (M <= 4 activation rows): the Q4_0
// design (q4_gemv.cuh) on GGUF-ordered Q4_K rows.
//  * Units are 16-row strips; a tile is 16 rows x 8 super-blocks, one bulk
//    copy per row into a ring slot whose rows are 16 bytes apart beyond their
//    1152 data bytes, so the 8 rows x 4 words an MMA fragment load touches
//    fall in 32 different banks.
//  * Warp w takes super-block w of a tile: sub-block j = 2c + h is nibble h of
//    code bytes 32c .. 32c + 31, i.e. element k of the sub-block is nibble h
//    of byte 32c + k -- the k order of the u8 A fragment of mma.sync
//    m16n8k32, so each fragment register is a masked 32-bit load.
//  * x is staged exactly as for Q4_0 (per-block power-of-two scale 2^e,
//    22-bit integer v split into three s8 digits); the MMA input C is 0, so
//    D = sum_k q_k digit_k.  A sub-block contributes
//      2^-e (s * sum q v - o * sum v),  s = d * scale, o = dmin * min,
//    with sum v per block and token taken from the staged digit sums.  Lane t
//    decodes the (scale, min) pairs of sub-blocks 2t, 2t + 1 of its two rows
//    (the byte permutes of q4k_pair) and the quad of lanes shares them by
//    shuffles.
// Bound: HBM, 144 bytes per 256 weights (+ x).
// ---------------------------------------------------------------------------
constexpr int kKmWarps = 8;                          // consumer warps
constexpr int kKmThreads = (kKmWarps + 1) * 32;      // + the producer warp
constexpr int kKmTileSb = 8;                         // super-blocks per tile row
constexpr int kKmRowStride = kKmTileSb * 144 + 16;   // 1168: rows 4 banks apart
constexpr int kKmTileBytes = 16 * kKmRowStride;      // 18688

template <int MV>
size_t q4k_mma_smem(int64_t K, int stages) {
  const int nb = (int)(K / 32);
  return 128 + (size_t)stages * kKmTileBytes + Q4X<MV>::bytes(nb) + (size_t)MV * nb * 4 +
         (size_t)2 * kKmWarps * kQ4StripRows * MV * 4;
}

template <int MV, int STAGES>
__global__ void __launch_bounds__(kKmThreads, 2)
    k_gemv_q4k_mma(const uint8_t *__restrict__ w, int64_t N, int64_t K, const float *__restrict__ x, int64_t ldx,
                   float *__restrict__ y, int64_t ldy, int *err) {
  constexpr int NM = Q4X<MV>::NM;
  extern __shared__ __align__(128) unsigned char km_smem[];
  unsigned char *ring = km_smem + ((128 - (smem_u32(km_smem) & 127)) & 127);
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES];
  __shared__ float s_sum[kKmWarps * MV];
  __shared__ float s_one[MV];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nsb = (int)(K / 256), nb = nsb * 8;
  const int ntile = (nsb + kKmTileSb - 1) / kKmTileSb;
  const Sched sc = make_sched(N, kQ4StripRows, 1, blockIdx.x, gridDim.x);
  Q4X<MV> X;
  X.carve(ring + STAGES * kKmTileBytes, nb, nb);
  float *fsv = reinterpret_cast<float *>(ring + STAGES * kKmTileBytes + Q4X<MV>::bytes(nb));  // [MV][nb]: sum v / 128
  float *red = fsv + MV * nb;                                                                // [2][8][16][MV]

  if (tid == 0) {
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kKmWarps);
    }
    fence_barrier_init();
  }
  if (tid < MV) s_one[tid] = 1.0f;
  __syncthreads();

  if (warp == kKmWarps) {
    // ---------------- producer: the tiles of strips [u0, u1), one bulk copy per row
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int i = 0;
      bool ok = true;
      for (int u = sc.u0; u < sc.u1 && ok; ++u) {
        const int nrows = (int)(N - (int64_t)u * kQ4StripRows < kQ4StripRows ? N - (int64_t)u * kQ4StripRows : kQ4StripRows);
        for (int tl = 0; tl < ntile && ok; ++tl, ++i) {
          const int st = i % STAGES;
          if (i >= STAGES && !mbar_wait(&empty[st], (uint32_t)(i / STAGES - 1) & 1, err, DEVERR_GEMV_EMPTY)) {
            ok = false;
            break;
          }
          const int nst = min(kKmTileSb, nsb - tl * kKmTileSb);
          mbar_arrive_expect_tx(&full[st], (uint32_t)(nrows * nst * 144));
          for (int r = 0; r < nrows; ++r)
            bulk_g2s(ring + st * kKmTileBytes + r * kKmRowStride,
                     w + (((int64_t)u * kQ4StripRows + r) * nsb + (int64_t)tl * kKmTileSb) * 144,
                     (uint32_t)(nst * 144), &full[st], pol);
        }
      }
      drain_ring<STAGES>(full, i, err);
    }
    return;
  }

  // ---------------- stage x; the blocks' digit sums for the min term
  constexpr int kC = kKmWarps * 32;
  q4_stage_x<MV>(X, x, ldx, nullptr, tid, kC, s_sum);
  named_sync(kC);
  for (int e = tid; e < MV * nb; e += kC) {
    const int m = e / nb, b = e % nb;
    // staged MMA offsets are -8 x (digit sums): sum v = 2^14 sum hi + 2^7 sum mid + sum lo
    const int sv = -(X.cx0[(2 * m) * nb + b] * 16384 + X.cx1[(2 * m) * nb + b] * 128 + X.cx0[(2 * m + 1) * nb + b]) / 8;
    fsv[e] = (float)sv * 0.0078125f;
  }
  named_sync(kC);

  // ---------------- consume
  Q4Lane<MV> L;
  L.init(X, lane);
  const int gq = lane >> 2, t = lane & 3;
  const float evn = (t & 1) ? 0.0f : 1.0f;  // lanes of the (hi, mid) columns carry the min term
  const float *fbp[NM], *fsp[NM];
#pragma unroll
  for (int im = 0; im < NM; ++im) {
    const int tok = min(2 * im + (t >> 1), MV - 1);  // padding tokens' columns are dropped at the end
    fbp[im] = X.fbk + tok * nb;
    fsp[im] = fsv + tok * nb;
  }
  QMat wq;
  wq.N = N;
  Epilogue ep;
  ep.mode = EPI_PLAIN;
  ep.y = y;
  ep.ldy = ldy;
  float2 acc[NM];
#pragma unroll
  for (int im = 0; im < NM; ++im) acc[im] = make_float2(0.0f, 0.0f);
  bool ok = true;
  int i = 0;
  for (int u = sc.u0; u < sc.u1; ++u) {
    for (int tl = 0; tl < ntile; ++tl, ++i) {
      const int st = i % STAGES;
      ok = ok && mbar_wait(&full[st], (uint32_t)(i / STAGES) & 1, err, DEVERR_GEMV_FULL);
      const int sbg = tl * kKmTileSb + warp;
      if (ok && sbg < nsb) {
        const unsigned char *r0 = ring + st * kKmTileBytes + gq * kKmRowStride + warp * 144, *r1 = r0 + 8 * kKmRowStride;
        const uint4 h0 = *reinterpret_cast<const uint4 *>(r0), h1 = *reinterpret_cast<const uint4 *>(r1);
        uint32_t sc0, mn0, sc1, mn1;
        q4k_pair(h0, t, sc0, mn0);
        q4k_pair(h1, t, sc1, mn1);
        const float d0 = __half2float(__ushort_as_half((unsigned short)(h0.x & 0xFFFF)));
        const float dm0 = __half2float(__ushort_as_half((unsigned short)(h0.x >> 16)));
        const float d1 = __half2float(__ushort_as_half((unsigned short)(h1.x & 0xFFFF)));
        const float dm1 = __half2float(__ushort_as_half((unsigned short)(h1.x >> 16)));
        // [row][sub-block 2t + hh]: s = d * scale, o = dmin * min
        const float sv0[2] = {d0 * (float)(sc0 & 0xFF), d0 * (float)(sc0 >> 8)};
        const float ov0[2] = {dm0 * (float)(mn0 & 0xFF), dm0 * (float)(mn0 >> 8)};
        const float sv1[2] = {d1 * (float)(sc1 & 0xFF), d1 * (float)(sc1 >> 8)};
        const float ov1[2] = {dm1 * (float)(mn1 & 0xFF), dm1 * (float)(mn1 >> 8)};
        const int b0 = sbg * 8;
        float4 FB[NM][2], SV[NM][2];
#pragma unroll
        for (int im = 0; im < NM; ++im)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            FB[im][hf] = *reinterpret_cast<const float4 *>(fbp[im] + b0 + 4 * hf);
            SV[im][hf] = *reinterpret_cast<const float4 *>(fsp[im] + b0 + 4 * hf);
          }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t w00 = *reinterpret_cast<const uint32_t *>(r0 + 16 + 32 * c + 4 * t);
          const uint32_t w01 = *reinterpret_cast<const uint32_t *>(r0 + 32 + 32 * c + 4 * t);
          const uint32_t w10 = *reinterpret_cast<const uint32_t *>(r1 + 16 + 32 * c + 4 * t);
          const uint32_t w11 = *reinterpret_cast<const uint32_t *>(r1 + 32 + 32 * c + 4 * t);
          const int src = (lane & ~3) | c;  // the lane holding sub-blocks 2c, 2c + 1 of these rows
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int j = 2 * c + hh, b = b0 + j;
            const float sa = __shfl_sync(0xffffffffu, sv0[hh], src), sb = __shfl_sync(0xffffffffu, sv1[hh], src);
            const float oa = __shfl_sync(0xffffffffu, ov0[hh], src), ob = __shfl_sync(0xffffffffu, ov1[hh], src);
            const uint32_t a0 = hh ? (w00 >> 4) & 0x0F0F0F0Fu : w00 & 0x0F0F0F0Fu;
            const uint32_t a1 = hh ? (w10 >> 4) & 0x0F0F0F0Fu : w10 & 0x0F0F0F0Fu;
            const uint32_t a2 = hh ? (w01 >> 4) & 0x0F0F0F0Fu : w01 & 0x0F0F0F0Fu;
            const uint32_t a3 = hh ? (w11 >> 4) & 0x0F0F0F0Fu : w11 & 0x0F0F0F0Fu;
#pragma unroll
            for (int im = 0; im < NM; ++im) {
              uint2 B = make_uint2(0u, 0u);
              if (L.xv[im]) B = L.xl[im][b * 3 * MV * 4];
              int di[4];
              imma_u8s8(di, a0, a1, a2, a3, B.x, B.y, 0, 0);
              const float vx = (float)(di[0] * 128 + di[1]), vy = (float)(di[2] * 128 + di[3]);
              const float4 &f4 = FB[im][j >> 2];
              const float4 &s4 = SV[im][j >> 2];
              const float fb = (j & 3) == 0 ? f4.x : (j & 3) == 1 ? f4.y : (j & 3) == 2 ? f4.z : f4.w;
              const float sv = evn * ((j & 3) == 0 ? s4.x : (j & 3) == 1 ? s4.y : (j & 3) == 2 ? s4.z : s4.w);
              const float2 r = make_float2(fmaf(sa, vx, -oa * sv), fmaf(sb, vy, -ob * sv));
              acc[im] = ffma2(make_float2(fb, fb), r, acc[im]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    float *rb = red + ((u - sc.u0) & 1) * (kKmWarps * kQ4StripRows * MV);
    q4_group_red<MV>(rb, acc, warp, lane);
    named_sync(kC);
    if (ok) finish_strip<MV>(wq, ep, u, rb, s_one, tid, kC);
  }
}

int q4k_num_sms() {
  static int sms[64] = {0};
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) FG_CUDA(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
  return sms[dev];
}

// Shared memory per CTA up to which two CTAs share an SM, and the most one CTA may take.
constexpr size_t kKmSmemTwo = 112 * 1024, kKmSmemOne = 225 * 1024;

// Ring depth: 4 stages, or 3 where only that keeps two CTAs per SM or fits one; 0: x of MV tokens does not
// fit beside a 3-stage ring (the CUDA-core GEMV takes the call).
template <int MV>
int q4k_mma_stages(int64_t K) {
  if (q4k_mma_smem<MV>(K, 4) <= kKmSmemTwo) return 4;
  if (q4k_mma_smem<MV>(K, 3) <= kKmSmemTwo) return 3;
  if (q4k_mma_smem<MV>(K, 4) <= kKmSmemOne) return 4;
  return q4k_mma_smem<MV>(K, 3) <= kKmSmemOne ? 3 : 0;
}

template <int MV>
void gemv_q4k_mma_launch(const uint8_t *w, int64_t N, int64_t K, const float *x, float *y, int *err,
                         cudaStream_t s) {
  const int stages = q4k_mma_stages<MV>(K);
  if (!stages) return gemv_q4k_launch<MV>(w, N, K, x, y, s);
  const size_t smem = q4k_mma_smem<MV>(K, stages);
  const int64_t strips = q4_strips(N);
  const int P = (int)std::min<int64_t>((smem <= kKmSmemTwo ? 2 : 1) * (int64_t)q4k_num_sms(), strips);
  static unsigned long long attr_set[2] = {0, 0};  // per ring depth, one bit per device
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  const int inst = stages == 3 ? 1 : 0;
  if (!(attr_set[inst] & (1ull << dev))) {
    if (stages == 3)
      FG_CUDA(cudaFuncSetAttribute(k_gemv_q4k_mma<MV, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kKmSmemOne));
    else
      FG_CUDA(cudaFuncSetAttribute(k_gemv_q4k_mma<MV, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kKmSmemOne));
    attr_set[inst] |= 1ull << dev;
  }
  if (stages == 3)
    k_gemv_q4k_mma<MV, 3><<<P, kKmThreads, smem, s>>>(w, N, K, x, K, y, N, err);
  else
    k_gemv_q4k_mma<MV, 4><<<P, kKmThreads, smem, s>>>(w, N, K, x, K, y, N, err);
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

// y[M, N] = x[M, K] W^T, W Q4_K [N, K]; `scratch` (N K floats) is used when M > 8; `err` (the context's
// device error word) takes the integer-MMA GEMV's wait timeouts (M <= 4; null: the CUDA-core GEMV).
void launch_qmatmul_q4k(const void *w, int64_t N, int64_t K, const float *x, int64_t M, float *y, float *scratch,
                        int *err, cudaStream_t s) {
  if (M == 0 || N == 0) return;
  const uint8_t *wb = (const uint8_t *)w;
  const bool mma = err && ((uintptr_t)x & 15) == 0 && K % 256 == 0 && std::getenv("FORGE_B200_Q4K") == nullptr;
  switch (M) {
    case 1: return mma ? gemv_q4k_mma_launch<1>(wb, N, K, x, y, err, s) : gemv_q4k_launch<1>(wb, N, K, x, y, s);
    case 2: return mma ? gemv_q4k_mma_launch<2>(wb, N, K, x, y, err, s) : gemv_q4k_launch<2>(wb, N, K, x, y, s);
    case 3: return mma ? gemv_q4k_mma_launch<3>(wb, N, K, x, y, err, s) : gemv_q4k_launch<3>(wb, N, K, x, y, s);
    case 4: return mma ? gemv_q4k_mma_launch<4>(wb, N, K, x, y, err, s) : gemv_q4k_launch<4>(wb, N, K, x, y, s);
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
