// Q4_0 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a):
//   Y[m, n] = sum_k X[m, k] W[n, k]   (+ the fused epilogues of epilogue.cuh)
// for more than 4 token rows (prefill chunks, batched decode).
//
// The weight matrix is the UMMA A operand: a CTA owns 128 weight rows (8 of
// the 16-row strips of the Q4_0 layout, common.cuh) and NT tokens (16..256,
// the UMMA N), so D = W_tile X_tile^T sits in TMEM as 128 lanes x NT fp32
// columns.  K advances by quads (128 columns = two 64-wide swizzle atoms),
// through three shared-memory rings:
//  * raw: one thread copies the quad of the tile's 8 strips (one 3-D TMA box,
//    9 KB) up to RAW quads ahead;
//  * A: warp w dequantises strip w into the canonical K-major, 128-byte
//    swizzled layout (row r at r * 128 bytes, 16-byte chunk c at c ^ (r & 7),
//    8-row atoms 1024 bytes apart): (q - 8) * d in one rounding (the fp16
//    pair 1024 + q, one exact add, one multiply), whole 16-byte chunks, no
//    bank conflicts.  Both operands are fp16: a Q4_0 weight (q - 8) * d
//    carries 15 significant bits, which fp16 keeps to 2^-12 (bf16 would lose
//    2^-9 and sit at the GEMM tolerance);
//  * B: one thread copies the quad's [2][NT][64] fp16 chunks of X (converted
//    and zero-padded to whole quads by k_x_to_f16) with the TMA unit's
//    128-byte swizzle, up to RB quads ahead;
//  * one thread of the MMA warp issues eight tcgen05.mma.kind::f16 (K = 16
//    each) per quad with shared-memory descriptors and commits them to the
//    A and B slots' "empty" mbarriers; after the last quad it commits to the
//    "accumulator" mbarrier;
//  * warps 0-3 (TMEM lanes 0..127) read D with tcgen05.ld into a shared tile
//    that the stages no longer use, then store it with 16-byte stores and the
//    epilogue on row pairs (RoPE / SwiGLU partners are neighbouring columns).
// Work per quad is counted in shared-memory instructions: the MMA thread's
// waits, MMAs and commits queue behind the producers' stores, so both sides
// work at quad granularity.  When the (weight tile, token tile) grid is
// small against the GPU, K is split over several CTAs (the split count that
// minimises waves x quads per CTA): each
// writes its partial tile and the last one of a tile to arrive sums them in
// split order (deterministic) and runs the epilogue.
//
// Every wait is bounded (tma.cuh): on a timeout the device error word is set,
// the CTA skips the remaining work, drains its copies, frees its TMEM and
// returns.
#include <algorithm>

#include "q4_gemv.cuh"
#include "tcgen05.cuh"
#include "tmap.cuh"

namespace fg {
namespace {

constexpr int kTcRows = 128;                 // UMMA M: weight rows per CTA
constexpr int kTcK = 64;                     // K per MMA group (one 128-byte swizzle atom of fp16)
constexpr int kTcProducerWarps = 8;          // warp w dequantises strip w (warps 0-3 also run the epilogue)
constexpr int kTcMmaWarp = kTcProducerWarps;       // TMEM owner, one thread issues the MMAs
constexpr int kTcRawWarp = kTcProducerWarps + 1;   // one thread loads the raw Q4_0 quads
constexpr int kTcThreads = (kTcProducerWarps + 3) * 32;  // + one thread that loads the B tiles
constexpr int kTcAQuad = 2 * kTcRows * kTcK * 2;  // dequantised A per quad: two 16 KB swizzled stages
constexpr int kTcRawBytes = (kTcRows / kQ4StripRows) * kQ4QuadBytes;  // 8 strips x 1152 bytes
constexpr int kTcMaxRing = 16;

// Three rings of whole quads (128 K columns), sized per token tile within 227 KB.
// A bulk-tensor copy takes 1-2.5 us to land under load, so the copy rings run far ahead:
//  * B: the quad's two 64-column chunks of X, [2][NT][64] fp16 swizzled (one 3-D box);
//  * A: the quad's dequantised weights, [2][128][64] fp16 swizzled (producer warps);
//  * raw: the quad of the tile's 8 strips (9 KB, one 3-D box).
//  Q8_0 (QT = FG_Q8_0, NT <= 128): the raw quad is the tile's 128 rows x 128 int8 codes (16 KB, one
//  2-D box) and their 8-scale groups (2 KB, one 2-D box of the scales of two quads).
constexpr int kTcQ8CodeBytes = kTcRows * 128, kTcQ8RawBytes = kTcQ8CodeBytes + kTcRows * 16;

template <int NT, int QT = FG_Q4_0>
struct TcGeo {
  static constexpr bool Q8 = QT == FG_Q8_0;
  static constexpr int RawBytes = Q8 ? kTcQ8RawBytes : kTcRawBytes;
  static constexpr int BQuad = 2 * NT * kTcK * 2;  // B bytes per quad
  static constexpr int RB = NT <= 16 ? 16 : NT <= 32 ? 8 : NT <= 64 ? 5 : NT <= 128 ? 3 : 2;
  static constexpr int SA = Q8 ? (NT >= 64 ? 2 : 3) : NT <= 128 ? 3 : 2;
  static constexpr int RAW = Q8 ? 3 : NT <= 32 ? 6 : NT <= 64 ? 4 : 3;
  static constexpr int TmemCols = NT < 32 ? 32 : NT;  // allocation: a power of two >= 32
  static constexpr size_t AOff = (size_t)RB * BQuad;
  static constexpr size_t RawOff = AOff + (size_t)SA * kTcAQuad;
  // + 1 KB for the 1024-byte alignment of the swizzled tiles
  static constexpr size_t Smem = 1024 + RawOff + (size_t)RAW * RawBytes;
  static_assert(!Q8 || NT <= 128, "Q8_0 token tiles up to 128");
  static_assert(RB <= kTcMaxRing && SA <= kTcMaxRing && RAW <= kTcMaxRing && Smem + 1024 <= 232448,
                "shared memory per CTA");
  static_assert(RawOff >= (size_t)NT * kTcRows * 4, "the epilogue tile reuses the B and A rings");
};

// Instruction descriptor: fp16 A and B, fp32 D, both K-major, M = 128, N = NT.
template <int NT>
__device__ __forceinline__ uint32_t idesc_f16() {
  return idesc_f16_f32acc(kTcRows, NT, false);
}

// Dequantised fp16 pair of two codes at bits 0-3 and 16-19 (low nibbles) or
// 4-7 and 20-23 (high nibbles) of `p`: the magic 0x6400 makes (1024 + q)
// (or 1024 + 16 q) exactly, one exact fp16 add turns it into q - 8, and one
// multiply by d rounds once: (q - 8) d.
__device__ __forceinline__ uint32_t dq_lo(uint32_t p, __half2 d2) {
  const uint32_t h = (p & 0x000F000Fu) | 0x64006400u;
  const __half2 t = __hsub2(*reinterpret_cast<const __half2 *>(&h), __float2half2_rn(1032.0f));
  const __half2 r = __hmul2(t, d2);
  return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t dq_hi(uint32_t p, __half2 d2) {
  const uint32_t h = (p & 0x00F000F0u) | 0x64006400u;
  const __half2 t = __hfma2(*reinterpret_cast<const __half2 *>(&h), __float2half2_rn(0.0625f),
                            __float2half2_rn(-72.0f));  // (1024 + 16 q) / 16 - 72 = q - 8
  const __half2 r = __hmul2(t, d2);
  return *reinterpret_cast<const uint32_t *>(&r);
}

// x [M][ldx] fp32 -> xh [M][Kp] fp16 (the B operand, loaded by TMA); columns
// K..Kp-1 (Kp = K rounded up to whole 128-column quads) are zero.
__global__ void k_x_to_f16(const float *__restrict__ x, int64_t ldx, int M, int64_t K, int64_t Kp,
                           __half *__restrict__ xh) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t n4 = (int64_t)M * (Kp / 4);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / (Kp / 4), k = (i % (Kp / 4)) * 4;
    uint2 h = make_uint2(0u, 0u);
    if (k < K) {
      const float4 v = *reinterpret_cast<const float4 *>(x + m * ldx + k);
      const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
      h = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
    }
    *reinterpret_cast<uint2 *>(xh + m * Kp + k) = h;
  }
}

// Q8_0: eight device codes (q + 128, unsigned) -> four fp16 pairs q * d: 0x6400 | (q + 128) is
// 1024 + q + 128 exactly, one exact subtraction leaves q, one multiply by d rounds once.
__device__ __forceinline__ uint4 dq8(uint2 c, __half2 d2) {
  const uint32_t u0 = c.x, u1 = c.y;
  const uint32_t h[4] = {__byte_perm(u0, 0x64646464u, 0x4140), __byte_perm(u0, 0x64646464u, 0x4342),
                         __byte_perm(u1, 0x64646464u, 0x4140), __byte_perm(u1, 0x64646464u, 0x4342)};
  const __half2 off = __float2half2_rn(1152.0f);
  uint32_t r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 t = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&h[i]), off), d2);
    r[i] = *reinterpret_cast<const uint32_t *>(&t);
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

template <int NT, int QT>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_qgemm_tc(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
               const __grid_constant__ CUtensorMap tms, QMat w, int M, Epilogue ep, GemvScratch scr, int splits) {
  using Geo = TcGeo<NT, QT>;
  extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
  unsigned char *sm = tc_smem_raw + ((1024 - (smem_u32(tc_smem_raw) & 1023)) & 1023);
  constexpr int RB = Geo::RB, SA = Geo::SA, R = Geo::RAW;
  unsigned char *bring = sm, *aring = sm + Geo::AOff, *raw = sm + Geo::RawOff;
  __shared__ __align__(8) uint64_t bfull[kTcMaxRing], bempty[kTcMaxRing], afull[kTcMaxRing], aempty[kTcMaxRing];
  __shared__ __align__(8) uint64_t rfull[kTcMaxRing], rempty[kTcMaxRing], accum;
  __shared__ uint32_t s_taddr;
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tile_n = blockIdx.x, tile_m = blockIdx.y, split = blockIdx.z;
  const int nq = Geo::Q8 ? (int)((w.K + 127) / 128) : (int)w.row_words;
  // this split's quads (128-wide K chunks, zero-padded at the end of a row)
  const int q0 = (int)((int64_t)split * nq / splits), q1 = (int)((int64_t)(split + 1) * nq / splits);
  const int nquads = q1 - q0;
  const int64_t strip0 = (int64_t)tile_n * (kTcRows / kQ4StripRows);
  const int nvalid = (int)std::min<int64_t>(kTcRows / kQ4StripRows, q4_strips(w.N) - strip0);  // strips in range
  const int m0 = tile_m * NT;

  if (tid == 0) {
    for (int s = 0; s < RB; ++s) {
      mbar_init(&bfull[s], 1);  // the B loader's expect_tx
      mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(&afull[s], kTcProducerWarps);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < R; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], kTcProducerWarps);
    }
    mbar_init(&accum, 1);
    fence_barrier_init();
  }
  if (warp == kTcMmaWarp) tmem_alloc(&s_taddr, Geo::TmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = s_taddr;
  asm volatile("griddepcontrol.wait;" ::: "memory");

  bool ok = true;
  if (Geo::Q8 && warp < kTcProducerWarps) {
    // ================= Q8_0 producers: warp w dequantises rows 16w .. 16w+15 =================
    // lane -> (row parity rp, 16-byte output chunk c = 8 codes): 16 lanes read one row's 128 code
    // bytes and write its two swizzled 128-byte rows; a quad's scale sits at 4 (quad & 1) + c / 4
    const int rp = lane >> 4, c = lane & 15;
    for (int qi = 0; qi < nquads; ++qi) {
      const int rs = qi % R, as = qi % SA, sq = 4 * ((q0 + qi) & 1) + (c >> 2);
      ok = ok && mbar_wait(&rfull[rs], (uint32_t)(qi / R) & 1, scr.err, DEVERR_GEMV_FULL);
      uint2 cd[8];
      unsigned short sc[8];
      const unsigned char *rq = raw + rs * Geo::RawBytes;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int row = 16 * warp + 2 * i + rp;
        cd[i] = ok ? *reinterpret_cast<const uint2 *>(rq + row * 128 + 8 * c) : make_uint2(0u, 0u);
        sc[i] = ok ? *reinterpret_cast<const unsigned short *>(rq + kTcQ8CodeBytes + row * 16 + 2 * sq) : 0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[rs]);  // the quad is in registers: its slot may be refilled
      if (qi >= SA) ok = ok && mbar_wait(&aempty[as], (uint32_t)(qi / SA - 1) & 1, scr.err, DEVERR_GEMV_EMPTY);
      if (ok) {
        unsigned char *st = aring + as * kTcAQuad + (c >> 3) * (kTcRows * 128);
        // columns past K are zero (the scale plane's padding past K / 32 blocks is not)
        const bool kin = (int64_t)(q0 + qi) * 128 + 8 * c < w.K;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = 16 * warp + 2 * i + rp;
          *reinterpret_cast<uint4 *>(st + row * 128 + (((c & 7) ^ (row & 7)) * 16)) =
              kin ? dq8(cd[i], __half2half2(__ushort_as_half(sc[i]))) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();  // the tensor core reads these bytes through the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[as]);
    }
  } else if (warp < kTcProducerWarps) {
    // ================= producers: warp w dequantises strip w, one quad per iteration =================
    // lane -> (row rr of the strip, lane-word pair tp): a quarter-warp holds 8 consecutive rows of
    // one pair, so its 16-byte stores into the swizzled rows hit 8 different chunk positions
    const int tp = (lane >> 3) & 1, rr = (lane & 7) + 8 * (lane >> 4), r = warp * kQ4StripRows + rr;
    const bool valid = warp < nvalid;
    for (int qi = 0; qi < nquads; ++qi) {
      const int rs = qi % R, as = qi % SA;
      ok = ok && mbar_wait(&rfull[rs], (uint32_t)(qi / R) & 1, scr.err, DEVERR_GEMV_FULL);
      uint4 U0 = make_uint4(0u, 0u, 0u, 0u), U1 = U0;  // lane-words 2tp, 2tp+1 of blocks 0..3
      uint2 D = make_uint2(0u, 0u);                     // the four block scales
      if (ok && valid) {
        const unsigned char *qb = raw + rs * Geo::RawBytes + warp * kQ4QuadBytes;
        U0 = *reinterpret_cast<const uint4 *>(qb + (rr * 4 + 2 * tp) * 16);
        U1 = *reinterpret_cast<const uint4 *>(qb + (rr * 4 + 2 * tp + 1) * 16);
        D = *reinterpret_cast<const uint2 *>(qb + kQ4QuadCodeBytes + rr * 8);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[rs]);  // the quad is in registers: its slot may be refilled
      if (qi >= SA) ok = ok && mbar_wait(&aempty[as], (uint32_t)(qi / SA - 1) & 1, scr.err, DEVERR_GEMV_EMPTY);
      if (ok) {
        unsigned char *row = aring + as * kTcAQuad + r * 128;
        const uint32_t wa[4] = {U0.x, U0.y, U0.z, U0.w}, wb[4] = {U1.x, U1.y, U1.z, U1.w};
        const uint32_t dd[2] = {D.x, D.y};
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {  // stage blk / 2, columns 32 (blk % 2) .. +31
          const __half2 d2 = __half2half2(
              __ushort_as_half((unsigned short)((blk & 1) ? (dd[blk >> 1] >> 16) : (dd[blk >> 1] & 0xFFFFu))));
          const uint32_t a0 = __byte_perm(wa[blk], 0u, 0x4140), a1 = __byte_perm(wa[blk], 0u, 0x4342);
          const uint32_t b0 = __byte_perm(wb[blk], 0u, 0x4140), b1 = __byte_perm(wb[blk], 0u, 0x4342);
          // low nibbles: elements 8tp..8tp+7 -> chunk 4 (blk % 2) + tp; high: 16 + 8tp.. -> chunk + 2
          const int clo = (blk & 1) * 4 + tp, chi = clo + 2;
          unsigned char *st = row + (blk >> 1) * (kTcRows * 128);
          *reinterpret_cast<uint4 *>(st + ((clo ^ (r & 7)) * 16)) =
              make_uint4(dq_lo(a0, d2), dq_lo(a1, d2), dq_lo(b0, d2), dq_lo(b1, d2));
          *reinterpret_cast<uint4 *>(st + ((chi ^ (r & 7)) * 16)) =
              make_uint4(dq_hi(a0, d2), dq_hi(a1, d2), dq_hi(b0, d2), dq_hi(b1, d2));
        }
      }
      fence_proxy_async_smem();  // the tensor core reads these bytes through the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[as]);
    }
  } else if (warp == kTcMmaWarp) {
    // ================= MMA issuer: 8 MMAs (K = 16 each) per quad =================
    if (lane == 0) {
      const uint32_t idesc = idesc_f16<NT>();
      for (int qi = 0; qi < nquads; ++qi) {
        const int as = qi % SA, bs = qi % RB;
        ok = ok && mbar_wait(&bfull[bs], (uint32_t)(qi / RB) & 1, scr.err, DEVERR_GEMV_FULL);
        ok = ok && mbar_wait(&afull[as], (uint32_t)(qi / SA) & 1, scr.err, DEVERR_GEMV_FULL);
        tc_fence_after();
        if (ok) {
          const uint32_t a = smem_u32(aring + as * kTcAQuad), bq = smem_u32(bring + bs * Geo::BQuad);
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int kk = 0; kk < kTcK / 16; ++kk)  // 32 bytes further into the swizzle atom per K = 16
              umma_f16(taddr, smem_desc_sw128(a + h * (kTcRows * 128) + 32 * kk),
                       smem_desc_sw128(bq + h * (NT * 128) + 32 * kk), idesc, (qi > 0 || h > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&aempty[as]);  // frees the A and B slots once the MMAs above have read them
        umma_commit(&bempty[bs]);
      }
      umma_commit(&accum);
    }
  } else if (warp == kTcRawWarp) {
    // ================= raw loader: one 3-D box per quad (8 strips), up to R ahead =================
    if (lane == 0) {
      const uint64_t pol_w = l2_evict_first_policy();
      tma_prefetch_desc(&tmw);
      int issued = 0;
      for (int qi = 0; qi < nquads; ++qi) {
        const int rs = qi % R;
        if (qi >= R) ok = ok && mbar_wait(&rempty[rs], (uint32_t)(qi / R - 1) & 1, scr.err, DEVERR_GEMV_EMPTY);
        if (ok) {  // strips (rows) past N and codes past K read as zero
          mbar_arrive_expect_tx(&rfull[rs], (uint32_t)Geo::RawBytes);
          if (Geo::Q8) {
            tma_load_2d(raw + rs * Geo::RawBytes, &tmw, 128 * (q0 + qi), tile_n * kTcRows, &rfull[rs], pol_w);
            tma_load_2d(raw + rs * Geo::RawBytes + kTcQ8CodeBytes, &tms, 8 * ((q0 + qi) >> 1), tile_n * kTcRows,
                        &rfull[rs], pol_w);
          } else {
            tma_load_3d(raw + rs * Geo::RawBytes, &tmw, 0, q0 + qi, (int32_t)strip0, &rfull[rs], pol_w);
          }
          issued = qi + 1;
        } else {
          mbar_arrive(&rfull[rs]);
        }
      }
      // drain: no copy may still be landing in shared memory when the CTA exits
      for (int qi = std::max(0, issued - R); qi < issued; ++qi) mbar_wait_drain(&rfull[qi % R], (uint32_t)(qi / R) & 1);
    }
  } else if (lane == 0) {
    // ================= B loader: the quad's NT token rows x 128 columns, up to RB ahead =================
    const uint64_t pol_x = l2_evict_last_policy();
    tma_prefetch_desc(&tmx);
    int issued = 0;
    for (int qi = 0; qi < nquads; ++qi) {
      const int bs = qi % RB;
      if (qi >= RB) ok = ok && mbar_wait(&bempty[bs], (uint32_t)(qi / RB - 1) & 1, scr.err, DEVERR_GEMV_EMPTY);
      if (ok) {
        mbar_arrive_expect_tx(&bfull[bs], (uint32_t)Geo::BQuad);
        tma_load_3d(bring + bs * Geo::BQuad, &tmx, 0, m0, 2 * (q0 + qi), &bfull[bs], pol_x);
        issued = qi + 1;
      } else {
        mbar_arrive(&bfull[bs]);
      }
    }
    for (int qi = std::max(0, issued - RB); qi < issued; ++qi) mbar_wait_drain(&bfull[qi % RB], (uint32_t)(qi / RB) & 1);
  }

  // ================= epilogue: warps 0..3 own TMEM lanes 0..127 =================
  // D goes TMEM -> shared tile [token j][weight row] (the stages are free once the
  // accumulator barrier fired) -> global with 16-byte stores: a warp writes 512
  // contiguous bytes of one token's output row per instruction.
  if (warp < 4) {
    ok = ok && mbar_wait(&accum, 0, scr.err, DEVERR_GEMV_FULL);
    tc_fence_after();
    float *tile = reinterpret_cast<float *>(sm);
    const uint32_t tw = taddr + ((uint32_t)(32 * warp) << 16);
    constexpr int CW = NT < 32 ? 16 : 32;
    for (int c0 = 0; c0 < NT; c0 += CW) {
      float v[32];
      if (CW == 32)
        tmem_ld32(tw + c0, v);
      else
        tmem_ld16(tw + c0, v);
#pragma unroll
      for (int j = 0; j < CW; ++j) tile[(c0 + j) * kTcRows + 32 * warp + lane] = v[j];
    }
    tc_fence_before();
    named_sync_id(1, 128);
    bool store = true;
    if (splits > 1) {
      // split-K: every split publishes its tile ([split][token][row] per tile); the last
      // one to arrive sums them in split order, so the result does not depend on timing
      constexpr int V4 = NT * kTcRows / 4;  // float4s per tile
      float4 *part = reinterpret_cast<float4 *>(scr.part) + (int64_t)(tile_m * gridDim.x + tile_n) * splits * V4;
      float4 *t4 = reinterpret_cast<float4 *>(tile);
      for (int e = tid; e < V4; e += 128) part[(int64_t)split * V4 + e] = t4[e];
      __threadfence();
      named_sync_id(1, 128);
      int *ticket = scr.tickets + tile_m * gridDim.x + tile_n;
      if (tid == 0) s_last = atomicAdd(ticket, 1) == splits - 1;
      named_sync_id(1, 128);
      store = s_last;
      if (store) {
        __threadfence();
        if (tid == 0) *ticket = 0;
        for (int e0 = tid; e0 < V4; e0 += 4 * 128) {
          float4 acc[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int q = 0; q < splits; ++q) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int e = e0 + u * 128;
              if (e < V4) {
                const float4 p4 = __ldcg(part + (int64_t)q * V4 + e);
                acc[u].x += p4.x;
                acc[u].y += p4.y;
                acc[u].z += p4.z;
                acc[u].w += p4.w;
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (e0 + u * 128 < V4) t4[e0 + u * 128] = acc[u];
        }
        named_sync_id(1, 128);
      }
    }
    if (store && ok) {
      const int64_t n = (int64_t)tile_n * kTcRows + 4 * lane;  // four output columns per lane
      for (int j = warp; j < NT && m0 + j < M; j += 4)
        epi_store_quad(ep, n, w.N, m0 + j, *reinterpret_cast<const float4 *>(tile + j * kTcRows + 4 * lane));
    }
  }
  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc_fence_after();
    tmem_dealloc(taddr, Geo::TmemCols);
  }
}

template <int NT, int QT>
void launch_tc_t(const QMat &w, const float *x, int M, int64_t ldx, const Epilogue &ep, const GemvScratch &sc,
                 int num_sms, cudaStream_t s) {
  using Geo = TcGeo<NT, QT>;
  const int tiles_n = (int)ceil_div(w.N, kTcRows), tiles_m = (int)ceil_div(M, NT);
  const int nq = Geo::Q8 ? (int)ceil_div(w.K, 128) : (int)w.row_words;  // K split in whole quads, >= 4 per split
  int splits = 1;
  const int tiles = tiles_n * tiles_m;
  // split K to minimise waves x (quads per CTA + a fixed per-CTA cost of about 4 quads: TMEM
  // allocation, pipeline fill, epilogue, fix-up); e.g. 86 tiles of 32 quads on 148 SMs run 3 splits
  // in 2 waves (2 x 15) rather than 1 split in 1 wave (36)
  if (tiles < 2 * num_sms) {
    int best = (tiles + num_sms - 1) / num_sms * (nq + 4);
    for (int s = 2; s <= std::min(16, nq / 4); ++s) {
      const int cost = (tiles * s + num_sms - 1) / num_sms * ((nq + s - 1) / s + 4);
      if (cost < best) {
        best = cost;
        splits = s;
      }
    }
  }
  if (splits > 1) {
    const uint64_t need = (uint64_t)tiles * splits * kTcRows * NT;
    if (need > sc.part_floats || tiles > sc.n_tickets) splits = 1;
  }
  const int64_t Kp = (int64_t)nq * 128;
  FG_REQUIRE(sc.xh && tc_xh_elems(M, w.K) <= sc.xh_elems, FG_ERR_VALIDATION, "GEMM: fp16 activation scratch too small");
  {
    const int64_t n4 = (int64_t)M * (Kp / 4);
    const int grid = (int)std::min<int64_t>(ceil_div(n4, 256), (int64_t)num_sms * 8);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FG_CUDA(cudaLaunchKernelEx(&cfg, k_x_to_f16, x, ldx, M, w.K, Kp, sc.xh));
  }
  // B operand: xh [M][Kp] viewed as [Kp/64 chunks][M rows][64], so one box (64, NT, 2) is a
  // quad's two swizzled [NT][64] chunks; rows past M read as zero
  const CUtensorMap tmx = make_tmap_3d(sc.xh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kTcK, (uint64_t)M,
                                       (uint64_t)(Kp / kTcK), (uint64_t)Kp * 2, kTcK * 2, kTcK, NT, 2,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  // A operand source.  Q4_0: the strips as [strip][quad][1152 bytes], one quad of 8 strips per box.
  // Q8_0: the codes [N][K] (boxes of 128 rows x 128 codes) and the scales [N][ldd] fp16 (boxes of
  // 128 rows x 8 scales, two quads)
  CUtensorMap tmw, tms;
  if (Geo::Q8) {
    tmw = make_tmap_2d(w.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)w.N, (uint64_t)w.row_words * 4,
                       (uint64_t)w.row_words * 4, kTcRows, 128);
    tms = make_tmap_2d(w.d, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)w.N, (uint64_t)w.ldd, (uint64_t)w.ldd * 2,
                       kTcRows, 8);
  } else {
    tmw = make_tmap_3d(w.qs, CU_TENSOR_MAP_DATA_TYPE_UINT64, 8, kQ4QuadBytes / 8, (uint64_t)nq,
                       (uint64_t)q4_strips(w.N), kQ4QuadBytes, (uint64_t)nq * kQ4QuadBytes, kQ4QuadBytes / 8, 1,
                       kTcRows / kQ4StripRows);
    tms = tmw;
  }
  const size_t smem = Geo::Smem;
  static unsigned long long attr_set = 0;
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << dev))) {
    FG_CUDA(cudaFuncSetAttribute(k_qgemm_tc<NT, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)tiles_n, (unsigned)tiles_m, (unsigned)splits);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FG_CUDA(cudaLaunchKernelEx(&cfg, k_qgemm_tc<NT, QT>, tmx, tmw, tms, w, M, ep, sc, splits));
}

}  // namespace

bool qgemm_tc_supported(const QMat &w, int M) {
  return (w.qtype == FG_Q4_0 || w.qtype == FG_Q8_0) && M >= 1 && w.K % 32 == 0 && w.K >= 32 && w.N >= 1;
}

void launch_qgemm_tc(const QMat &w, const float *x, int M, int64_t ldx, const Epilogue &ep, const GemvScratch &sc,
                     int num_sms, cudaStream_t s) {
  FG_REQUIRE(qgemm_tc_supported(w, M), FG_ERR_SHAPE, "tensor-core GEMM: unsupported matrix");
  FG_REQUIRE(ldx % 4 == 0 && ((uintptr_t)x & 15) == 0, FG_ERR_VALIDATION, "GEMM: x must be 16-byte aligned rows");
  if (M == 0 || w.N == 0) return;
  // token tile: the smallest UMMA N that covers M, up to 256 tokens per CTA (128 for Q8_0, whose raw
  // quads are twice as large)
  if (w.qtype == FG_Q8_0) {
    if (M <= 16)
      launch_tc_t<16, FG_Q8_0>(w, x, M, ldx, ep, sc, num_sms, s);
    else if (M <= 32)
      launch_tc_t<32, FG_Q8_0>(w, x, M, ldx, ep, sc, num_sms, s);
    else if (M <= 64)
      launch_tc_t<64, FG_Q8_0>(w, x, M, ldx, ep, sc, num_sms, s);
    else
      launch_tc_t<128, FG_Q8_0>(w, x, M, ldx, ep, sc, num_sms, s);
  } else if (M <= 16) {
    launch_tc_t<16, FG_Q4_0>(w, x, M, ldx, ep, sc, num_sms, s);
  } else if (M <= 32) {
    launch_tc_t<32, FG_Q4_0>(w, x, M, ldx, ep, sc, num_sms, s);
  } else if (M <= 64) {
    launch_tc_t<64, FG_Q4_0>(w, x, M, ldx, ep, sc, num_sms, s);
  } else if (M <= 128) {
    launch_tc_t<128, FG_Q4_0>(w, x, M, ldx, ep, sc, num_sms, s);
  } else {
    launch_tc_t<256, FG_Q4_0>(w, x, M, ldx, ep, sc, num_sms, s);
  }
}

}  // namespace fg
