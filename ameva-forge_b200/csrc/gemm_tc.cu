// Q4_0 / Q8_0 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a):
//   Y[m, n] = sum_k X[m, k] W[n, k]   (+ the fused epilogues of epilogue.cuh)
// for more than 4 token rows (prefill chunks, batched decode).
//
// The weight matrix is the UMMA A operand and lives in TMEM: a CTA owns 128
// weight rows (one per TMEM lane) and NT tokens (16..256, the UMMA N), so
// D = W_tile X_tile^T sits in TMEM as 128 lanes x NT fp32 columns, next to a
// ring of dequantised A stages of 64 columns (one quad = 128 K columns as fp16
// pairs).  K advances by quads through
//  * raw: one thread copies the quad's codes and scales with TMA boxes laid
//    out [row][16 bytes] (Q4_0: one box per lane-word index of the strip
//    layout; Q8_0: one box per 16 codes), so that a warp reading one 16-byte
//    unit for 32 consecutive rows hits every bank once;
//  * A: producer warp w owns TMEM lanes 32 (w % 4) .. + 31 (= weight rows) and
//    half w / 4 of the quad's K: each thread dequantises its row's 64 values
//    ((q - 8) d, resp. q d, in one fp16 rounding) into 32 registers and stores
//    them with one tcgen05.st;
//  * B: one thread copies the quad's [2][NT][64] fp16 chunks of X (converted
//    and zero-padded to whole quads by k_x_to_f16) with the TMA unit's
//    128-byte swizzle;
//  * one thread of the MMA warp issues eight tcgen05.mma.kind::f16 (K = 16
//    each, A from TMEM, B from shared memory) per quad and commits them to
//    the A and B stages' "empty" mbarriers; after the last quad it commits to
//    the "accumulator" mbarrier;
//  * warps 0-3 (TMEM lanes 0..127) read D with tcgen05.ld into a shared tile
//    that the stages no longer use, then store it with 16-byte stores and the
//    epilogue on row pairs (RoPE / SwiGLU partners are neighbouring columns).
// Shared memory holds only the raw quads and X, so up to 64 tokens two CTAs
// share an SM (256 TMEM columns each) and their small-N MMAs overlap: A read
// from TMEM leaves the shared-memory bandwidth to the copies.  When the
// (weight tile, token tile) grid is small against the GPU, K is split over
// several CTAs (the split count that minimises waves x quads per CTA): each
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

constexpr int kTcRows = 128;                 // UMMA M: weight rows per CTA = TMEM lanes
constexpr int kTcK = 64;                     // K per B chunk (one 128-byte swizzle atom of fp16)
constexpr int kTcProducerWarps = 8;          // warp w: TMEM lanes 32 (w % 4).., K half w / 4 (warps 0-3 also
                                             // run the epilogue)
constexpr int kTcMmaWarp = kTcProducerWarps;       // TMEM owner, one thread issues the MMAs
constexpr int kTcRawWarp = kTcProducerWarps + 1;   // one thread loads the raw quads
constexpr int kTcThreads = (kTcProducerWarps + 3) * 32;  // + one thread that loads the B tiles
constexpr int kTcACols = 64;                 // TMEM columns of one dequantised quad (128 fp16 per row)
constexpr int kTcMaxRing = 16;
// raw quad: Q4_0 4 x [128 rows][16 B] codes (lane-words t = 0..3 of blocks 0..3) + [128 rows][8 B] scales;
// Q8_0 8 x [128 rows][16 B] codes (16 codes each) + [128 rows][8 scales] (two quads)
constexpr int kTcUnitBytes = kTcRows * 16;
constexpr int kTcQ4RawBytes = 4 * kTcUnitBytes + kTcRows * 8;
constexpr int kTcQ8RawBytes = 8 * kTcUnitBytes + kTcRows * 16;

// Rings sized per token tile: up to NT = 64 two CTAs share an SM (<= 110 KB of shared memory and 256
// TMEM columns each), NT = 128 and 256 take an SM (512 columns; at NT = 128 two CTAs with two B stages
// each ran 2.2 times slower).  A bulk-tensor copy takes 1-2.5 us to land
// under load, so the copy rings run far ahead.
template <int NT, int QT = FG_Q4_0>
struct TcGeo {
  static constexpr bool Q8 = QT == FG_Q8_0;
  static constexpr bool Two = NT <= 64;  // two CTAs per SM
  static constexpr int RawBytes = Q8 ? kTcQ8RawBytes : kTcQ4RawBytes;
  static constexpr int BQuad = 2 * NT * kTcK * 2;  // B bytes per quad
  static constexpr int RB = Q8 ? (NT <= 16 ? 8 : NT <= 32 ? 4 : NT <= 64 ? 3 : 3)
                               : (NT <= 16 ? 8 : NT <= 32 ? 6 : NT <= 64 ? 4 : NT <= 128 ? 3 : 2);
  static constexpr int RAW = Q8 ? (NT <= 64 ? 3 : 4) : (NT <= 16 ? 6 : NT <= 32 ? 5 : 4);
  static constexpr int SA = 3;  // dequantised A stages in TMEM
  static constexpr int TmemCols = Two ? 256 : 512;
  static constexpr int ACol = TmemCols - SA * kTcACols;  // first column of the A ring (after D)
  static constexpr size_t RawOff = (size_t)RB * BQuad;
  // + 1 KB for the 1024-byte alignment of the swizzled tiles
  static constexpr size_t Smem = 1024 + RawOff + (size_t)RAW * RawBytes;
  static_assert(RB <= kTcMaxRing && RAW <= kTcMaxRing, "rings");
  static_assert(ACol >= NT, "TMEM: accumulator and A ring");
  static_assert(Smem + 1024 <= (Two ? 113u * 1024 : 232448u), "shared memory per CTA");
  static_assert(Smem - 1024 >= (size_t)NT * kTcRows * 4, "the epilogue tile reuses the rings");
  static_assert(!Q8 || NT <= 128, "Q8_0 token tiles up to 128");
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
__global__ void __launch_bounds__(kTcThreads, NT <= 64 ? 2 : 1)  // two CTAs per SM up to 64 tokens
    k_qgemm_tc(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
               const __grid_constant__ CUtensorMap tms, QMat w, int M, Epilogue ep, GemvScratch scr, int splits) {
  using Geo = TcGeo<NT, QT>;
  extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
  unsigned char *sm = tc_smem_raw + ((1024 - (smem_u32(tc_smem_raw) & 1023)) & 1023);
  constexpr int RB = Geo::RB, SA = Geo::SA, R = Geo::RAW;
  unsigned char *bring = sm, *raw = sm + Geo::RawOff;
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
  if (warp < kTcProducerWarps) {
    // ============ producers: thread = weight row r = TMEM lane, warp half hb of the quad's K ============
    const int quad = warp & 3, hb = warp >> 2, r = 32 * quad + lane;
    // this thread's 32 columns of A stage `as`: lane quadrant of the warp, columns 32 hb ..
    const uint32_t ta = taddr + ((uint32_t)(32 * quad) << 16) + Geo::ACol + 32 * hb;
    for (int qi = 0; qi < nquads; ++qi) {
      const int rs = qi % R, as = qi % SA, Q = q0 + qi;
      ok = ok && mbar_wait(&rfull[rs], (uint32_t)(qi / R) & 1, scr.err, DEVERR_GEMV_FULL);
      const unsigned char *rq = raw + rs * Geo::RawBytes;
      uint32_t out[32];
      if constexpr (Geo::Q8) {
        // units 4 hb .. 4 hb + 3 of 16 codes (device codes q + 128), block = unit / 2; the quad's four
        // scales are half (Q & 1) of the row's 8-scale box
        uint4 c[4];
        uint32_t sc = 0u;
#pragma unroll
        for (int uu = 0; uu < 4; ++uu)
          c[uu] = ok ? *reinterpret_cast<const uint4 *>(rq + (4 * hb + uu) * kTcUnitBytes + r * 16)
                     : make_uint4(0u, 0u, 0u, 0u);
        if (ok) sc = *reinterpret_cast<const uint32_t *>(rq + 8 * kTcUnitBytes + r * 16 + 8 * (Q & 1) + 4 * hb);
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[rs]);  // the quad is in registers: its slot may be refilled
#pragma unroll
        for (int uu = 0; uu < 4; ++uu) {
          // columns past K are zero (the scale plane's padding past K / 32 blocks is not)
          const bool kin = (int64_t)Q * 128 + 16 * (4 * hb + uu) < w.K;
          const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)((uu >> 1) ? (sc >> 16) : (sc & 0xFFFFu))));
          const uint4 lo = kin ? dq8(make_uint2(c[uu].x, c[uu].y), d2) : make_uint4(0u, 0u, 0u, 0u);
          const uint4 hi = kin ? dq8(make_uint2(c[uu].z, c[uu].w), d2) : make_uint4(0u, 0u, 0u, 0u);
          out[8 * uu + 0] = lo.x;
          out[8 * uu + 1] = lo.y;
          out[8 * uu + 2] = lo.z;
          out[8 * uu + 3] = lo.w;
          out[8 * uu + 4] = hi.x;
          out[8 * uu + 5] = hi.y;
          out[8 * uu + 6] = hi.z;
          out[8 * uu + 7] = hi.w;
        }
      } else {
        // lane-word t of blocks 2 hb, 2 hb + 1: byte j holds elements 4t + j (low nibble) and 4t + j + 16
        // (high nibble) of its block
        uint2 c[4];
        uint32_t sc = 0u;
#pragma unroll
        for (int t = 0; t < 4; ++t)
          c[t] = ok ? *reinterpret_cast<const uint2 *>(rq + t * kTcUnitBytes + r * 16 + 8 * hb) : make_uint2(0u, 0u);
        if (ok) sc = *reinterpret_cast<const uint32_t *>(rq + 4 * kTcUnitBytes + r * 8 + 4 * hb);
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[rs]);
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)(bi ? (sc >> 16) : (sc & 0xFFFFu))));
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const uint32_t wd = bi ? c[t].y : c[t].x;
            const uint32_t a0 = __byte_perm(wd, 0u, 0x4140), a1 = __byte_perm(wd, 0u, 0x4342);
            out[16 * bi + 2 * t] = dq_lo(a0, d2);      // elements 4t, 4t+1 of the block
            out[16 * bi + 2 * t + 1] = dq_lo(a1, d2);  // 4t+2, 4t+3
            out[16 * bi + 8 + 2 * t] = dq_hi(a0, d2);  // 4t+16, 4t+17
            out[16 * bi + 9 + 2 * t] = dq_hi(a1, d2);  // 4t+18, 4t+19
          }
        }
      }
      if (qi >= SA) ok = ok && mbar_wait(&aempty[as], (uint32_t)(qi / SA - 1) & 1, scr.err, DEVERR_GEMV_EMPTY);
      tc_fence_after();
      if (ok) {
        const uint32_t ts = ta + as * kTcACols;
        tmem_st16_issue(ts, *reinterpret_cast<const uint32_t(*)[16]>(&out[0]));
        tmem_st16_issue(ts + 16, *reinterpret_cast<const uint32_t(*)[16]>(&out[16]));
        tmem_st_wait();
      }
      tc_fence_before();  // the MMA reads these TMEM columns after the barrier below
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[as]);
    }
  } else if (warp == kTcMmaWarp) {
    // ================= MMA issuer: 8 MMAs (K = 16 each, A from TMEM) per quad =================
    if (lane == 0) {
      const uint32_t idesc = idesc_f16<NT>();
      for (int qi = 0; qi < nquads; ++qi) {
        const int as = qi % SA, bs = qi % RB;
        ok = ok && mbar_wait(&bfull[bs], (uint32_t)(qi / RB) & 1, scr.err, DEVERR_GEMV_FULL);
        ok = ok && mbar_wait(&afull[as], (uint32_t)(qi / SA) & 1, scr.err, DEVERR_GEMV_FULL);
        tc_fence_after();
        if (ok) {
          const uint32_t bq = smem_u32(bring + bs * Geo::BQuad), ta = taddr + Geo::ACol + as * kTcACols;
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int kk = 0; kk < kTcK / 16; ++kk)  // K = 64 h + 16 kk: 8 A columns, 32 bytes into the B atom
              umma_f16_tmem_a(taddr, ta + 8 * (4 * h + kk), smem_desc_sw128(bq + h * (NT * 128) + 32 * kk), idesc,
                              (qi > 0 || h > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&aempty[as]);  // frees the A and B stages once the MMAs above have read them
        umma_commit(&bempty[bs]);
      }
      umma_commit(&accum);
    }
  } else if (warp == kTcRawWarp) {
    // ================= raw loader: one quad of 128 rows per slot, up to R ahead =================
    if (lane == 0) {
      const uint64_t pol_w = l2_evict_first_policy();
      tma_prefetch_desc(&tmw);
      tma_prefetch_desc(&tms);
      const int strip0 = tile_n * (kTcRows / kQ4StripRows);
      int issued = 0;
      for (int qi = 0; qi < nquads; ++qi) {
        const int rs = qi % R, Q = q0 + qi;
        if (qi >= R) ok = ok && mbar_wait(&rempty[rs], (uint32_t)(qi / R - 1) & 1, scr.err, DEVERR_GEMV_EMPTY);
        if (ok) {  // rows past N and codes past K read as zero
          unsigned char *dst = raw + rs * Geo::RawBytes;
          mbar_arrive_expect_tx(&rfull[rs], (uint32_t)Geo::RawBytes);
          if constexpr (Geo::Q8) {
            for (int u = 0; u < 8; ++u)
              tma_load_2d(dst + u * kTcUnitBytes, &tmw, 128 * Q + 16 * u, tile_n * kTcRows, &rfull[rs], pol_w);
            tma_load_2d(dst + 8 * kTcUnitBytes, &tms, 8 * (Q >> 1), tile_n * kTcRows, &rfull[rs], pol_w);
          } else {
            for (int t = 0; t < 4; ++t)
              tma_load_4d(dst + t * kTcUnitBytes, &tmw, 4 * t, 0, Q, strip0, &rfull[rs], pol_w);
            tma_load_3d(dst + 4 * kTcUnitBytes, &tms, 0, Q, strip0, &rfull[rs], pol_w);
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
  const int slots = num_sms * (Geo::Two ? 2 : 1);  // resident CTAs
  // split K to minimise waves x (quads per CTA + a fixed per-CTA cost of about 4 quads: TMEM
  // allocation, pipeline fill, epilogue, fix-up)
  if (tiles < 2 * slots) {
    int best = (tiles + slots - 1) / slots * (nq + 4);
    for (int sp = 2; sp <= std::min(16, nq / 4); ++sp) {
      const int cost = (tiles * sp + slots - 1) / slots * ((nq + sp - 1) / sp + 4);
      if (cost < best) {
        best = cost;
        splits = sp;
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
  // A operand sources, each box landing as [rows][16 bytes]:
  //  Q4_0: the strips [strip][quad][16 rows][4 lane-words][4 blocks] u32 -> for lane-word t one box
  //        (4 words at t, 16 rows, 1 quad, 8 strips); the scales at byte 1024 of each strip-quad,
  //        [16 rows][4] fp16 -> one box (128 bytes, 1 quad, 8 strips)
  //  Q8_0: the codes [N][K] (boxes of 128 rows x 16 codes) and the scales [N][ldd] fp16 (boxes of
  //        128 rows x 8 scales, two quads)
  CUtensorMap tmw, tms;
  if (Geo::Q8) {
    tmw = make_tmap_2d(w.qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)w.N, (uint64_t)w.row_words * 4,
                       (uint64_t)w.row_words * 4, kTcRows, 16);
    tms = make_tmap_2d(w.d, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)w.N, (uint64_t)w.ldd, (uint64_t)w.ldd * 2,
                       kTcRows, 8);
  } else {
    const uint64_t strips = (uint64_t)q4_strips(w.N);
    const uint64_t dims[4] = {16, kQ4StripRows, (uint64_t)nq, strips};
    const uint64_t strides[3] = {64, kQ4QuadBytes, (uint64_t)nq * kQ4QuadBytes};
    const uint32_t box[4] = {4, kQ4StripRows, 1, kTcRows / kQ4StripRows};
    tmw = make_tmap_4d(w.qs, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, dims, strides, box);
    tms = make_tmap_3d(reinterpret_cast<const unsigned char *>(w.qs) + kQ4QuadCodeBytes, CU_TENSOR_MAP_DATA_TYPE_UINT32,
                       4, (kQ4QuadBytes - kQ4QuadCodeBytes) / 4, (uint64_t)nq, strips, kQ4QuadBytes,
                       (uint64_t)nq * kQ4QuadBytes, (kQ4QuadBytes - kQ4QuadCodeBytes) / 4, 1,
                       kTcRows / kQ4StripRows);
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
