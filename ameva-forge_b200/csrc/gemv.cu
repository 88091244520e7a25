// Fused dequant-GEMV for batch-1..4 decode: y[m, n] = sum_k x[m, k] W[n, k],
// W in Q4_0 / Q8_0 (device layout: common.cuh).
//
// Roofline: HBM-bound.  Algorithmic bytes per launch = N*K/32 blocks *
// (18 B Q4_0 | 34 B Q8_0) + 4*M*(K + N); every weight byte is read once.
//
// Shared structure (sm_100a):
//  * a producer thread plus 8 consumer warps per CTA, two CTAs per SM (one
//    when the staged x needs more shared memory).  The producer streams the
//    weights into a shared-memory ring tracked by mbarriers: Q4_0 one
//    contiguous 18 KB tile (128 rows x 8 blocks with their scales, the
//    device layout of common.cuh) per stage with a 1-D bulk copy
//    (cp.async.bulk), 4 stages; Q8_0 32 rows x 512 code bytes plus scales
//    with two 2-D tensor-map loads (cp.async.bulk.tensor), 3 stages.  The
//    kernel releases its dependents at start (programmatic dependent
//    launch), so the next kernel's CTAs fill the SM slots freed by this
//    kernel's retiring CTAs and begin streaming their own weights -- which do
//    not depend on this kernel -- during its tail;
//  * (row-group, chunk) work units are split evenly over the CTAs
//    (stream-K): a CTA's units are consecutive tiles, i.e. one contiguous
//    range of the matrix.  A row group cut between CTAs is finished by the
//    last CTA to arrive (atomic ticket), which sums the partials in CTA
//    order, so results are deterministic and every fused epilogue sees
//    complete sums;
//  * the x vector(s) are staged once per CTA in shared memory with the
//    RMSNorm that precedes every projection fused in.
//
// Q4_0 math (k_qgemv_q4): integer tensor-core MMA, see the comment above the
// kernel.  Q8_0 math (k_qgemv_q8): CUDA cores.  PRMT places a byte into the
// mantissa of 2^23 (0x4B000000 | byte); one packed FADD2 removes 2^23 + 128
// exactly and packed FFMA2 accumulates in fp32, scaled by d once per block.
#include "epilogue.cuh"
#include "tma.cuh"
#include "tmap.cuh"

namespace fg {
namespace {

constexpr int kRows = 32;        // Q8_0 rows per row group (one TMA box high)
constexpr int kConsumers = 8;    // consumer warps (two CTAs share an SM)
constexpr int kCThreads = kConsumers * 32;
constexpr int kThreads = kCThreads + 32;  // + producer warp
constexpr int kTileBytes = 512;  // code bytes per row per chunk (one TMA box wide)
constexpr int kStages = 3;

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// CTA that owns work unit u when U units are split evenly over P CTAs
// (CTA k owns [k*U/P, (k+1)*U/P)).
__host__ __device__ __forceinline__ int cta_of(int u, int U, int P) {
  return (int)(((int64_t)(u + 1) * P + U - 1) / U - 1);
}

// Stage geometry: ROWS rows x TB code bytes (CB blocks) per TMA tile.
template <int ROWS, int TB, int CB>
struct Geo {
  static constexpr int SQ = ROWS * TB;            // code bytes per stage
  static constexpr int SB = SQ + ROWS * CB * 2;   // + scales
};

struct Sched {
  int nc, G, U, P, u0, u1;
};
template <int ROWS>
__device__ __forceinline__ Sched schedule(const QMat &w, int nb_chunked) {
  Sched s;
  s.nc = nb_chunked;
  s.G = (int)((w.N + ROWS - 1) / ROWS);
  s.U = s.G * s.nc;
  s.P = gridDim.x;
  s.u0 = (int)((int64_t)blockIdx.x * s.U / s.P);
  s.u1 = (int)(((int64_t)blockIdx.x + 1) * s.U / s.P);
  return s;
}

// Producer thread, Q4_0: unit u is tile u of the tiled layout (common.cuh),
// one contiguous bulk copy; a CTA's units are consecutive tiles, so each CTA
// streams one contiguous range of the matrix.
template <int STAGES>
__device__ __forceinline__ void produce_tiles(const unsigned char *tiles, const Sched &sc, unsigned char *ring,
                                              uint64_t *full, uint64_t *empty, int *err) {
  const uint64_t pol = l2_evict_first_policy();
  int i = 0;
  for (int u = sc.u0; u < sc.u1; ++u, ++i) {
    const int s = i % STAGES;
    const uint32_t k = (uint32_t)(i / STAGES);
    if (i >= STAGES && !mbar_wait(&empty[s], (k - 1) & 1, err, DEVERR_GEMV_EMPTY)) break;
    mbar_arrive_expect_tx(&full[s], kQ4TileBytes);
    bulk_g2s(ring + s * kQ4TileBytes, tiles + (int64_t)u * kQ4TileBytes, kQ4TileBytes, &full[s], pol);
  }
  // drain: no copy may still be landing in this CTA's shared memory on exit
  for (int j = i > STAGES ? i - STAGES : 0; j < i; ++j)
    mbar_wait(&full[j % STAGES], (uint32_t)(j / STAGES) & 1, err, DEVERR_DRAIN);
}

// Producer thread, Q8_0: stream the units [u0, u1) through the ring with 2-D
// tensor-map loads of the codes and scales.
template <int ROWS, int TB, int CB>
__device__ __forceinline__ void produce(const CUtensorMap *tq, const CUtensorMap *td, const Sched &sc,
                                        unsigned char *ring, uint64_t *full, uint64_t *empty, int *err) {
  using Gm = Geo<ROWS, TB, CB>;
  tma_prefetch_desc(tq);
  tma_prefetch_desc(td);
  const uint64_t pol = l2_evict_first_policy();
  int i = 0, g = sc.u0 / sc.nc, c = sc.u0 % sc.nc;
  for (int u = sc.u0; u < sc.u1; ++u, ++i) {
    const int s = i % kStages;
    const uint32_t k = (uint32_t)(i / kStages);
    if (i >= kStages && !mbar_wait(&empty[s], (k - 1) & 1, err, DEVERR_GEMV_EMPTY)) break;
    unsigned char *st = ring + s * Gm::SB;
    mbar_arrive_expect_tx(&full[s], Gm::SB);
    tma_load_2d(st, tq, c * (TB / 4), g * ROWS, &full[s], pol);
    tma_load_2d(st + Gm::SQ, td, c * CB, g * ROWS, &full[s], pol);
    if (++c == sc.nc) {
      c = 0;
      ++g;
    }
  }
  // drain: no copy may still be landing in this CTA's shared memory on exit
  for (int j = i > kStages ? i - kStages : 0; j < i; ++j)
    mbar_wait(&full[j % kStages], (uint32_t)(j / kStages) & 1, err, DEVERR_DRAIN);
}

// Finish row group g from the CTA's partial vector red[ROWS][MV] (already
// reduced over this CTA's warps): epilogue directly, or stream-K fix-up.
template <int ROWS, int MV>
__device__ __forceinline__ void finish_group(const QMat &w, const Epilogue &ep, const GemvScratch &scr,
                                             const Sched &sc, int g, const float *red, const float *mul, int *s_last,
                                             bool ok) {
  constexpr int kRows = ROWS;
  const int tid = threadIdx.x;
  const int first = g * sc.nc, last = first + sc.nc - 1;
  const bool whole = first >= sc.u0 && last < sc.u1;
  float *pg = nullptr;
  int ncontrib = 1;
  if (!whole) {
    const int k0 = cta_of(first, sc.U, sc.P), k1 = cta_of(last, sc.U, sc.P);
    const int j = blockIdx.x - k0;
    ncontrib = k1 - k0 + 1;
    pg = scr.part + (int64_t)g * scr.maxc * kRows * MV;
    for (int i = tid; i < kRows * MV; i += kCThreads) pg[j * kRows * MV + i] = red[i];
    __threadfence();
    named_sync(kCThreads);
    if (tid == 0) *s_last = atomicAdd(scr.tickets + g, 1) == ncontrib - 1;
    named_sync(kCThreads);
    if (!*s_last) return;
    __threadfence();
    if (tid == 0) scr.tickets[g] = 0;  // ready for the next launch
  }
  if (!ok) return;
  // thread -> (row pair p, token m): pairs finish RoPE / SwiGLU epilogues
  for (int q = tid; q < (kRows / 2) * MV; q += kCThreads) {
    const int p = q / MV, m = q % MV;
    float v0 = 0.0f, v1 = 0.0f;
    if (whole) {
      v0 = red[(2 * p) * MV + m];
      v1 = red[(2 * p + 1) * MV + m];
    } else {
      for (int jj = 0; jj < ncontrib; ++jj) {
        v0 += __ldcg(pg + jj * kRows * MV + (2 * p) * MV + m);
        v1 += __ldcg(pg + jj * kRows * MV + (2 * p + 1) * MV + m);
      }
    }
    if (mul) {
      v0 *= mul[m];
      v1 *= mul[m];
    }
    const int64_t n = (int64_t)g * kRows + 2 * p;
    if (n + 1 < w.N)
      epi_store_pair(ep, n, m, v0, v1);
    else if (n < w.N && ep.mode == EPI_PLAIN)
      epi_store_one(ep, n, m, v0);
  }
}

// ---------------------------------------------------------------------------
// Q4_0 tensor-core GEMV (integer MMA).  128-row groups; warp w owns rows
// 16w..16w+15 of the group for the whole K sweep (no cross-warp reduction); a
// stage is one tile (128 rows x 8 blocks), one mma.sync m16n8k32 per block
// and 16 rows: A = the u8 codes (q + 8, straight from the GGUF bytes), B = two
// s8 digit columns per token, D = exact int32 dot products.
//
// x staging: every 32-element block of x' (x, times gamma when the RMSNorm is
// fused) gets a power-of-two scale 2^e with max|x'| 2^e in [2^20, 2^21);
// v = rn(x' 2^e) (22 bits) splits into digits hi = v >> 14 in [-128, 127],
// mid = (v >> 7) & 127 and lo = v & 127.  A token takes four B columns (hi,
// mid, lo, 0), so one MMA serves two tokens; the lanes of D columns (hi, mid)
// accumulate 128 D_hi + D_mid, those of (lo, 0) accumulate 128 D_lo, and the
// two combine exactly at the end as 128 a + b / 128.  The MMA accumulator
// input is -8 * (sum of the block's digits), which removes the code offset
// exactly, so D = sum (q - 8) * digit, and per block and row the kernel adds
// d * 2^-e * D' into an fp32 accumulator.  Scales are local to a block, so
// one large activation does not coarsen the others.  The RMSNorm's 1/rms
// multiplies the finished sums.
// ---------------------------------------------------------------------------
constexpr int kQ4Rows = kQ4TileRows, kQ4TB = 128, kQ4CB = kQ4TileBlocks;
constexpr int kQ4Stages = 4;
using GeoQ4 = Geo<kQ4Rows, kQ4TB, kQ4CB>;
static_assert(GeoQ4::SB == kQ4TileBytes && GeoQ4::SQ == kQ4TileCodeBytes, "stage = one Q4_0 tile");

__device__ __forceinline__ void imma_u8s8(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1, int c0, int c1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}

// Digits of 4 consecutive elements packed as s8 bytes.
__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) | ((uint32_t)d << 24);
}

template <int MV>
__global__ void __launch_bounds__(kThreads, 2)
    k_qgemv_q4(QMat w, const float *__restrict__ x, int64_t ldx, const float *__restrict__ gamma, float eps, int do_norm,
               Epilogue ep, GemvScratch scr) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *ring = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
  __shared__ __align__(8) uint64_t full[kQ4Stages], empty[kQ4Stages];
  __shared__ float s_sum[kConsumers][MV];
  __shared__ float s_inv[MV];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = (int)(w.K >> 5);
  const Sched sc = schedule<kQ4Rows>(w, (nb + kQ4CB - 1) / kQ4CB);
  const int nbx = sc.nc * kQ4CB;  // blocks staged (zero past nb)
  constexpr int NM = (MV + 1) / 2;  // MMAs per block: two tokens each
  uint2 *xb = reinterpret_cast<uint2 *>(ring + kQ4Stages * GeoQ4::SB);  // [nbx][3 MV digit cols][4 t]
  int *cx0 = reinterpret_cast<int *>(xb + nbx * 3 * MV * 4);            // [2 MV][nbx] MMA C, col 2t
  int *cx1 = cx0 + 2 * MV * nbx;                                        // [2 MV][nbx] MMA C, col 2t+1
  float *fbk = reinterpret_cast<float *>(cx1 + 2 * MV * nbx);           // [MV][nbx] 2^-e
  float *red = fbk + MV * nbx;                                          // [128][MV]

  if (tid == 0) {
    for (int s = 0; s < kQ4Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // Let the next kernel of the stream launch now: its CTAs take SM slots as
  // this kernel's CTAs retire and start streaming their weights while this
  // kernel finishes (they wait for this kernel's results before reading x).
  asm volatile("griddepcontrol.launch_dependents;");
  if (warp == kConsumers) {
    if (lane == 0)
      produce_tiles<kQ4Stages>(reinterpret_cast<const unsigned char *>(w.qs), sc, ring, full, empty, scr.err);
    return;
  }

  // ---------------- stage x (after the producer of x has finished)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  {
    const int q = lane & 7;  // 4-element group of the block; 8 lanes per block
#pragma unroll
    for (int m = 0; m < MV; ++m) {
      float ss = 0.0f;
      for (int item = tid; item < nbx * 8; item += kCThreads) {
        const int bb = item >> 3;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (bb < nb) {
          const int k = bb * 32 + 4 * q;
          v = *reinterpret_cast<const float4 *>(x + m * ldx + k);
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
          if (do_norm && gamma) {
            const float4 g = *reinterpret_cast<const float4 *>(gamma + k);
            v.x *= g.x;
            v.y *= g.y;
            v.z *= g.z;
            v.w *= g.w;
          }
        }
        float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        // amax in [2^E, 2^(E+1)) -> scale 2^(20 - E); zero / subnormal blocks keep 2^126 (digits ~0)
        const int E = ((__float_as_int(amax) >> 23) & 0xFF) - 127;
        const int e = min(max(20 - E, -126), 126);
        const float scl = __int_as_float((e + 127) << 23);
        const float vf[4] = {v.x, v.y, v.z, v.w};
        int hi[4], mi[4], lo[4], shi = 0, smi = 0, slo = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int vi = __float2int_rn(fminf(fmaxf(vf[i] * scl, -2097152.0f), 2097151.0f));
          hi[i] = vi >> 14;
          mi[i] = (vi >> 7) & 127;
          lo[i] = vi & 127;
          shi += hi[i];
          smi += mi[i];
          slo += lo[i];
        }
        {
          // B fragment words of digit columns 3m, 3m+1, 3m+2: lane-word t = q & 3, half q >> 2
          uint32_t *col = reinterpret_cast<uint32_t *>(xb + (bb * 3 * MV + 3 * m) * 4) + (q & 3) * 2 + (q >> 2);
          col[0] = pack_s8x4(hi[0], hi[1], hi[2], hi[3]);
          col[8] = pack_s8x4(mi[0], mi[1], mi[2], mi[3]);
          col[16] = pack_s8x4(lo[0], lo[1], lo[2], lo[3]);
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
          shi += __shfl_xor_sync(0xffffffffu, shi, o);
          smi += __shfl_xor_sync(0xffffffffu, smi, o);
          slo += __shfl_xor_sync(0xffffffffu, slo, o);
        }
        if (q == 0) {
          // C of the lanes holding (hi, mid) and (lo, 0) of token m
          cx0[(2 * m) * nbx + bb] = -8 * shi;
          cx1[(2 * m) * nbx + bb] = -8 * smi;
          cx0[(2 * m + 1) * nbx + bb] = -8 * slo;
          cx1[(2 * m + 1) * nbx + bb] = 0;
          // non-finite inputs make the block factor NaN, so the outputs are NaN
          fbk[m * nbx + bb] = amax <= 3.402823466e38f ? __int_as_float((127 - e) << 23) : __int_as_float(0x7fc00000);
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) s_sum[warp][m] = ss;
    }
  }
  named_sync(kCThreads);
  if (tid < MV) {
    float s = 0.0f;
    for (int i = 0; i < kConsumers; ++i) s += s_sum[i][tid];
    s_inv[tid] = do_norm ? __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)w.K), eps))) : 1.0f;
  }

  // ---------------- consume
  const int gq = lane >> 2, t = lane & 3;
  const int a_off = (16 * warp + gq) * kQ4TB + t * 16;     // byte offset of row gq's lane word in a stage
  const int par = gq & 1;                                   // quad halves swapped on odd rows
  const int d_off = GeoQ4::SQ + (16 * warp + gq) * kQ4CB * 2;
  // B column gq of MMA i = digit (gq & 3) of token 2i + (gq >> 2); digit 3 is the zero column
  const uint2 *xl[NM];
  bool xv[NM];
  const int *c0l[NM], *c1l[NM];
  const float *fbl[NM];
#pragma unroll
  for (int im = 0; im < NM; ++im) {
    const int btok = 2 * im + (gq >> 2), dtok = 2 * im + (t >> 1);
    xv[im] = (gq & 3) < 3 && btok < MV;
    xl[im] = xb + (xv[im] ? 3 * btok + (gq & 3) : 0) * 4 + t;
    // lanes of a padding token (odd MV) read token 0's values; their D columns are dropped
    c0l[im] = cx0 + (dtok < MV ? 4 * im + t : (t & 1)) * nbx;
    c1l[im] = cx1 + (dtok < MV ? 4 * im + t : (t & 1)) * nbx;
    fbl[im] = fbk + (dtok < MV ? dtok : 0) * nbx;
  }
  float2 acc[NM];
#pragma unroll
  for (int im = 0; im < NM; ++im) acc[im] = make_float2(0.0f, 0.0f);  // rows gq, gq+8
  bool ok = true;
  int i = 0, g = sc.u0 / sc.nc, c = sc.u0 % sc.nc;
  for (int u = sc.u0; u < sc.u1; ++u, ++i) {
    const int s = i % kQ4Stages;
    ok = ok && mbar_wait(&full[s], (uint32_t)(i / kQ4Stages) & 1, scr.err, DEVERR_GEMV_FULL);
    if (ok) {
      const unsigned char *st = ring + s * GeoQ4::SB;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int bb0 = c * kQ4CB + 4 * j;  // first block of the quad
        const uint4 A0 = *reinterpret_cast<const uint4 *>(st + a_off + (j ^ par) * 64);
        const uint4 A1 = *reinterpret_cast<const uint4 *>(st + a_off + (j ^ par) * 64 + 8 * kQ4TB);
        const uint2 D0 = *reinterpret_cast<const uint2 *>(st + d_off + j * 8);
        const uint2 D1 = *reinterpret_cast<const uint2 *>(st + d_off + j * 8 + 8 * kQ4CB * 2);
        const uint32_t a0w[4] = {A0.x, A0.y, A0.z, A0.w}, a1w[4] = {A1.x, A1.y, A1.z, A1.w};
#pragma unroll
        for (int im = 0; im < NM; ++im) {
          const int4 C0 = *reinterpret_cast<const int4 *>(c0l[im] + bb0);
          const int4 C1 = *reinterpret_cast<const int4 *>(c1l[im] + bb0);
          const float4 FB = *reinterpret_cast<const float4 *>(fbl[im] + bb0);
          const int c0v[4] = {C0.x, C0.y, C0.z, C0.w}, c1v[4] = {C1.x, C1.y, C1.z, C1.w};
          const float fbv[4] = {FB.x, FB.y, FB.z, FB.w};
#pragma unroll
          for (int bi = 0; bi < 4; ++bi) {
            uint2 B = make_uint2(0u, 0u);
            if (xv[im]) B = xl[im][(bb0 + bi) * 3 * MV * 4];
            const uint32_t wa = a0w[bi], wb = a1w[bi];
            int di[4];
            imma_u8s8(di, wa & 0x0F0F0F0Fu, wb & 0x0F0F0F0Fu, (wa >> 4) & 0x0F0F0F0Fu, (wb >> 4) & 0x0F0F0F0Fu, B.x,
                      B.y, c0v[bi], c1v[bi]);
            const float2 v = make_float2((float)(di[0] * 128 + di[1]), (float)(di[2] * 128 + di[3]));
            // scale pair (row gq, row gq+8) of block bi: halves bi of D0 and D1
            const uint32_t dpair =
                __byte_perm(bi < 2 ? D0.x : D0.y, bi < 2 ? D1.x : D1.y, (bi & 1) ? 0x7632 : 0x5410);
            float2 dsc = __half22float2(*reinterpret_cast<const __half2 *>(&dpair));
            dsc = fmul2(dsc, make_float2(fbv[bi], fbv[bi]));
            acc[im] = ffma2(dsc, v, acc[im]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const bool group_end = (c == sc.nc - 1) || (u == sc.u1 - 1);
    if (group_end) {
#pragma unroll
      for (int im = 0; im < NM; ++im) {
        // lanes t even hold 128 D_hi + D_mid sums, lane t + 1 the 128 D_lo sums
        const float bx = __shfl_down_sync(0xffffffffu, acc[im].x, 1);
        const float by = __shfl_down_sync(0xffffffffu, acc[im].y, 1);
        const int tk = 2 * im + (t >> 1);
        if ((t & 1) == 0 && tk < MV) {
          red[(16 * warp + gq) * MV + tk] = acc[im].x * 128.0f + bx * 0.0078125f;
          red[(16 * warp + gq + 8) * MV + tk] = acc[im].y * 128.0f + by * 0.0078125f;
        }
        acc[im] = make_float2(0.0f, 0.0f);
      }
      named_sync(kCThreads);
      finish_group<kQ4Rows, MV>(w, ep, scr, sc, g, red, s_inv, &s_last, ok);
      named_sync(kCThreads);
    }
    if (++c == sc.nc) {
      c = 0;
      ++g;
    }
  }
}

// ---------------------------------------------------------------------------
// Q8_0 CUDA-core GEMV: 16 warps x 4 rows; lane -> half (16 values) of a block
// ---------------------------------------------------------------------------
__device__ __forceinline__ void unpack_q8(uint32_t w, float2 v[2]) {
  const uint32_t M = 0x4B000000u;
  const float2 off = make_float2(-8388736.0f, -8388736.0f);  // 2^23 + 128
  v[0] = fadd2(make_float2(__uint_as_float(__byte_perm(w, M, 0x7540)), __uint_as_float(__byte_perm(w, M, 0x7541))),
               off);
  v[1] = fadd2(make_float2(__uint_as_float(__byte_perm(w, M, 0x7542)), __uint_as_float(__byte_perm(w, M, 0x7543))),
               off);
}

template <int MV>
__global__ void __launch_bounds__(kThreads, 2)
    k_qgemv_q8(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap td, QMat w,
               const float *__restrict__ x, int64_t ldx, const float *__restrict__ gamma, float eps, int do_norm,
               Epilogue ep, GemvScratch scr) {
  constexpr int CB = 16;
  using Gm = Geo<kRows, kTileBytes, CB>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *ring = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ float s_norm[kConsumers][MV];
  __shared__ float s_inv[MV];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = (int)(w.K >> 5);
  const Sched sc = schedule<kRows>(w, (nb + CB - 1) / CB);
  float4 *xs = reinterpret_cast<float4 *>(ring + kStages * Gm::SB);  // [MV][nb][8], swizzled
  float *red = reinterpret_cast<float *>(xs + (size_t)MV * nb * 8);  // [64][MV]

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // Let the next kernel of the stream launch now: its CTAs take SM slots as
  // this kernel's CTAs retire and start streaming their weights while this
  // kernel finishes (they wait for this kernel's results before reading x).
  asm volatile("griddepcontrol.launch_dependents;");
  if (warp == kConsumers) {
    if (lane == 0) produce<kRows, kTileBytes, CB>(&tq, &td, sc, ring, full, empty, scr.err);
    return;
  }

  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (do_norm) {
    float ss[MV];
#pragma unroll
    for (int m = 0; m < MV; ++m) ss[m] = 0.0f;
    for (int i = tid; i < nb * 8; i += kCThreads) {
#pragma unroll
      for (int m = 0; m < MV; ++m) {
        const float4 v = *reinterpret_cast<const float4 *>(x + m * ldx + 4 * i);
        ss[m] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
    }
#pragma unroll
    for (int m = 0; m < MV; ++m) {
      const float s = warp_sum(ss[m]);
      if (lane == 0) s_norm[warp][m] = s;
    }
    named_sync(kCThreads);
    if (tid < MV) {
      float s = 0.0f;
      for (int i = 0; i < kConsumers; ++i) s += s_norm[i][tid];
      s_inv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)w.K), eps)));
    }
    named_sync(kCThreads);
  }
  for (int idx = tid; idx < MV * nb * 8; idx += kCThreads) {
    const int m = idx / (nb * 8);
    const int rem = idx - m * nb * 8;
    const int b = rem >> 3, q = rem & 7;
    float4 v = *reinterpret_cast<const float4 *>(x + m * ldx + 32 * b + 4 * q);
    if (do_norm) {
      const float iv = s_inv[m];
      v.x = __fmul_rn(v.x, iv);
      v.y = __fmul_rn(v.y, iv);
      v.z = __fmul_rn(v.z, iv);
      v.w = __fmul_rn(v.w, iv);
      if (gamma) {
        const float4 gm = *reinterpret_cast<const float4 *>(gamma + 32 * b + 4 * q);
        v.x = __fmul_rn(v.x, gm.x);
        v.y = __fmul_rn(v.y, gm.y);
        v.z = __fmul_rn(v.z, gm.z);
        v.w = __fmul_rn(v.w, gm.w);
      }
    }
    xs[(m * nb + b) * 8 + (q ^ (b & 7))] = v;
  }
  named_sync(kCThreads);

  float2 acc[4][MV];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int m = 0; m < MV; ++m) acc[r][m] = make_float2(0.0f, 0.0f);
  bool ok = true;
  int i = 0, g = sc.u0 / sc.nc, c = sc.u0 % sc.nc;
  const int bl = lane >> 1, h = lane & 1;  // block of the chunk, half of the block
  for (int u = sc.u0; u < sc.u1; ++u, ++i) {
    const int s = i % kStages;
    ok = ok && mbar_wait(&full[s], (uint32_t)(i / kStages) & 1, scr.err, DEVERR_GEMV_FULL);
    const int b = c * CB + bl;
    if (ok && b < nb) {
      const unsigned char *st = ring + s * Gm::SB;
      const int sw = b & 7;
      float2 part[4][MV];
      float dsc[4];
      uint4 qv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int rr = warp * 4 + r;  // rows past N arrive zero-filled (scale 0)
#pragma unroll
        for (int m = 0; m < MV; ++m) part[r][m] = make_float2(0.0f, 0.0f);
        qv[r] = *reinterpret_cast<const uint4 *>(st + rr * kTileBytes + lane * 16);
        dsc[r] = __half2float(*reinterpret_cast<const __half *>(st + Gm::SQ + (rr * CB + bl) * 2));
      }
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        float4 xa[MV];
#pragma unroll
        for (int m = 0; m < MV; ++m) xa[m] = xs[(m * nb + b) * 8 + ((4 * h + tt) ^ sw)];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const uint32_t word = tt == 0 ? qv[r].x : tt == 1 ? qv[r].y : tt == 2 ? qv[r].z : qv[r].w;
          float2 v[2];
          unpack_q8(word, v);
#pragma unroll
          for (int m = 0; m < MV; ++m) {
            part[r][m] = ffma2(v[0], make_float2(xa[m].x, xa[m].y), part[r][m]);
            part[r][m] = ffma2(v[1], make_float2(xa[m].z, xa[m].w), part[r][m]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int m = 0; m < MV; ++m) acc[r][m] = ffma2(part[r][m], make_float2(dsc[r], dsc[r]), acc[r][m]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const bool group_end = (c == sc.nc - 1) || (u == sc.u1 - 1);
    if (group_end) {
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int m = 0; m < MV; ++m) {
          const float v = warp_sum(acc[r][m].x + acc[r][m].y);
          if (lane == 0) red[(warp * 4 + r) * MV + m] = v;
          acc[r][m] = make_float2(0.0f, 0.0f);
        }
      named_sync(kCThreads);
      finish_group<kRows, MV>(w, ep, scr, sc, g, red, nullptr, &s_last, ok);
      named_sync(kCThreads);
    }
    if (++c == sc.nc) {
      c = 0;
      ++g;
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
size_t q4_smem(int64_t K, int MV) {
  const int64_t nbx = ceil_div(K / 32, kQ4CB) * kQ4CB;
  const int nm = (MV + 1) / 2;
  (void)nm;
  return 128 + (size_t)kQ4Stages * GeoQ4::SB + (size_t)nbx * 3 * MV * 4 * 8 + (size_t)4 * MV * nbx * 4 +
         (size_t)MV * nbx * 4 + (size_t)kQ4Rows * MV * 4;
}
size_t q8_smem(int64_t K, int MV) {
  return 128 + (size_t)kStages * Geo<kRows, kTileBytes, 16>::SB + (size_t)MV * K * 4 + (size_t)kRows * MV * 4;
}

// Shared memory per CTA: up to kSmemTwo two CTAs share an SM; larger x
// staging (long K, several tokens) runs one CTA per SM with up to kSmemOne.
constexpr size_t kSmemTwo = 112 * 1024, kSmemOne = 225 * 1024;

template <int MV>
void launch_mv(const QMat &w, const float *x, int64_t ldx, const float *gamma, float eps, bool do_norm,
               const Epilogue &ep, const GemvScratch &sc, int num_sms, cudaStream_t s) {
  const bool q4 = w.qtype == FG_Q4_0;
  const int CB = q4 ? kQ4CB : 16, ROWS = q4 ? kQ4Rows : kRows, TB = q4 ? kQ4TB : kTileBytes;
  const int64_t nb = w.K / 32, nc = ceil_div(nb, CB), G = ceil_div(w.N, ROWS), U = G * nc;
  FG_REQUIRE(U < (1ll << 31), FG_ERR_SHAPE, "gemv: matrix too large");
  const size_t smem = q4 ? q4_smem(w.K, MV) : q8_smem(w.K, MV);
  const int P = (int)std::min<int64_t>((smem <= kSmemTwo ? 2LL : 1LL) * num_sms, U);
  int maxc = 1;
  for (int64_t g = 0; g < G; ++g)
    maxc = std::max(maxc, cta_of((int)(g * nc + nc - 1), (int)U, P) - cta_of((int)(g * nc), (int)U, P) + 1);
  FG_REQUIRE((uint64_t)G * maxc * ROWS * MV <= sc.part_floats && G <= sc.n_tickets, FG_ERR_SHAPE,
             "gemv: workspace too small for N=%lld K=%lld", (long long)w.N, (long long)w.K);
  GemvScratch scx = sc;
  scx.maxc = maxc;
  static unsigned long long attr_set[2] = {0, 0};  // per instantiation, one bit per device
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set[q4] & (1ull << dev))) {
    if (q4)
      FG_CUDA(cudaFuncSetAttribute(k_qgemv_q4<MV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOne));
    else
      FG_CUDA(cudaFuncSetAttribute(k_qgemv_q8<MV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOne));
    attr_set[q4] |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)P);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (q4) {
    FG_REQUIRE(((uintptr_t)w.qs & 15) == 0, FG_ERR_VALIDATION, "gemv: Q4_0 tiles must be 16-byte aligned");
    FG_CUDA(cudaLaunchKernelEx(&cfg, k_qgemv_q4<MV>, w, x, ldx, gamma, eps, do_norm ? 1 : 0, ep, scx));
  } else {
    const CUtensorMap tq = make_tmap_2d(w.qs, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w.N, w.row_words, w.row_words * 4,
                                        ROWS, TB / 4);
    const CUtensorMap td = make_tmap_2d(w.d, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w.N, w.ldd, w.ldd * 2, ROWS, CB);
    FG_CUDA(cudaLaunchKernelEx(&cfg, k_qgemv_q8<MV>, tq, td, w, x, ldx, gamma, eps, do_norm ? 1 : 0, ep, scx));
  }
}

}  // namespace

bool gemv_supported(const QMat &w, int M) {
  if (M < 1 || M > 4 || w.K % 32 != 0 || w.K < 32) return false;
  const size_t smem = w.qtype == FG_Q4_0 ? q4_smem(w.K, M) : q8_smem(w.K, M);
  return smem <= kSmemOne;
}

void launch_qgemv_ld(const QMat &w, const float *x, int M, int64_t ldx, const float *norm_gamma, float norm_eps,
                     bool do_norm, const Epilogue &ep, const GemvScratch &sc, int num_sms, cudaStream_t s) {
  FG_REQUIRE(gemv_supported(w, M), FG_ERR_SHAPE, "gemv: unsupported M=%d K=%lld", M, (long long)w.K);
  FG_REQUIRE(ldx % 4 == 0 && ((uintptr_t)x & 15) == 0, FG_ERR_VALIDATION, "gemv: x must be 16-byte aligned rows");
  if (w.N == 0) return;
  switch (M) {
    case 1: launch_mv<1>(w, x, ldx, norm_gamma, norm_eps, do_norm, ep, sc, num_sms, s); break;
    case 2: launch_mv<2>(w, x, ldx, norm_gamma, norm_eps, do_norm, ep, sc, num_sms, s); break;
    case 3: launch_mv<3>(w, x, ldx, norm_gamma, norm_eps, do_norm, ep, sc, num_sms, s); break;
    default: launch_mv<4>(w, x, ldx, norm_gamma, norm_eps, do_norm, ep, sc, num_sms, s); break;
  }
}

}  // namespace fg
