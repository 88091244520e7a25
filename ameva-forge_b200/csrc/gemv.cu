// Fused dequant-GEMV for batch-1..4 decode: y[m, n] = sum_k x[m, k] W[n, k],
// W in Q4_0 / Q8_0 (device layout: common.cuh).
//
// Roofline: HBM-bound.  Algorithmic bytes per launch = N*K/32 blocks *
// (18 B Q4_0 | 34 B Q8_0) + 4*M*(K + N); every weight byte is read once.
//
// Shared structure (sm_100a):
//  * two CTAs per SM, each a producer thread plus 8 consumer warps: the
//    producer streams weight tiles (Q4_0: 128 rows x 128 code bytes, Q8_0: 32
//    rows x 512, plus their fp16 scales) with two 2-D TMA loads
//    (cp.async.bulk.tensor, out-of-range rows zero-filled by the TMA unit)
//    into a 3-stage shared-memory ring tracked by mbarriers (~100 KB per SM in
//    flight).  The kernel releases its dependents at start (programmatic
//    dependent launch), so the next kernel's CTAs fill the SM slots freed by
//    this kernel's retiring CTAs and begin streaming their own weights --
//    which do not depend on this kernel -- during its tail;
//  * (row-group, chunk) work units are split evenly over the CTAs
//    (stream-K): a row group cut between CTAs is finished by the last CTA
//    to arrive (atomic ticket), which sums the partials in CTA order, so
//    results are deterministic and every fused epilogue sees complete sums;
//  * the x vector(s) are staged once per CTA in shared memory with the
//    RMSNorm that precedes every projection fused in.
//
// Q4_0 math (k_qgemv_q4): tensor cores do the multiply-add.  One LOP3 turns
// two 4-bit codes into the fp16 pair (1024 + n, 1024 + n') -- or (1024 + 16n,
// ...) for the codes stored at nibble offsets 4 -- which mma.sync m16n8k16
// multiplies by x with fp32 accumulation.  x enters as a pair of fp16 columns
// (hi, lo = x - hi) per token, i.e. with ~22 significant bits, after a
// power-of-two range scaling; the 16x weight scale of half the codes is
// folded into x, and the 1024 offset and the -8 zero point are removed
// exactly by a per-block correction sum(x) * (1024 + 8 s) fed in as the MMA
// accumulator input.  Each block's fp32 result is scaled by its fp16 d.  The
// codes are stored in fragment order at upload (q4_elem), so every lane
// loads one u32 per row and block and spends 5 integer ops per 8 weights.
//
// Q8_0 math (k_qgemv_q8): CUDA cores.  PRMT places a byte into the mantissa
// of 2^23 (0x4B000000 | byte); one packed FADD2 removes 2^23 + 128 exactly and
// packed FFMA2 accumulates in fp32, scaled by d once per block.
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

// Producer thread: stream the units [u0, u1) through the ring.
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
                                             const Sched &sc, int g, const float *red, int *s_last, bool ok) {
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
    const int64_t n = (int64_t)g * kRows + 2 * p;
    if (n + 1 < w.N)
      epi_store_pair(ep, n, m, v0, v1);
    else if (n < w.N && ep.mode == EPI_PLAIN)
      epi_store_one(ep, n, m, v0);
  }
}

// ---------------------------------------------------------------------------
// Q4_0 tensor-core GEMV: 128-row groups; warp w owns rows 16w..16w+15 of the
// group for the whole K sweep (no cross-warp reduction); a stage is 128 rows
// x 8 blocks (two quads), one m16n8k16 pair per block.
// ---------------------------------------------------------------------------
constexpr int kQ4Rows = 128, kQ4TB = 128, kQ4CB = 8;
using GeoQ4 = Geo<kQ4Rows, kQ4TB, kQ4CB>;

__device__ __forceinline__ void mma_f16_zc(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}
__device__ __forceinline__ void mma_f16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int MV>
__global__ void __launch_bounds__(kThreads, 2)
    k_qgemv_q4(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap td, QMat w,
               const float *__restrict__ x, int64_t ldx, const float *__restrict__ gamma, float eps, int do_norm,
               Epilogue ep, GemvScratch scr) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *ring = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages];
  __shared__ float s_sum[kConsumers][MV], s_max[kConsumers][MV], s_gmax[kConsumers];
  __shared__ float s_mul[MV], s_sigma[MV], s_inv_sigma[MV];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = (int)(w.K >> 5);
  const Sched sc = schedule<kQ4Rows>(w, (nb + kQ4CB - 1) / kQ4CB);
  const int nbx = sc.nc * kQ4CB;  // blocks staged (zero past nb)
  uint4 *xf = reinterpret_cast<uint4 *>(ring + kStages * GeoQ4::SB);  // [nbx][2MV][4] fp16 fragments
  float *corr = reinterpret_cast<float *>(xf + nbx * 2 * MV * 4);      // [MV][nbx] negated corrections
  float *red = corr + MV * nbx;                                        // [256][MV]

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
    if (lane == 0) produce<kQ4Rows, kQ4TB, kQ4CB>(&tq, &td, sc, ring, full, empty, scr.err);
    return;
  }

  // ---------------- stage x (after the producer of x has finished)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int K = (int)w.K;
  {  // statistics: sum of squares (RMSNorm), max |x|, max |gamma|
    float ss[MV], mx[MV], gm = 0.0f;
#pragma unroll
    for (int m = 0; m < MV; ++m) ss[m] = mx[m] = 0.0f;
    for (int i = tid; i < K / 4; i += kCThreads) {
#pragma unroll
      for (int m = 0; m < MV; ++m) {
        const float4 v = *reinterpret_cast<const float4 *>(x + m * ldx + 4 * i);
        ss[m] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        mx[m] = fmaxf(mx[m], fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
      if (do_norm && gamma) {
        const float4 gv = *reinterpret_cast<const float4 *>(gamma + 4 * i);
        gm = fmaxf(gm, fmaxf(fmaxf(fabsf(gv.x), fabsf(gv.y)), fmaxf(fabsf(gv.z), fabsf(gv.w))));
      }
    }
#pragma unroll
    for (int m = 0; m < MV; ++m) {
      const float s = warp_sum(ss[m]), a = warp_max(mx[m]);
      if (lane == 0) {
        s_sum[warp][m] = s;
        s_max[warp][m] = a;
      }
    }
    gm = warp_max(gm);
    if (lane == 0) s_gmax[warp] = gm;
    named_sync(kCThreads);
    if (tid < MV) {
      float s = 0.0f, a = 0.0f, gmax = 0.0f;
      for (int i = 0; i < kConsumers; ++i) {
        s += s_sum[i][tid];
        a = fmaxf(a, s_max[i][tid]);
        gmax = fmaxf(gmax, s_gmax[i]);
      }
      float inv = 1.0f, bound = a;
      if (do_norm) {
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)K), eps)));
        bound = a * inv * (gamma ? gmax : 1.0f);
      }
      // power-of-two range scaling: max |x * sigma| < 2^14 in fp16
      int e = 0;
      if (bound > 0.0f && bound < INFINITY) frexpf(bound, &e);
      e = min(max(14 - e, -100), 100);
      s_mul[tid] = inv;
      s_sigma[tid] = ldexpf(1.0f, e);
      s_inv_sigma[tid] = ldexpf(1.0f, -e);
    }
    named_sync(kCThreads);
  }
  for (int item = tid; item < MV * nbx * 4; item += kCThreads) {
    const int t = item & 3;
    const int bb = (item >> 2) % nbx;
    const int m = (item >> 2) / nbx;
    const float inv = s_mul[m], sigma = s_sigma[m];
    uint32_t hi[4], lo[4];
    float csum = 0.0f;
#pragma unroll
    for (int f = 0; f < 4; ++f) {
      // fragment f of lane-word t: elements (2t, 2t+1) + {0, 8, 16, 24}[f]
      float2 v = make_float2(0.0f, 0.0f);
      if (bb < nb) {
        const int k = bb * 32 + 2 * t + 8 * f;
        v = *reinterpret_cast<const float2 *>(x + m * ldx + k);
        if (do_norm) {
          v.x = __fmul_rn(v.x, inv);
          v.y = __fmul_rn(v.y, inv);
          if (gamma) {
            const float2 gv = *reinterpret_cast<const float2 *>(gamma + k);
            v.x = __fmul_rn(v.x, gv.x);
            v.y = __fmul_rn(v.y, gv.y);
          }
        }
      }
      const float sf = (f & 1) ? 0.0625f * sigma : sigma;  // logical k >= 8 of a half: codes carry x16
      v.x *= sf;
      v.y *= sf;
      const __half2 h = __floats2half2_rn(v.x, v.y);
      const float2 hf = __half22float2(h);
      const __half2 l = __floats2half2_rn(v.x - hf.x, v.y - hf.y);
      const float2 lf = __half22float2(l);
      hi[f] = *reinterpret_cast<const uint32_t *>(&h);
      lo[f] = *reinterpret_cast<const uint32_t *>(&l);
      const float wgt = (f & 1) ? 1024.0f + 128.0f : 1024.0f + 8.0f;  // 1024 + 8 s
      csum += wgt * ((hf.x + lf.x) + (hf.y + lf.y));
    }
    uint4 *dst = xf + (bb * 2 * MV + 2 * m) * 4 + t;
    dst[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    dst[4] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    csum += __shfl_xor_sync(0xffffffffu, csum, 1);
    csum += __shfl_xor_sync(0xffffffffu, csum, 2);
    if (t == 0) corr[m * nbx + bb] = -csum;
  }
  named_sync(kCThreads);

  // ---------------- consume
  const int gq = lane >> 2, t = lane & 3;
  const bool xlane = gq < 2 * MV;  // lanes holding a real B column
  const int a_off = (16 * warp + gq) * kQ4TB + t * 16;     // byte offset of row gq's lane word in a stage
  const int d_off = GeoQ4::SQ + (16 * warp + gq) * kQ4CB * 2;
  const uint4 *xl = xf + gq * 4 + t;                       // + block * 2MV*4
  const float *cl = corr + t * nbx;
  float2 acc = make_float2(0.0f, 0.0f);                    // rows gq, gq+8; token t
  bool ok = true;
  int i = 0, g = sc.u0 / sc.nc, c = sc.u0 % sc.nc;
  for (int u = sc.u0; u < sc.u1; ++u, ++i) {
    const int s = i % kStages;
    ok = ok && mbar_wait(&full[s], (uint32_t)(i / kStages) & 1, scr.err, DEVERR_GEMV_FULL);
    if (ok) {
      const unsigned char *st = ring + s * GeoQ4::SB;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int bb0 = c * kQ4CB + 4 * j;  // first block of the quad
        const uint4 A0 = *reinterpret_cast<const uint4 *>(st + a_off + j * 64);
        const uint4 A1 = *reinterpret_cast<const uint4 *>(st + a_off + j * 64 + 8 * kQ4TB);
        const uint2 D0 = *reinterpret_cast<const uint2 *>(st + d_off + j * 8);
        const uint2 D1 = *reinterpret_cast<const uint2 *>(st + d_off + j * 8 + 8 * kQ4CB * 2);
        float4 cr = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < MV) cr = *reinterpret_cast<const float4 *>(cl + bb0);
        const uint32_t a0w[4] = {A0.x, A0.y, A0.z, A0.w}, a1w[4] = {A1.x, A1.y, A1.z, A1.w};
        const float crv[4] = {cr.x, cr.y, cr.z, cr.w};
#pragma unroll
        for (int bi = 0; bi < 4; ++bi) {
          uint4 B = make_uint4(0u, 0u, 0u, 0u);
          if (xlane) B = xl[(bb0 + bi) * 2 * MV * 4];
          const uint32_t M = 0x64006400u;
          const uint32_t wa = a0w[bi], wb = a1w[bi];
          const uint32_t wa8 = wa >> 8, wb8 = wb >> 8;
          const uint32_t ah0[4] = {(wa & 0x000F000Fu) | M, (wb & 0x000F000Fu) | M, (wa & 0x00F000F0u) | M,
                                   (wb & 0x00F000F0u) | M};
          const uint32_t ah1[4] = {(wa8 & 0x000F000Fu) | M, (wb8 & 0x000F000Fu) | M, (wa8 & 0x00F000F0u) | M,
                                   (wb8 & 0x00F000F0u) | M};
          float dacc[4];
          mma_f16_zc(dacc, ah0, B.x, B.y);
          mma_f16(dacc, ah1, B.z, B.w);
          // scale pair (row gq, row gq+8) of block bi: halves bi of D0 and D1
          const uint32_t dpair = __byte_perm(bi < 2 ? D0.x : D0.y, bi < 2 ? D1.x : D1.y, (bi & 1) ? 0x7632 : 0x5410);
          const float2 dsc = __half22float2(*reinterpret_cast<const __half2 *>(&dpair));
          float2 v = fadd2(make_float2(dacc[0], dacc[2]), make_float2(dacc[1], dacc[3]));
          v = fadd2(v, make_float2(crv[bi], crv[bi]));
          acc = ffma2(dsc, v, acc);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const bool group_end = (c == sc.nc - 1) || (u == sc.u1 - 1);
    if (group_end) {
      if (t < MV) {
        red[(16 * warp + gq) * MV + t] = acc.x * s_inv_sigma[t];
        red[(16 * warp + gq + 8) * MV + t] = acc.y * s_inv_sigma[t];
      }
      named_sync(kCThreads);
      finish_group<kQ4Rows, MV>(w, ep, scr, sc, g, red, &s_last, ok);
      named_sync(kCThreads);
      acc = make_float2(0.0f, 0.0f);
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
      finish_group<kRows, MV>(w, ep, scr, sc, g, red, &s_last, ok);
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
  return 128 + (size_t)kStages * GeoQ4::SB + (size_t)nbx * 2 * MV * 4 * 16 + (size_t)MV * nbx * 4 +
         (size_t)kQ4Rows * MV * 4;
}
size_t q8_smem(int64_t K, int MV) {
  return 128 + (size_t)kStages * Geo<kRows, kTileBytes, 16>::SB + (size_t)MV * K * 4 + (size_t)kRows * MV * 4;
}

template <int MV>
void launch_mv(const QMat &w, const float *x, int64_t ldx, const float *gamma, float eps, bool do_norm,
               const Epilogue &ep, const GemvScratch &sc, int num_sms, cudaStream_t s) {
  const bool q4 = w.qtype == FG_Q4_0;
  const int CB = q4 ? kQ4CB : 16, ROWS = q4 ? kQ4Rows : kRows, TB = q4 ? kQ4TB : kTileBytes;
  const int64_t nb = w.K / 32, nc = ceil_div(nb, CB), G = ceil_div(w.N, ROWS), U = G * nc;
  FG_REQUIRE(U < (1ll << 31), FG_ERR_SHAPE, "gemv: matrix too large");
  const int P = (int)std::min<int64_t>(2LL * num_sms, U);
  int maxc = 1;
  for (int64_t g = 0; g < G; ++g)
    maxc = std::max(maxc, cta_of((int)(g * nc + nc - 1), (int)U, P) - cta_of((int)(g * nc), (int)U, P) + 1);
  FG_REQUIRE((uint64_t)G * maxc * ROWS * MV <= sc.part_floats && G <= sc.n_tickets, FG_ERR_SHAPE,
             "gemv: workspace too small for N=%lld K=%lld", (long long)w.N, (long long)w.K);
  GemvScratch scx = sc;
  scx.maxc = maxc;
  const size_t smem = q4 ? q4_smem(w.K, MV) : q8_smem(w.K, MV);
  auto kern = q4 ? k_qgemv_q4<MV> : k_qgemv_q8<MV>;
  static unsigned long long attr_set[2] = {0, 0};  // per instantiation, one bit per device
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set[q4] & (1ull << dev))) {
    FG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 112 * 1024));
    attr_set[q4] |= 1ull << dev;
  }
  const CUtensorMap tq = make_tmap_2d(w.qs, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, w.N, w.row_words, w.row_words * 4,
                                      ROWS, TB / 4);
  const CUtensorMap td = make_tmap_2d(w.d, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w.N, w.ldd, w.ldd * 2, ROWS, CB);
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
  FG_CUDA(cudaLaunchKernelEx(&cfg, kern, tq, td, w, x, ldx, gamma, eps, do_norm ? 1 : 0, ep, scx));
}

}  // namespace

bool gemv_supported(const QMat &w, int M) {
  if (M < 1 || M > 4 || w.K % 32 != 0 || w.K < 32) return false;
  const size_t smem = w.qtype == FG_Q4_0 ? q4_smem(w.K, M) : q8_smem(w.K, M);
  return smem <= 112 * 1024;
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
