// Device building blocks of the fused dequant-GEMV, shared by the stand-alone
// GEMV kernels (gemv.cu) and the persistent decode-step kernel
// (decode_step.cu).
//
// Work is split into units split evenly over P "virtual CTAs": a virtual CTA
// is one producer thread plus 8 consumer warps with their own shared-memory
// ring; a stand-alone GEMV CTA is one virtual CTA, a decode-step CTA holds
// two.  Q4_0 units are 16-row strips (common.cuh): a virtual CTA computes
// whole output rows, its 8 warps split K and reduce in shared memory, so
// there is no cross-CTA reduction.  Q8_0 units are (32-row group, K chunk)
// pairs (stream-K) with a deterministic last-arriver fix-up (finish_group).
//
// Q4_0 math (integer tensor cores): a stage is one tile of up to 16 quads of
// a strip; warp w takes quads w, w+8 and runs one mma.sync m16n8k32 per block
// and 16 rows: A = the u8 codes (q + 8, straight from the GGUF bytes), B = s8
// digit columns of x, D = exact int32 dot products.
//
// x staging: every 32-element block of x' (x, times gamma when an RMSNorm is
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
#pragma once
#include "epilogue.cuh"
#include "tma.cuh"

namespace fg {

constexpr int kGroupWarps = 8;                      // consumer warps of a virtual CTA
constexpr int kGroupThreads = kGroupWarps * 32;

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// Virtual CTA that owns unit u when U units are split evenly over P of them
// (virtual CTA k owns [k*U/P, (k+1)*U/P)).
__host__ __device__ __forceinline__ int cta_of(int u, int U, int P) {
  return (int)(((int64_t)(u + 1) * P + U - 1) / U - 1);
}

struct Sched {
  int nc, G, U, P, k, u0, u1;  // chunks per row group, row groups, units, virtual CTAs, this one, its units
};
// Only the first min(P, U) virtual CTAs take units, so every one of them owns
// at least one unit: the fix-up counts the owners of a row group as the
// consecutive virtual CTAs cta_of(first) .. cta_of(last).
__device__ __forceinline__ Sched make_sched(int64_t N, int rows, int nc, int k, int P) {
  Sched s;
  s.nc = nc;
  s.G = (int)((N + rows - 1) / rows);
  s.U = s.G * s.nc;
  s.P = max(1, min(P, s.U));
  s.k = k;
  s.u0 = k < s.P ? (int)((int64_t)k * s.U / s.P) : 0;
  s.u1 = k < s.P ? (int)(((int64_t)k + 1) * s.U / s.P) : 0;
  return s;
}

// Producer thread, Q4_0: the tiles of strips [u0, u1) in order, each one
// contiguous bulk copy into ring slot (i % STAGES) (a virtual CTA's strips are
// consecutive, i.e. one contiguous range of the matrix).  `i` is the running
// count of stages this ring has filled (it continues across calls).
template <int STAGES>
__device__ __forceinline__ bool produce_q4_strips(const QMat &w, int u0, int u1, unsigned char *ring, uint64_t *full,
                                                  uint64_t *empty, int &i, uint64_t pol, int *err) {
  const int nq = (int)w.row_words;
  for (int u = u0; u < u1; ++u) {
    const unsigned char *src = reinterpret_cast<const unsigned char *>(w.qs) + (int64_t)u * nq * kQ4QuadBytes;
    for (int q0 = 0; q0 < nq; q0 += kQ4TileQuads, ++i) {
      const int s = i % STAGES;
      if (i >= STAGES && !mbar_wait(&empty[s], (uint32_t)(i / STAGES - 1) & 1, err, DEVERR_GEMV_EMPTY)) return false;
      const uint32_t bytes = (uint32_t)min(kQ4TileQuads, nq - q0) * kQ4QuadBytes;
      mbar_arrive_expect_tx(&full[s], bytes);
      bulk_g2s(ring + s * kQ4TileBytes, src + (int64_t)q0 * kQ4QuadBytes, bytes, &full[s], pol);
    }
  }
  return true;
}

// Wait until no copy of the ring is still landing (`i` stages were filled).
template <int STAGES>
__device__ __forceinline__ void drain_ring(uint64_t *full, int i, int *err) {
  for (int j = i > STAGES ? i - STAGES : 0; j < i; ++j)
    mbar_wait(&full[j % STAGES], (uint32_t)(j / STAGES) & 1, err, DEVERR_DRAIN);
}

// Finish row group g from the virtual CTA's partial vector red[ROWS][MV]:
// epilogue directly, or stream-K fix-up (the last contributor to arrive sums
// the partials in virtual-CTA order, so results are deterministic).  Called by
// the group's `nth` consumer threads (tid in [0, nth)) with named barrier
// `bar`.  `mul` (per token, may be null) scales the finished sums.
template <int ROWS, int MV>
__device__ __forceinline__ void finish_group(const QMat &w, const Epilogue &ep, const GemvScratch &scr,
                                             const Sched &sc, int g, const float *red, const float *mul, int *s_last,
                                             bool ok, int tid, int nth, int bar) {
  const int first = g * sc.nc, last = first + sc.nc - 1;
  const bool whole = first >= sc.u0 && last < sc.u1;
  float *pg = nullptr;
  int ncontrib = 1;
  if (!whole) {
    const int k0 = cta_of(first, sc.U, sc.P), k1 = cta_of(last, sc.U, sc.P);
    const int j = sc.k - k0;
    ncontrib = k1 - k0 + 1;
    pg = scr.part + (int64_t)g * scr.maxc * ROWS * MV;
    for (int i = tid; i < ROWS * MV; i += nth) pg[j * ROWS * MV + i] = red[i];
    __threadfence();
    named_sync_id(bar, nth);
    if (tid == 0) *s_last = atomicAdd(scr.tickets + g, 1) == ncontrib - 1;
    named_sync_id(bar, nth);
    if (!*s_last) return;
    __threadfence();
    if (tid == 0) scr.tickets[g] = 0;  // ready for the next use
  }
  if (!ok) return;
  // thread -> (row pair p, token m): pairs finish RoPE / SwiGLU epilogues
  for (int q = tid; q < (ROWS / 2) * MV; q += nth) {
    const int p = q / MV, m = q % MV;
    float v0 = 0.0f, v1 = 0.0f;
    if (whole) {
      v0 = red[(2 * p) * MV + m];
      v1 = red[(2 * p + 1) * MV + m];
    } else {
      for (int jj = 0; jj < ncontrib; ++jj) {
        v0 += __ldcg(pg + jj * ROWS * MV + (2 * p) * MV + m);
        v1 += __ldcg(pg + jj * ROWS * MV + (2 * p + 1) * MV + m);
      }
    }
    if (mul) {
      v0 *= mul[m];
      v1 *= mul[m];
    }
    const int64_t n = (int64_t)g * ROWS + 2 * p;
    if (n + 1 < w.N)
      epi_store_pair(ep, n, m, v0, v1);
    else if (n < w.N && ep.mode == EPI_PLAIN)
      epi_store_one(ep, n, m, v0);
  }
}

// ---------------------------------------------------------------------------
// Q4_0 x staging
// ---------------------------------------------------------------------------
template <int MV>
struct Q4X {
  static constexpr int NM = (MV + 1) / 2;  // MMAs per block: two tokens each
  uint2 *xb;    // [nbx][3 MV digit columns][4 lane-words t] digit pairs (k 4t.., 16+4t..)
  int *cx0;     // [2 MV][nbx] MMA C of lane kind (token, t & 1), column 2t
  int *cx1;     // [2 MV][nbx] column 2t+1
  float *fbk;   // [MV][nbx] block factors 2^-e
  int nb, nbx;  // blocks of K, blocks staged (a multiple of 4; zero past nb)

  __host__ __device__ static size_t bytes(int nbx) {
    return (size_t)nbx * 3 * MV * 32 + (size_t)4 * MV * nbx * 4 + (size_t)MV * nbx * 4;
  }
  __device__ void carve(unsigned char *base, int nb_, int nbx_) {
    nb = nb_;
    nbx = nbx_;
    xb = reinterpret_cast<uint2 *>(base);
    cx0 = reinterpret_cast<int *>(xb + nbx * 3 * MV * 4);
    cx1 = cx0 + 2 * MV * nbx;
    fbk = reinterpret_cast<float *>(cx1 + 2 * MV * nbx);
  }
};

// Digits of 4 consecutive elements packed as s8 bytes.
__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) | ((uint32_t)d << 24);
}

// Stage x [MV][ldx] (times gamma when given) for the Q4_0 MMA; threads
// [0, nth) take part (nth a multiple of 64), 8 lanes per 32-element block.
// x is read through L2 (it may have been written by other SMs this kernel).
// ss_out[warp][m] receives each warp's sum of x^2 (for the RMSNorm).
template <int MV, int U = 4>
__device__ __forceinline__ void q4_stage_x(const Q4X<MV> &X, const float *x, int64_t ldx, const float *gamma, int tid,
                                           int nth, float *ss_out) {
  const int lane = tid & 31, warp = tid >> 5;
  const int q = lane & 7;  // 4-element group of the block; U items' x (and gamma) loads are in flight together
#pragma unroll
  for (int m = 0; m < MV; ++m) {
    float ss = 0.0f;
    // nbx * 8 items is a multiple of 32 and nth a multiple of 32: an item index is valid for a whole warp or
    // for none of its lanes, so the shuffles below always run warp-wide
    for (int base = tid; base < X.nbx * 8; base += U * nth) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int item = base + u * nth, bb = item >> 3;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (item < X.nbx * 8 && bb < X.nb) v[u] = __ldcg(reinterpret_cast<const float4 *>(x + m * ldx + bb * 32 + 4 * q));
      }
      float4 g[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int item = base + u * nth, bb = item >> 3;
        g[u] = make_float4(1.f, 1.f, 1.f, 1.f);
        if (gamma && item < X.nbx * 8 && bb < X.nb) g[u] = *reinterpret_cast<const float4 *>(gamma + bb * 32 + 4 * q);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int item = base + u * nth, bb = item >> 3;
        if (item >= X.nbx * 8) break;  // warp-uniform
        float4 vv = v[u];
        ss += vv.x * vv.x + vv.y * vv.y + vv.z * vv.z + vv.w * vv.w;
        if (gamma) {
          vv.x *= g[u].x;
          vv.y *= g[u].y;
          vv.z *= g[u].z;
          vv.w *= g[u].w;
        }
        float amax = fmaxf(fmaxf(fabsf(vv.x), fabsf(vv.y)), fmaxf(fabsf(vv.z), fabsf(vv.w)));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        // amax in [2^E, 2^(E+1)) -> scale 2^(20 - E); zero / subnormal blocks keep 2^126 (digits ~0)
        const int E = ((__float_as_int(amax) >> 23) & 0xFF) - 127;
        const int e = min(max(20 - E, -126), 126);
        const float scl = __int_as_float((e + 127) << 23);
        const float vf[4] = {vv.x, vv.y, vv.z, vv.w};
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
        // B fragment words of digit columns 3m, 3m+1, 3m+2: lane-word t = q & 3, half q >> 2
        uint32_t *col = reinterpret_cast<uint32_t *>(X.xb + (bb * 3 * MV + 3 * m) * 4) + (q & 3) * 2 + (q >> 2);
        col[0] = pack_s8x4(hi[0], hi[1], hi[2], hi[3]);
        col[8] = pack_s8x4(mi[0], mi[1], mi[2], mi[3]);
        col[16] = pack_s8x4(lo[0], lo[1], lo[2], lo[3]);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
          shi += __shfl_xor_sync(0xffffffffu, shi, o);
          smi += __shfl_xor_sync(0xffffffffu, smi, o);
          slo += __shfl_xor_sync(0xffffffffu, slo, o);
        }
        if (q == 0) {
          // C of the lanes holding (hi, mid) and (lo, 0) of token m
          X.cx0[(2 * m) * X.nbx + bb] = -8 * shi;
          X.cx1[(2 * m) * X.nbx + bb] = -8 * smi;
          X.cx0[(2 * m + 1) * X.nbx + bb] = -8 * slo;
          X.cx1[(2 * m + 1) * X.nbx + bb] = 0;
          // non-finite inputs make the block factor NaN, so the outputs are NaN
          X.fbk[m * X.nbx + bb] =
              amax <= 3.402823466e38f ? __int_as_float((127 - e) << 23) : __int_as_float(0x7fc00000);
        }
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) ss_out[warp * MV + m] = ss;
  }
}

// q4_stage_x (MV = 1) of the tensor-parallel residual fold: the staged vector is h + parts[0] + ...
// + parts[np - 1] (in that order), and its elements [s0, s1) are also stored to hout.  K = stride.
static __device__ __forceinline__ void q4_stage_x_fold(const Q4X<1> &X, const float *h, const float *parts, int np,
                                             int64_t stride, float *hout, int s0, int s1, const float *gamma, int tid,
                                             int nth, float *ss_out) {
  const int lane = tid & 31, warp = tid >> 5;
  const int q = lane & 7;
  float ss = 0.0f;
  for (int item = tid; item < X.nbx * 8; item += nth) {
    const int bb = item >> 3;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (bb < X.nb) {
      const int k = bb * 32 + 4 * q;
      v = __ldcg(reinterpret_cast<const float4 *>(h + k));
      for (int r = 0; r < np; ++r) {
        const float4 pr = __ldcg(reinterpret_cast<const float4 *>(parts + r * stride + k));
        v.x += pr.x;
        v.y += pr.y;
        v.z += pr.z;
        v.w += pr.w;
      }
      const float e4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (k + i >= s0 && k + i < s1) hout[k + i] = e4[i];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      if (gamma) {
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
    uint32_t *col = reinterpret_cast<uint32_t *>(X.xb + (bb * 3) * 4) + (q & 3) * 2 + (q >> 2);
    col[0] = pack_s8x4(hi[0], hi[1], hi[2], hi[3]);
    col[8] = pack_s8x4(mi[0], mi[1], mi[2], mi[3]);
    col[16] = pack_s8x4(lo[0], lo[1], lo[2], lo[3]);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      shi += __shfl_xor_sync(0xffffffffu, shi, o);
      smi += __shfl_xor_sync(0xffffffffu, smi, o);
      slo += __shfl_xor_sync(0xffffffffu, slo, o);
    }
    if (q == 0) {
      X.cx0[bb] = -8 * shi;
      X.cx1[bb] = -8 * smi;
      X.cx0[X.nbx + bb] = -8 * slo;
      X.cx1[X.nbx + bb] = 0;
      X.fbk[bb] = amax <= 3.402823466e38f ? __int_as_float((127 - e) << 23) : __int_as_float(0x7fc00000);
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) ss_out[warp] = ss;
}

__device__ __forceinline__ void imma_u8s8(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1, int c0, int c1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}

// Per-lane constants of the Q4_0 tile consumer (lane of a consumer warp).
template <int MV>
struct Q4Lane {
  static constexpr int NM = Q4X<MV>::NM;
  int a_off, d_off;  // row g's lane word group / scales within a quad (row g + 8: + 512 / + 64)
  const uint2 *xl[NM];
  bool xv[NM];
  const int *c0l[NM], *c1l[NM];
  const float *fbl[NM];
  __device__ void init(const Q4X<MV> &X, int lane) {
    const int gq = lane >> 2, t = lane & 3;
    a_off = (gq * 4 + t) * 16;
    d_off = kQ4QuadCodeBytes + gq * 8;
    // B column gq of MMA i = digit (gq & 3) of token 2i + (gq >> 2); digit 3 is the zero column
#pragma unroll
    for (int im = 0; im < NM; ++im) {
      const int btok = 2 * im + (gq >> 2), dtok = 2 * im + (t >> 1);
      xv[im] = (gq & 3) < 3 && btok < MV;
      xl[im] = X.xb + (xv[im] ? 3 * btok + (gq & 3) : 0) * 4 + t;
      // lanes of a padding token (odd MV) read token 0's values; their D columns are dropped
      c0l[im] = X.cx0 + (dtok < MV ? 4 * im + t : (t & 1)) * X.nbx;
      c1l[im] = X.cx1 + (dtok < MV ? 4 * im + t : (t & 1)) * X.nbx;
      fbl[im] = X.fbk + (dtok < MV ? dtok : 0) * X.nbx;
    }
  }
};

// Multiply-accumulate quad q (global quad index Q of its strip) at qb into acc
// (rows g, g+8 of the strip).
template <int MV>
__device__ __forceinline__ void q4_quad(const unsigned char *qb, int Q, const Q4Lane<MV> &L,
                                        float2 (&acc)[Q4X<MV>::NM]) {
  constexpr int NM = Q4X<MV>::NM;
  const int bb0 = 4 * Q;  // first block of the quad
  const uint4 A0 = *reinterpret_cast<const uint4 *>(qb + L.a_off);
  const uint4 A1 = *reinterpret_cast<const uint4 *>(qb + L.a_off + 512);
  const uint2 D0 = *reinterpret_cast<const uint2 *>(qb + L.d_off);
  const uint2 D1 = *reinterpret_cast<const uint2 *>(qb + L.d_off + 64);
  const uint32_t a0w[4] = {A0.x, A0.y, A0.z, A0.w}, a1w[4] = {A1.x, A1.y, A1.z, A1.w};
#pragma unroll
  for (int im = 0; im < NM; ++im) {
    const int4 C0 = *reinterpret_cast<const int4 *>(L.c0l[im] + bb0);
    const int4 C1 = *reinterpret_cast<const int4 *>(L.c1l[im] + bb0);
    const float4 FB = *reinterpret_cast<const float4 *>(L.fbl[im] + bb0);
    const int c0v[4] = {C0.x, C0.y, C0.z, C0.w}, c1v[4] = {C1.x, C1.y, C1.z, C1.w};
    const float fbv[4] = {FB.x, FB.y, FB.z, FB.w};
#pragma unroll
    for (int bi = 0; bi < 4; ++bi) {
      uint2 B = make_uint2(0u, 0u);
      if (L.xv[im]) B = L.xl[im][(bb0 + bi) * 3 * MV * 4];
      const uint32_t wa = a0w[bi], wb = a1w[bi];
      int di[4];
      imma_u8s8(di, wa & 0x0F0F0F0Fu, wb & 0x0F0F0F0Fu, (wa >> 4) & 0x0F0F0F0Fu, (wb >> 4) & 0x0F0F0F0Fu, B.x, B.y,
                c0v[bi], c1v[bi]);
      const float2 v = make_float2((float)(di[0] * 128 + di[1]), (float)(di[2] * 128 + di[3]));
      // scale pair (row g, row g+8) of block bi: halves bi of D0 and D1
      const uint32_t dpair = __byte_perm(bi < 2 ? D0.x : D0.y, bi < 2 ? D1.x : D1.y, (bi & 1) ? 0x7632 : 0x5410);
      float2 dsc = __half22float2(*reinterpret_cast<const __half2 *>(&dpair));
      dsc = fmul2(dsc, make_float2(fbv[bi], fbv[bi]));
      acc[im] = ffma2(dsc, v, acc[im]);
    }
  }
}

// One tile at st: quads [Q0, Q0 + nqt) of a strip; warp w of the group takes
// quads w, w + 8.
template <int MV>
__device__ __forceinline__ void q4_tile(const unsigned char *st, int Q0, int nqt, int warp, const Q4Lane<MV> &L,
                                        float2 (&acc)[Q4X<MV>::NM]) {
#pragma unroll
  for (int k = 0; k < kQ4TileQuads / kGroupWarps; ++k) {
    const int q = warp + k * kGroupWarps;
    if (q < nqt) q4_quad<MV>(st + q * kQ4QuadBytes, Q0 + q, L, acc);
  }
}

// End of a strip: combine this warp's digit-lane partial sums into
// red[warp][16 rows][MV] and clear acc.
template <int MV>
__device__ __forceinline__ void q4_group_red(float *red, float2 (&acc)[Q4X<MV>::NM], int warp, int lane) {
  const int gq = lane >> 2, t = lane & 3;
#pragma unroll
  for (int im = 0; im < Q4X<MV>::NM; ++im) {
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
}

// Finish strip `strip` (rows 16 strip ..): sum the 8 warps' partials of
// red[8][16][MV] in warp order, scale by mul[m], run the epilogue.  Threads
// [0, nth) of the group take part.  XCHG: the kernel may pass an EPI_XCHG epilogue.
template <int MV, bool XCHG = false>
__device__ __forceinline__ void finish_strip(const QMat &w, const Epilogue &ep, int strip, const float *red,
                                             const float *mul, int tid, int nth) {
  for (int q = tid; q < (kQ4StripRows / 2) * MV; q += nth) {
    const int p = q / MV, m = q % MV;
    float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
    for (int wp = 0; wp < kGroupWarps; ++wp) {
      v0 += red[(wp * kQ4StripRows + 2 * p) * MV + m];
      v1 += red[(wp * kQ4StripRows + 2 * p + 1) * MV + m];
    }
    v0 *= mul[m];
    v1 *= mul[m];
    const int64_t n = (int64_t)strip * kQ4StripRows + 2 * p;
    if constexpr (XCHG) {
      if (ep.mode == EPI_XCHG) {
        if (n + 1 < w.N)
          epi_xchg_pair(ep, n, m, v0, v1);
        else if (n < w.N)
          epi_xchg_one(ep, n, m, v0);
        continue;
      }
    }
    if (n + 1 < w.N)
      epi_store_pair(ep, n, m, v0, v1);
    else if (n < w.N && ep.mode == EPI_PLAIN)
      epi_store_one(ep, n, m, v0);
  }
}

// 1/rms of token m from the per-warp sums of squares (or 1 without a norm).
__device__ __forceinline__ float rms_inv(const float *ss, int nwarps, int MV, int m, int64_t K, float eps,
                                         bool do_norm) {
  float s = 0.0f;
  for (int i = 0; i < nwarps; ++i) s += ss[i * MV + m];
  return do_norm ? __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)K), eps))) : 1.0f;
}

}  // namespace fg
