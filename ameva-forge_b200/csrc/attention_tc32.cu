// Flash attention on tcgen05 for fp32 Q/K/V (the drop-in executeGraph path sends fp32 tensors), with the
// reference semantics (packages/forge/src/tensor/kernels/flash_attention.wgsl.ts:13-178) and fp32-class
// accuracy:
//  * scores carry ~22 bits: every operand is split into fp16 halves, x = hi + lo with hi = fp16(x) and
//    lo = fp16(x - hi), and S = Qh Kh^T + Qh Kl^T + Ql Kh^T (three tcgen05.mma passes, fp32 accumulation
//    in TMEM; the dropped Ql Kl^T is ~2^-22 relative);
//  * P V likewise: O += Ph Vh + Ph Vl + Pl Vh with P = Ph + Pl written by the softmax (P <= 256 keeps
//    both halves in range) and V = Vh + Vl;
//  * fp16 range: K and V of each (batch, KV head) are scaled by a power of two that puts their largest
//    magnitude in [2^14, 2^15), each query row by its own; the scales are exact and are divided out of
//    the softmax scale (scores) and of the output (values).
// A pre-pass (k_kv_absmax, k_kv_split) writes Kh, Kl, Vh, Vl [B][H_kv][capacity][d] fp16 and the two
// scales per KV head into scratch.  The attention kernel (k_attn_tc32) owns 128 query rows of one (batch, head):
//  * TMEM (512 columns): S double buffer [0, 256), O [256, 256 + d), Qh at 384, Ql at 384 + d/2 (Q is
//    the A operand from TMEM, 128 lanes = query rows, fp16 pairs);
//  * four softmax warps, one thread per query row = TMEM lane: load the fp32 Q row, split and store it
//    to TMEM; per 128-key block read the row of S (tcgen05.ld), apply the row's scale and the mask,
//    update the running max m and sum l (exp2 domain; m moves only when a row's maximum grows past 2^8,
//    so P <= 256) and write Ph and Pl as fp16 pairs over the block's S buffer (64 columns each);
//  * one thread of the MMA warp issues S of block j + 2 into the buffer of block j right after
//    O += P_j V_j (the tensor core runs one thread's MMAs in issue order), so S of block j + 1 is being
//    computed while block j is in softmax;
//  * a loader thread brings the K (Kh + Kl) and V (Vh + Vl) blocks with 4-D TMA boxes into one ring of
//    three slots, in the order the MMA thread consumes them: K0, K1, V0, K2, V1, K3, ...
// Every wait is bounded (tma.cuh); on a timeout the device error word is set and the CTA skips its
// stores, drains its copies and frees its TMEM.
#include <cmath>
#include <cstdlib>
#include <string>

#include "q4_gemv.cuh"
#include "runtime.cuh"
#include "tcgen05.cuh"
#include "tmap.cuh"

namespace fg {
namespace {

constexpr int kF32Rows = 128, kF32Keys = 128;
constexpr int kF32SoftmaxWarps = 4, kF32MmaWarp = 4;  // warp 5: the loader
constexpr int kF32Threads = 6 * 32;
constexpr int kF32TmemCols = 512, kF32OCol = 256, kF32QCol = 384;
constexpr float kF32Log2e = 1.4426950408889634f;
constexpr float kF32Lazy = 8.f;

template <int D>
struct F32Geo {
  static constexpr int Atoms = D / 64;
  static constexpr int AtomBytes = 128 * 128;        // [128 keys][64] fp16
  static constexpr int KVBytes = Atoms * AtomBytes;  // one hi or lo block of K or V
  static constexpr int Slot = 2 * KVBytes;           // a ring slot: the hi then the lo block
  static constexpr size_t Need = 1024 + 3 * (size_t)Slot;
  static constexpr size_t Smem = Need > 122880 ? Need : 122880;  // one CTA per SM (512 TMEM columns)
  static_assert(Smem + 512 <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ float f32_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float f32_max3(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}
__device__ __forceinline__ uint32_t f32_pack(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}
// Power of two that puts a largest magnitude `amax` in [2^14, 2^15) (1 for 0 or a non-finite amax).
__device__ __forceinline__ float f32_range_scale(float amax) {
  if (!(amax > 0.f) || !(amax <= 3.402823466e38f)) return 1.f;
  const int e = ((__float_as_int(amax) >> 23) & 0xFF) - 127;  // amax in [2^e, 2^(e+1)) (normal amax)
  const int s = min(max(14 - e, -126), 127);
  return __int_as_float((s + 127) << 23);
}

// Largest |K| and |V| of each (batch, KV head) over every cache row: amax[0][bh], amax[1][bh] as float
// bits (non-negative floats order like their bit patterns), zeroed by the host.
__global__ void k_kv_absmax(const float *__restrict__ k, const float *__restrict__ v, int64_t kv_sb, int64_t kv_sh,
                            int Hkv, int64_t elems, unsigned *__restrict__ amax) {
  const int bh = blockIdx.y, b = bh / Hkv, hk = bh % Hkv;
  const float *kb = k + (int64_t)b * kv_sb + (int64_t)hk * kv_sh, *vb = v + (int64_t)b * kv_sb + (int64_t)hk * kv_sh;
  float mk = 0.f, mv = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < elems / 4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4 *>(kb)[i], c = reinterpret_cast<const float4 *>(vb)[i];
    mk = fmaxf(mk, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
    mv = fmaxf(mv, fmaxf(fmaxf(fabsf(c.x), fabsf(c.y)), fmaxf(fabsf(c.z), fabsf(c.w))));
    // a NaN anywhere makes the head's scale 1 (the outputs are NaN as in the reference)
    if (isnan(a.x + a.y + a.z + a.w)) mk = INFINITY;
    if (isnan(c.x + c.y + c.z + c.w)) mv = INFINITY;
  }
  mk = warp_max(mk);
  mv = warp_max(mv);
  if ((threadIdx.x & 31) == 0) {
    atomicMax(amax + bh, __float_as_uint(mk));
    atomicMax(amax + gridDim.y + bh, __float_as_uint(mv));
  }
}

// Kh, Kl, Vh, Vl [B][H_kv][rows][d] fp16 of K and V scaled per (batch, KV head); inv[0][bh] = 1 / (K scale),
// inv[1][bh] = 1 / (V scale).
__global__ void k_kv_split(const float *__restrict__ k, const float *__restrict__ v, int64_t kv_sb, int64_t kv_sh,
                           int Hkv, int64_t elems, const unsigned *__restrict__ amax, __half *__restrict__ kh,
                           __half *__restrict__ kl, __half *__restrict__ vh, __half *__restrict__ vl,
                           float *__restrict__ inv) {
  const int bh = blockIdx.y, b = bh / Hkv, hk = bh % Hkv;
  const float sk = f32_range_scale(__uint_as_float(amax[bh])), sv = f32_range_scale(__uint_as_float(amax[gridDim.y + bh]));
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    inv[bh] = 1.f / sk;  // exact: a power of two
    inv[gridDim.y + bh] = 1.f / sv;
  }
  const float *kb = k + (int64_t)b * kv_sb + (int64_t)hk * kv_sh, *vb = v + (int64_t)b * kv_sb + (int64_t)hk * kv_sh;
  const int64_t ob = (int64_t)bh * elems;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < elems / 4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4 *>(kb)[i], c = reinterpret_cast<const float4 *>(vb)[i];
    const float ka[4] = {a.x * sk, a.y * sk, a.z * sk, a.w * sk}, va[4] = {c.x * sv, c.y * sv, c.z * sv, c.w * sv};
    uint32_t hi[2], lo[2], vhi[2], vlo[2];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const __half2 h = __floats2half2_rn(ka[2 * p], ka[2 * p + 1]);
      const float2 hf = __half22float2(h);
      const __half2 l = __floats2half2_rn(ka[2 * p] - hf.x, ka[2 * p + 1] - hf.y);
      hi[p] = *reinterpret_cast<const uint32_t *>(&h);
      lo[p] = *reinterpret_cast<const uint32_t *>(&l);
      const __half2 g = __floats2half2_rn(va[2 * p], va[2 * p + 1]);
      const float2 gf = __half22float2(g);
      const __half2 gl = __floats2half2_rn(va[2 * p] - gf.x, va[2 * p + 1] - gf.y);
      vhi[p] = *reinterpret_cast<const uint32_t *>(&g);
      vlo[p] = *reinterpret_cast<const uint32_t *>(&gl);
    }
    reinterpret_cast<uint2 *>(kh + ob)[i] = make_uint2(hi[0], hi[1]);
    reinterpret_cast<uint2 *>(kl + ob)[i] = make_uint2(lo[0], lo[1]);
    reinterpret_cast<uint2 *>(vh + ob)[i] = make_uint2(vhi[0], vhi[1]);
    reinterpret_cast<uint2 *>(vl + ob)[i] = make_uint2(vlo[0], vlo[1]);
  }
}

struct F32Args {
  AttnArgs a;
  const float *kinv;  // [B * H_kv] 1 / (K scale) of each (batch, KV head); V's follow
};

template <int D>
__global__ void __launch_bounds__(kF32Threads, 1)
    k_attn_tc32(const __grid_constant__ CUtensorMap tkh, const __grid_constant__ CUtensorMap tkl,
                const __grid_constant__ CUtensorMap tvh, const __grid_constant__ CUtensorMap tvl, F32Args f) {
  using G = F32Geo<D>;
  const AttnArgs &a = f.a;
  extern __shared__ __align__(1024) unsigned char f32_smem_raw[];
  unsigned char *sm = f32_smem_raw + ((1024 - (smem_u32(f32_smem_raw) & 1023)) & 1023);
  __shared__ __align__(8) uint64_t rfull[3], rempty[3], sfull[2], pfull, pvdone, qready;
  __shared__ uint32_t s_taddr;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qb = gridDim.x - 1 - blockIdx.x;  // the longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z, hk = h / (a.H / a.Hkv);
  const int i0 = qb * kF32Rows;

  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int nkv = a.n_kv_dev ? a.n_kv_dev[b] + a.n_kv_add : a.n_kv;
  int kend = nkv;
  if (a.causal) kend = min(kend, nkv - a.Nq + i0 + kF32Rows);
  const int nblk = kend > 0 ? (kend + kF32Keys - 1) / kF32Keys : 0;
  if (nblk == 0) {  // no row of the tile sees a key: out = 0
    if (tid < kF32Rows && i0 + tid < a.Nq) {
      float *o = a.o + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + (int64_t)(i0 + tid) * a.o_si;
      for (int c = 0; c < D; c += 4) *reinterpret_cast<float4 *>(o + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < 3; ++s) {
      mbar_init(&rfull[s], 1);  // the loader's expect_tx
      mbar_init(&rempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) mbar_init(&sfull[s], 1);
    mbar_init(&pfull, kF32SoftmaxWarps);
    mbar_init(&pvdone, 1);
    mbar_init(&qready, kF32SoftmaxWarps);
    fence_barrier_init();
  }
  if (warp == kF32MmaWarp) tmem_alloc(&s_taddr, kF32TmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = s_taddr;
  bool ok = true;

  if (warp < kF32SoftmaxWarps) {
    // ============ softmax warps: thread = query row = TMEM lane ============
    const int r = 32 * warp + lane, qi = i0 + r;
    const uint32_t trow = taddr + ((uint32_t)(32 * warp) << 16);
    float rs = 1.f;  // this row's range scale
    {
      // the fp32 row of Q, scaled and split into fp16 halves, into TMEM columns [384, 384 + d/2) (hi)
      // and [384 + d/2, 384 + d) (lo)
      float qv[D];
      const float *qp = reinterpret_cast<const float *>(a.q) + (int64_t)b * a.q_sb + (int64_t)h * a.q_sh +
                        (int64_t)qi * a.q_si;
#pragma unroll
      for (int c = 0; c < D; c += 4) {
        const float4 x = qi < a.Nq ? *reinterpret_cast<const float4 *>(qp + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        qv[c] = x.x;
        qv[c + 1] = x.y;
        qv[c + 2] = x.z;
        qv[c + 3] = x.w;
      }
      float am = 0.f;
      bool nan = false;
#pragma unroll
      for (int c = 0; c < D; ++c) {
        am = fmaxf(am, fabsf(qv[c]));
        nan = nan || isnan(qv[c]);
      }
      rs = f32_range_scale(nan ? INFINITY : am);
#pragma unroll
      for (int c0 = 0; c0 < D / 2; c0 += 16) {  // 16 columns = 32 values per store
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const float x0 = qv[2 * (c0 + p)] * rs, x1 = qv[2 * (c0 + p) + 1] * rs;
          const __half2 hh = __floats2half2_rn(x0, x1);
          const float2 hf = __half22float2(hh);
          hi[p] = *reinterpret_cast<const uint32_t *>(&hh);
          lo[p] = f32_pack(x0 - hf.x, x1 - hf.y);
        }
        tmem_st16_issue(trow + kF32QCol + c0, hi);
        tmem_st16_issue(trow + kF32QCol + D / 2 + c0, lo);
      }
      tmem_st_wait();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&qready);

    // scores in log2 units: the scale, undone for Q's and K's range scales (powers of two: exact)
    const float sl2 = a.scale * kF32Log2e / rs * f.kinv[b * a.Hkv + hk];
    const int lim = a.causal ? min(nkv - a.Nq + qi + 1, nkv) : nkv;  // keys [0, lim) visible to this row
    float m = -1e30f * kF32Log2e, l = 0.f;
    const uint32_t to = trow + kF32OCol;
    for (int j = 0; j < nblk; ++j) {
      const int sb = j & 1, kb = j * kF32Keys;
      const uint32_t ts = trow + sb * kF32Keys;
      ok = ok && mbar_wait(&sfull[sb], (uint32_t)(j >> 1) & 1, a.err, DEVERR_ATTN_FULL);
      __syncwarp();
      tc_fence_after();
      uint32_t s0[32], s1[32], s2[32], s3[32];
      tmem_ld32_issue(ts, s0);
      tmem_ld32_issue(ts + 32, s1);
      tmem_ld32_issue(ts + 64, s2);
      tmem_ld32_issue(ts + 96, s3);
      tmem_ld_wait(s0);
      tmem_ld_wait(s1);
      tmem_ld_wait(s2);
      tmem_ld_wait(s3);
      float v[128];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        v[e] = __uint_as_float(s0[e]);
        v[32 + e] = __uint_as_float(s1[e]);
        v[64 + e] = __uint_as_float(s2[e]);
        v[96 + e] = __uint_as_float(s3[e]);
      }
      float mul = sl2;
      if (__any_sync(0xffffffffu, kb + kF32Keys > lim)) {  // the causal diagonal or the live-length edge
#pragma unroll
        for (int e = 0; e < 128; ++e) v[e] = kb + e < lim ? v[e] * sl2 : -INFINITY;
        mul = 1.f;
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < 128; e += 8) {
        mx4[0] = f32_max3(mx4[0], v[e], v[e + 1]);
        mx4[1] = f32_max3(mx4[1], v[e + 2], v[e + 3]);
        mx4[2] = f32_max3(mx4[2], v[e + 4], v[e + 5]);
        mx4[3] = f32_max3(mx4[3], v[e + 6], v[e + 7]);
      }
      const float mx = fmaxf(f32_max3(mx4[0], mx4[1], mx4[2]), mx4[3]) * mul;
      const float mc = fmaxf(m, mx);
      const bool grow = mc - m > kF32Lazy;
      float alpha = 1.f;
      if (grow) {
        alpha = f32_ex2(m - mc);
        m = mc;
      }
      float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 mul2 = make_float2(mul, mul), negm = make_float2(-m, -m);
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // keys 32c .. 32c+31 -> Ph columns 16c .., Pl columns 64 + 16c ..
        uint32_t ph[16], pl[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 x = ffma2(make_float2(v[32 * c + e], v[32 * c + e + 1]), mul2, negm);
          const float2 p = make_float2(f32_ex2(x.x), f32_ex2(x.y));
          sum2[(e >> 1) & 1] = fadd2(sum2[(e >> 1) & 1], p);
          const __half2 hh = __floats2half2_rn(p.x, p.y);
          const float2 hf = __half22float2(hh);
          ph[e >> 1] = *reinterpret_cast<const uint32_t *>(&hh);
          pl[e >> 1] = f32_pack(p.x - hf.x, p.y - hf.y);
        }
        tmem_st16_issue(ts + 16 * c, ph);
        tmem_st16_issue(ts + 64 + 16 * c, pl);
      }
      if (__any_sync(0xffffffffu, grow && j > 0)) {
        // O *= alpha once P V of the previous block has completed (S of this block was issued before it)
        ok = ok && mbar_wait(&pvdone, (uint32_t)(j - 1) & 1, a.err, DEVERR_ATTN_EMPTY);
        __syncwarp();
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 16; ++c) {
          float o[32];
          tmem_ld16(to + 16 * c, o);
          uint32_t ob[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) ob[e] = __float_as_uint(o[e] * alpha);
          tmem_st16_issue(to + 16 * c, ob);
          tmem_st_wait();
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull);
      l = l * alpha + ((sum2[0].x + sum2[0].y) + (sum2[1].x + sum2[1].y));
    }
    // P V of the last two blocks: completion nblk - 3 is known (the last scores were issued after it),
    // so the phases are waited for in order (a parity wait alone could see an older phase)
    if (nblk >= 2) ok = ok && mbar_wait(&pvdone, (uint32_t)(nblk - 2) & 1, a.err, DEVERR_ATTN_FULL);
    ok = ok && mbar_wait(&pvdone, (uint32_t)(nblk - 1) & 1, a.err, DEVERR_ATTN_FULL);
    __syncwarp();
    tc_fence_after();
    // out = O / l, undone for V's range scale
    const float inv = f.kinv[gridDim.z * a.Hkv + b * a.Hkv + hk] / fmaxf(l, 1e-12f);
    float *orow = a.o + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + (int64_t)qi * a.o_si;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      float o[32];
      tmem_ld32(to + 32 * c, o);
      if (ok && qi < a.Nq) {
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4 *>(orow + 32 * c + e) =
              make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
      }
    }
    tc_fence_before();
  } else if (warp == kF32MmaWarp) {
    // ================= MMA issuer: consumes the ring items in the order S0, S1, PV0, S2, PV1, S3, ... =========
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16_f32acc(kF32Rows, kF32Keys, false);
      constexpr uint32_t idO = idesc_f16_f32acc(kF32Rows, D, true);
      ok = ok && mbar_wait(&qready, 0, a.err, DEVERR_ATTN_FULL);
      int it = 0;  // ring items taken
      auto take = [&]() {
        const int slot = it % 3;
        ok = ok && mbar_wait(&rfull[slot], (uint32_t)(it / 3) & 1, a.err, DEVERR_ATTN_FULL);
        ++it;
        tc_fence_after();
        return smem_u32(sm + slot * G::Slot);
      };
      // S_j = Qh Kh^T + Qh Kl^T + Ql Kh^T into buffer j % 2 (Q from TMEM, K = 16 head columns per MMA)
      auto issue_s = [&](int j) {
        const int sb = j & 1, slot = it % 3;
        const uint32_t kh = take(), kl = kh + G::KVBytes;
        if (ok) {
#pragma unroll
          for (int pass = 0; pass < 3; ++pass) {
            const uint32_t qcol = taddr + kF32QCol + (pass == 2 ? D / 2 : 0), kb = pass == 1 ? kl : kh;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * G::AtomBytes + 32 * (kk & 3);
              umma_f16_tmem_a(taddr + sb * kF32Keys, qcol + 8 * kk, smem_desc_sw128(kb + off), idS,
                              (pass > 0 || kk > 0) ? 1u : 0u);
            }
          }
        }
        umma_commit(&sfull[sb]);
        umma_commit(&rempty[slot]);
      };
      // O += Ph Vh + Ph Vl + Pl Vh (P from TMEM: Ph at the block's S buffer, Pl 64 columns further; K = 16
      // keys = 8 columns per MMA; V MN-major)
      auto issue_pv = [&](int j) {
        const int sb = j & 1;
        ok = ok && mbar_wait_poll(&pfull, (uint32_t)j & 1, a.err, DEVERR_ATTN_FULL);
        const int slot = it % 3;
        const uint32_t vh = take(), vl = vh + G::KVBytes;
        if (ok) {
#pragma unroll
          for (int pass = 0; pass < 3; ++pass) {
            const uint32_t pcol = taddr + sb * kF32Keys + (pass == 2 ? 64 : 0), vb = pass == 1 ? vl : vh;
#pragma unroll
            for (int kk = 0; kk < kF32Keys / 16; ++kk)
              umma_f16_tmem_a(taddr + kF32OCol, pcol + 8 * kk, smem_desc_sw128(vb + kk * 2048, G::AtomBytes, 1024),
                              idO, (j > 0 || pass > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&pvdone);
        umma_commit(&rempty[slot]);
      };
      issue_s(0);
      if (nblk > 1) issue_s(1);
      for (int j = 0; j < nblk; ++j) {
        issue_pv(j);
        // S of block j + 2 overwrites P_j: issued after P_j V_j by this thread, it runs after P_j is read
        if (j + 2 < nblk) issue_s(j + 2);
      }
    }
  } else if (lane == 0) {
    // ================= loader: the ring items in the MMA thread's order, three slots =================
    const uint64_t pol = l2_evict_last_policy();  // re-read by the other query blocks and GQA heads
    tma_prefetch_desc(&tkh);
    tma_prefetch_desc(&tkl);
    tma_prefetch_desc(&tvh);
    tma_prefetch_desc(&tvl);
    int it = 0, issued = 0;
    auto put = [&](bool isv, int j) {
      const int slot = it % 3;
      if (it >= 3) ok = ok && mbar_wait(&rempty[slot], (uint32_t)(it / 3 - 1) & 1, a.err, DEVERR_ATTN_EMPTY);
      if (ok) {
        unsigned char *dst = sm + slot * G::Slot;
        mbar_arrive_expect_tx(&rfull[slot], (uint32_t)G::Slot);
        for (int u = 0; u < G::Atoms; ++u) {
          tma_load_4d(dst + u * G::AtomBytes, isv ? &tvh : &tkh, 64 * u, j * kF32Keys, hk, b, &rfull[slot], pol);
          tma_load_4d(dst + G::KVBytes + u * G::AtomBytes, isv ? &tvl : &tkl, 64 * u, j * kF32Keys, hk, b, &rfull[slot],
                      pol);
        }
        issued = it + 1;
      } else {
        mbar_arrive(&rfull[slot]);
      }
      ++it;
    };
    put(false, 0);
    if (nblk > 1) put(false, 1);
    for (int j = 0; j < nblk; ++j) {
      put(true, j);
      if (j + 2 < nblk) put(false, j + 2);
    }
    // drain: no copy may still be landing in shared memory when the CTA exits
    for (int i = issued > 3 ? issued - 3 : 0; i < issued; ++i) mbar_wait_drain(&rfull[i % 3], (uint32_t)(i / 3) & 1);
  }
  __syncthreads();
  if (warp == kF32MmaWarp) {
    tc_fence_after();
    tmem_dealloc(taddr, kF32TmemCols);
  }
}

template <int D>
void launch_tc32_d(Ctx &c, const AttnArgs &a, cudaStream_t s) {
  using G = F32Geo<D>;
  const int64_t bh = (int64_t)a.B * a.Hkv, elems = a.kv_sh, rows = a.kv_sh / D;
  const uint64_t half_bytes = align_up((uint64_t)bh * elems * 2, 256), head = align_up((uint64_t)16 * bh, 256);
  const uint64_t bytes = head + 4 * half_bytes;
  unsigned char *scr = static_cast<unsigned char *>(c.alloc(bytes));
  try {
    unsigned *amax = reinterpret_cast<unsigned *>(scr);  // [2][B H_kv], then the inverse scales [2][B H_kv]
    float *inv = reinterpret_cast<float *>(scr) + 2 * bh;
    __half *kh = reinterpret_cast<__half *>(scr + head), *kl = reinterpret_cast<__half *>(scr + head + half_bytes),
           *vh = reinterpret_cast<__half *>(scr + head + 2 * half_bytes),
           *vl = reinterpret_cast<__half *>(scr + head + 3 * half_bytes);
    FG_CUDA(cudaMemsetAsync(amax, 0, (size_t)2 * bh * 4, s));
    const dim3 pg((unsigned)std::min<int64_t>(std::max<int64_t>(1, ceil_div(elems / 4, 256)), 64), (unsigned)bh);
    k_kv_absmax<<<pg, 256, 0, s>>>(reinterpret_cast<const float *>(a.k), reinterpret_cast<const float *>(a.v), a.kv_sb,
                                   a.kv_sh, a.Hkv, elems, amax);
    FG_LAUNCH_CHECK();
    k_kv_split<<<pg, 256, 0, s>>>(reinterpret_cast<const float *>(a.k), reinterpret_cast<const float *>(a.v), a.kv_sb,
                                  a.kv_sh, a.Hkv, elems, amax, kh, kl, vh, vl, inv);
    FG_LAUNCH_CHECK();
    // Kh, Kl, Vh, Vl [B][H_kv][rows][D] fp16: boxes of [128 keys][64 columns]
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)rows, (uint64_t)a.Hkv, (uint64_t)a.B};
    const uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)elems * 2, (uint64_t)a.Hkv * elems * 2};
    const uint32_t box[4] = {64, kF32Keys, 1, 1};
    const CUtensorMap tkh = make_tmap_4d(kh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap tkl = make_tmap_4d(kl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap tvh = make_tmap_4d(vh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap tvl = make_tmap_4d(vl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    static unsigned long long attr_set = 0;
    int dev = 0;
    FG_CUDA(cudaGetDevice(&dev));
    if (!(attr_set & (1ull << dev))) {
      FG_CUDA(cudaFuncSetAttribute(k_attn_tc32<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G::Smem));
      attr_set |= 1ull << dev;
    }
    F32Args f{a, inv};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(a.Nq, kF32Rows), (unsigned)a.H, (unsigned)a.B);
    cfg.blockDim = dim3(kF32Threads);
    cfg.dynamicSmemBytes = G::Smem;
    cfg.stream = s;
    FG_CUDA(cudaLaunchKernelEx(&cfg, k_attn_tc32<D>, tkh, tkl, tvh, tvl, f));
  } catch (...) {
    c.free_async(scr, bytes);
    throw;
  }
  c.free_async(scr, bytes);
}

bool f32_aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

bool attn_tc32_supported(const AttnArgs &a) {
  static const bool simt = [] {
    const char *e = std::getenv("FORGE_B200_ATTN");
    return e && std::string(e) == "simt";
  }();
  return !simt && !a.kv_f16 && !a.q_f16 && (a.d == 64 || a.d == 128) && a.Nq >= 16 && a.Hkv >= 1 &&
         a.H % a.Hkv == 0 && a.scale >= 0.f && f32_aligned16(a.q) && f32_aligned16(a.k) && f32_aligned16(a.v) &&
         f32_aligned16(a.o) && a.q_sb % 4 == 0 && a.q_sh % 4 == 0 && a.q_si % 4 == 0 && a.o_sb % 4 == 0 &&
         a.o_sh % 4 == 0 && a.o_si % 4 == 0 && a.kv_sh >= (int64_t)a.d && a.kv_sh % a.d == 0 &&
         (a.B == 1 || a.kv_sb == (int64_t)a.Hkv * a.kv_sh) && a.B <= 65535;
}

void launch_attention(Ctx &c, const AttnArgs &a, cudaStream_t s) {
  if (a.B > 0 && a.Nq > 0 && a.H > 0 && attn_tc32_supported(a)) {
    if (a.d == 64)
      launch_tc32_d<64>(c, a, s);
    else
      launch_tc32_d<128>(c, a, s);
    return;
  }
  launch_attention(a, c.num_sms, s);
}

}  // namespace fg
