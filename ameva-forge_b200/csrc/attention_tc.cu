// Flash attention on the 5th-generation tensor cores (tcgen05, sm_100a) for
// fp16 K/V (fp32 or fp16 Q) and head_dim 64 or 128, with the reference
// semantics (packages/forge/src/tensor/kernels/flash_attention.wgsl.ts:13-178):
//   GQA kv_head = h / (H / H_kv); causal: key j visible iff
//   j < N_kv - N_q + i + 1; running max starts at -1e30; out = acc / max(l, 1e-12).
//
// A CTA owns two tiles of 128 query rows of one (batch, head), the query
// blocks 2p and 2p + 1, which share every K/V block they read, and walks the
// visible keys in blocks of 128.  The two tiles take turns on the tensor core:
// while one tile's softmax runs, the MMA pipe computes the other tile's P V and
// next scores.
//  * a loader thread brings K and V blocks into two-slot rings with 4-D TMA
//    boxes [128 keys][64 head columns] (128-byte swizzle, rows past the cache
//    extent read as zero);
//  * one thread of the MMA warp issues, per tile t, S_t = Q_t K^T (M = 128
//    queries, N = 128 keys, K = head_dim) into TMEM columns [128 t, 128 t + 128)
//    and O_t += P_t V (N = head_dim, K = 128 keys, V read MN-major) into
//    columns [256 + 128 t, ...), with P_t read from TMEM (the A operand) where
//    the softmax wrote it over the first 64 columns of S_t.  S_t of the next
//    block is issued right after P_t V: the tensor core runs one thread's MMAs
//    in issue order, so it lands after P_t V has read P_t.  The issuing thread
//    polls for P with a short suspend time, to start the MMAs soon after the
//    softmax warps arrive;
//  * each tile has a softmax warpgroup, one thread per query row = TMEM lane:
//    it reads the row of S (tcgen05.ld), applies the scale and the
//    causal/extent mask, updates the running max m and sum l (exp2 domain), and
//    writes P as fp16 pairs (tcgen05.st).  m moves only when a row's maximum
//    grows by more than 2^8 (P then stays <= 256, exact in fp16 range); only
//    then is the O row rescaled in TMEM (P_t V of the previous block completed
//    before this block's scores did);
//  * the same threads finish with out = O / max(l, 1e-12) in fp32.
// Every wait is bounded (tma.cuh); on a timeout the device error word is set
// and the CTA skips its stores, drains its copies and frees its TMEM.
#include <cstdlib>
#include <string>

#include "q4_gemv.cuh"
#include "runtime.cuh"
#include "tcgen05.cuh"
#include "tmap.cuh"

namespace fg {
namespace {

constexpr int kFaRows = 128;  // queries per tile: UMMA M, TMEM lanes
constexpr int kFaKeys = 128;  // keys per block: N of S = Q K^T, K of O += P V
constexpr int kFaTiles = 2;   // query tiles per CTA
constexpr int kFaSoftmaxWarps = 4 * kFaTiles;
constexpr int kFaMmaWarp = kFaSoftmaxWarps;       // then the loader warp
constexpr int kFaThreads = (kFaSoftmaxWarps + 2) * 32;
constexpr int kFaTmemCols = 512;  // S_t / P_t at [128 t, 128 t + 128), O_t at [256 + 128 t, + head_dim)
constexpr int kFaOCol = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazy = 8.f;  // log2 of the largest P before the reference max moves

template <int D>
struct FaGeo {
  static constexpr int Atoms = D / 64;              // 64-column swizzle atoms along head_dim
  static constexpr int AtomBytes = 128 * 128;       // [128 rows][64] fp16
  static constexpr int QBytes = Atoms * AtomBytes;  // one Q tile, K-major
  static constexpr int KVBytes = Atoms * AtomBytes; // one K or V block
  static constexpr size_t KOff = kFaTiles * (size_t)QBytes, VOff = KOff + 2 * (size_t)KVBytes,
                          End = VOff + 2 * (size_t)KVBytes;
  // + 1 KB for the 1024-byte alignment; at least 120 KB, so that one CTA
  // holds an SM (it allocates all 512 TMEM columns)
  static constexpr size_t Need = 1024 + End;
  static constexpr size_t Smem = Need > 122880 ? Need : 122880;
  static_assert(Smem + 512 <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// Visible keys of query tile `qb`: [0, kend), in 128-key blocks.
__device__ __forceinline__ int fa_blocks(const AttnArgs &a, int nkv, int qb) {
  const int i0 = qb * kFaRows;
  if (i0 >= a.Nq) return 0;
  int kend = nkv;
  if (a.causal) kend = min(kend, nkv - a.Nq + i0 + kFaRows);
  return kend > 0 ? (kend + kFaKeys - 1) / kFaKeys : 0;
}

template <int D>
__global__ void __launch_bounds__(kFaThreads, 1)
    k_attn_tc(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, AttnArgs a) {
  using G = FaGeo<D>;
  extern __shared__ __align__(1024) unsigned char fa_smem_raw[];
  unsigned char *sm = fa_smem_raw + ((1024 - (smem_u32(fa_smem_raw) & 1023)) & 1023);
  unsigned char *qs = sm, *ks = sm + G::KOff, *vs = sm + G::VOff;
  __shared__ __align__(8) uint64_t kfull[2], kempty[2], vfull[2], vempty[2];
  __shared__ __align__(8) uint64_t sfull[kFaTiles], pfull[kFaTiles], pvdone[kFaTiles], qready;
  __shared__ uint32_t s_taddr;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.x, b = blockIdx.y, pair = gridDim.z - 1 - blockIdx.z;  // the longest causal rows first
  const int hk = h / (a.H / a.Hkv);

  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int nkv = a.n_kv_dev ? a.n_kv_dev[b] + a.n_kv_add : a.n_kv;
  int nb[kFaTiles];
#pragma unroll
  for (int t = 0; t < kFaTiles; ++t) nb[t] = fa_blocks(a, nkv, kFaTiles * pair + t);
  const int nblk = max(nb[0], nb[1]);

  if (nblk == 0) {  // no row of either tile sees a key: acc = 0, l = 0, out = 0
    const int qi = (kFaTiles * pair + (tid >> 7)) * kFaRows + (tid & 127);
    if (tid < kFaTiles * kFaRows && qi < a.Nq) {
      float *o = a.o + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + (int64_t)qi * a.o_si;
      for (int c = 0; c < D; c += 4) *reinterpret_cast<float4 *>(o + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kfull[s], 1);  // the loader's expect_tx
      mbar_init(&kempty[s], 1);
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    for (int t = 0; t < kFaTiles; ++t) {
      mbar_init(&sfull[t], 1);
      mbar_init(&pfull[t], 4);  // the tile's four softmax warps
      mbar_init(&pvdone[t], 1);
    }
    mbar_init(&qready, kFaSoftmaxWarps);
    fence_barrier_init();
  }
  if (warp == kFaMmaWarp) tmem_alloc(&s_taddr, kFaTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = s_taddr;
  bool ok = true;

  if (warp < kFaSoftmaxWarps) {
    // ============ softmax warpgroup t: thread = query row = TMEM lane of tile t ============
    const int t = warp >> 2, quad = warp & 3, r = 32 * quad + lane, qi = (kFaTiles * pair + t) * kFaRows + r;
    const int nbt = t ? nb[1] : nb[0];
    {  // the row of Q, fp16, into the K-major swizzled tile (row r at r * 128, chunk c at c ^ (r & 7))
      unsigned char *qt = qs + t * G::QBytes;
      const int64_t qoff = (int64_t)b * a.q_sb + (int64_t)h * a.q_sh + (int64_t)qi * a.q_si;
#pragma unroll 4
      for (int c = 0; c < D / 8; ++c) {  // 16-byte chunk c: head columns 8c .. 8c+7
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (nbt > 0 && qi < a.Nq) {
          if (a.q_f16) {
            v = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __half *>(a.q) + qoff + 8 * c);
          } else {
            const float *qf = reinterpret_cast<const float *>(a.q) + qoff + 8 * c;
            const float4 x0 = *reinterpret_cast<const float4 *>(qf), x1 = *reinterpret_cast<const float4 *>(qf + 4);
            v = make_uint4(pack_f16x2(x0.x, x0.y), pack_f16x2(x0.z, x0.w), pack_f16x2(x1.x, x1.y),
                           pack_f16x2(x1.z, x1.w));
          }
        }
        *reinterpret_cast<uint4 *>(qt + (c >> 3) * G::AtomBytes + r * 128 + (((c & 7) ^ (r & 7)) * 16)) = v;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&qready);

    const float sl2 = a.scale * kLog2e;  // scores in log2 units (scale >= 0, checked on the host)
    const int lim = a.causal ? min(nkv - a.Nq + qi + 1, nkv) : nkv;  // keys [0, lim) visible to this row
    float m = -1e30f * kLog2e, l = 0.f;
    const uint32_t trow = taddr + ((uint32_t)(32 * quad) << 16), ts = trow + kFaKeys * t,
                   to = trow + kFaOCol + 128 * t;
    for (int j = 0; j < nbt; ++j) {
      const int kb = j * kFaKeys;
      ok = ok && mbar_wait(&sfull[t], (uint32_t)j & 1, a.err, DEVERR_ATTN_FULL);
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
      if (__any_sync(0xffffffffu, kb + kFaKeys > lim)) {  // the causal diagonal or the live-length edge
#pragma unroll
        for (int e = 0; e < 128; ++e) v[e] = kb + e < lim ? v[e] * sl2 : -INFINITY;
        mul = 1.f;
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < 128; e += 8) {  // four independent chains of three-input maxima
        mx4[0] = fmax3(mx4[0], v[e], v[e + 1]);
        mx4[1] = fmax3(mx4[1], v[e + 2], v[e + 3]);
        mx4[2] = fmax3(mx4[2], v[e + 4], v[e + 5]);
        mx4[3] = fmax3(mx4[3], v[e + 6], v[e + 7]);
      }
      const float mx = fmaxf(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3]) * mul;
      // the reference max moves only when this row's maximum grew by more than kLazy
      const float mc = fmaxf(m, mx);
      const bool grow = mc - m > kLazy;
      float alpha = 1.f;
      if (grow) {
        alpha = ex2(m - mc);
        m = mc;
      }
      float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 mul2 = make_float2(mul, mul), negm = make_float2(-m, -m);
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // keys 32c .. 32c+31 -> P columns 16c .. 16c+15 (two fp16 per column)
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 x = ffma2(make_float2(v[32 * c + e], v[32 * c + e + 1]), mul2, negm);
          const float2 p = make_float2(ex2(x.x), ex2(x.y));
          sum2[(e >> 1) & 1] = fadd2(sum2[(e >> 1) & 1], p);
          pk[e >> 1] = pack_f16x2(p.x, p.y);
        }
        tmem_st16_issue(ts + 16 * c, pk);
      }
      if (__any_sync(0xffffffffu, grow && j > 0)) {
        // O_t *= alpha: P_t V of the previous block completed before these scores were issued
#pragma unroll 1
        for (int c = 0; c < D / 16; ++c) {  // 16 columns at a time: few registers besides the loop state
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
      if (lane == 0) mbar_arrive(&pfull[t]);
      l = l * alpha + ((sum2[0].x + sum2[0].y) + (sum2[1].x + sum2[1].y));
    }
    if (nbt > 0) {
      ok = ok && mbar_wait(&pvdone[t], (uint32_t)(nbt - 1) & 1, a.err, DEVERR_ATTN_FULL);
      __syncwarp();
      tc_fence_after();
    }
    const float inv = 1.f / fmaxf(l, 1e-12f);
    float *orow = a.o + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + (int64_t)qi * a.o_si;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      float o[32];
      if (nbt > 0) {
        tmem_ld32(to + 32 * c, o);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = 0.f;
      }
      if (ok && qi < a.Nq) {
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4 *>(orow + 32 * c + e) =
              make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
      }
    }
    tc_fence_before();
  } else if (warp == kFaMmaWarp) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16_f32acc(kFaRows, kFaKeys, false);
      constexpr uint32_t idO = idesc_f16_f32acc(kFaRows, D, true);
      const uint32_t qa = smem_u32(qs);
      ok = ok && mbar_wait(&qready, 0, a.err, DEVERR_ATTN_FULL);
      auto issue_s = [&](int t, int j) {  // S_t = Q_t K_j^T, K = 16 head columns per MMA
        const uint32_t ka = smem_u32(ks + (j & 1) * G::KVBytes), qt = qa + t * G::QBytes;
        if (ok) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * G::AtomBytes + 32 * (kk & 3);
            umma_f16(taddr + kFaKeys * t, smem_desc_sw128(qt + off), smem_desc_sw128(ka + off), idS,
                     kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(&sfull[t]);
      };
      auto issue_pv = [&](int t, int j) {  // O_t += P_t V_j, K = 16 keys (8 TMEM columns of P) per MMA
        const uint32_t va = smem_u32(vs + (j & 1) * G::KVBytes);
        if (ok) {
#pragma unroll
          for (int kk = 0; kk < kFaKeys / 16; ++kk) {
            // V block [atom of 64 head columns][128 keys][64], MN-major: 16 keys = 2048 bytes
            // per step, 8-key atoms 1024 bytes apart, the next 64 head columns one atom further
            umma_f16_tmem_a(taddr + kFaOCol + 128 * t, taddr + kFaKeys * t + 8 * kk,
                            smem_desc_sw128(va + kk * 2048, G::AtomBytes, 1024), idO, (j > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&pvdone[t]);
      };
      ok = ok && mbar_wait(&kfull[0], 0, a.err, DEVERR_ATTN_FULL);
      tc_fence_after();
#pragma unroll
      for (int t = 0; t < kFaTiles; ++t)
        if (nb[t] > 0) issue_s(t, 0);
      umma_commit(&kempty[0]);
      for (int j = 0; j < nblk; ++j) {
        bool vin = false, kin = false;
#pragma unroll
        for (int t = 0; t < kFaTiles; ++t) {
          if (j >= nb[t]) continue;
          ok = ok && mbar_wait_poll(&pfull[t], (uint32_t)j & 1, a.err, DEVERR_ATTN_FULL);
          if (!vin) {
            ok = ok && mbar_wait(&vfull[j & 1], (uint32_t)(j >> 1) & 1, a.err, DEVERR_ATTN_FULL);
            vin = true;
          }
          tc_fence_after();
          issue_pv(t, j);
          if (j + 1 < nb[t]) {
            // a tile that sees block j + 1 sees block j: the first such tile waits for K_{j+1}
            if (!kin) {
              ok = ok && mbar_wait(&kfull[(j + 1) & 1], (uint32_t)((j + 1) >> 1) & 1, a.err, DEVERR_ATTN_FULL);
              kin = true;
            }
            // S_t of the next block overwrites P_t; issued after P_t V by this thread, the tensor core
            // runs it after P_t V has read P_t
            tc_fence_after();
            issue_s(t, j + 1);
          }
        }
        umma_commit(&vempty[j & 1]);
        if (j + 1 < nblk) umma_commit(&kempty[(j + 1) & 1]);
      }
    }
  } else if (lane == 0) {
    // ================= loader (last warp): K and V blocks, two slots each =================
    const uint64_t pol = l2_evict_last_policy();  // re-read by the other query tiles and GQA heads
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
    int kiss = 0, viss = 0;
    for (int j = 0; j < nblk; ++j) {
      const int sb = j & 1;
      if (j >= 2) ok = ok && mbar_wait(&kempty[sb], (uint32_t)((j >> 1) - 1) & 1, a.err, DEVERR_ATTN_EMPTY);
      if (ok) {
        mbar_arrive_expect_tx(&kfull[sb], (uint32_t)G::KVBytes);
        for (int u = 0; u < G::Atoms; ++u)
          tma_load_4d(ks + sb * G::KVBytes + u * G::AtomBytes, &tmk, 64 * u, j * kFaKeys, hk, b, &kfull[sb], pol);
        kiss = j + 1;
      } else {
        mbar_arrive(&kfull[sb]);
      }
      if (j >= 2) ok = ok && mbar_wait(&vempty[sb], (uint32_t)((j >> 1) - 1) & 1, a.err, DEVERR_ATTN_EMPTY);
      if (ok) {
        mbar_arrive_expect_tx(&vfull[sb], (uint32_t)G::KVBytes);
        for (int u = 0; u < G::Atoms; ++u)
          tma_load_4d(vs + sb * G::KVBytes + u * G::AtomBytes, &tmv, 64 * u, j * kFaKeys, hk, b, &vfull[sb], pol);
        viss = j + 1;
      } else {
        mbar_arrive(&vfull[sb]);
      }
    }
    // drain: no copy may still be landing in shared memory when the CTA exits
    for (int j = kiss > 2 ? kiss - 2 : 0; j < kiss; ++j) mbar_wait_drain(&kfull[j & 1], (uint32_t)(j >> 1) & 1);
    for (int j = viss > 2 ? viss - 2 : 0; j < viss; ++j) mbar_wait_drain(&vfull[j & 1], (uint32_t)(j >> 1) & 1);
  }
  __syncthreads();
  if (warp == kFaMmaWarp) {
    tc_fence_after();
    tmem_dealloc(taddr, kFaTmemCols);
  }
}

template <int D>
void launch_tc_d(const AttnArgs &a, cudaStream_t s) {
  using G = FaGeo<D>;
  // K/V [B][H_kv][capacity][D] fp16 with element strides kv_sb, kv_sh: boxes of [128 tokens][64 columns]
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)(a.kv_sh / D), (uint64_t)a.Hkv, (uint64_t)a.B};
  const uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)a.kv_sh * 2, (uint64_t)std::max<int64_t>(a.kv_sb, 1) * 2};
  const uint32_t box[4] = {64, kFaKeys, 1, 1};
  const CUtensorMap tmk =
      make_tmap_4d(a.k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tmv =
      make_tmap_4d(a.v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  static unsigned long long attr_set = 0;
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << dev))) {
    FG_CUDA(cudaFuncSetAttribute(k_attn_tc<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G::Smem));
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  // pairs of query tiles in the slowest grid dimension, so that the longest causal pairs start first
  cfg.gridDim = dim3((unsigned)a.H, (unsigned)a.B, (unsigned)ceil_div(ceil_div(a.Nq, kFaRows), kFaTiles));
  cfg.blockDim = dim3(kFaThreads);
  cfg.dynamicSmemBytes = G::Smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FG_CUDA(cudaLaunchKernelEx(&cfg, k_attn_tc<D>, tmk, tmv, a));
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

bool attn_tc_supported(const AttnArgs &a) {
  static const bool simt = [] {
    const char *e = std::getenv("FORGE_B200_ATTN");
    return e && std::string(e) == "simt";
  }();
  // a non-negative scale keeps the row maximum of the raw scores the maximum of the scaled ones
  if (simt || !a.kv_f16 || !(a.d == 64 || a.d == 128) || a.Hkv < 1 || a.H % a.Hkv != 0 || !(a.scale >= 0.f) ||
      a.B > 65535 || ceil_div(ceil_div(a.Nq, kFaRows), kFaTiles) > 65535)
    return false;
  const int qe = a.q_f16 ? 8 : 4;  // elements per 16 bytes
  return aligned16(a.q) && aligned16(a.k) && aligned16(a.v) && aligned16(a.o) && a.q_sb % qe == 0 &&
         a.q_sh % qe == 0 && a.q_si % qe == 0 && a.o_sb % 4 == 0 && a.o_sh % 4 == 0 && a.o_si % 4 == 0 &&
         a.kv_sh % 8 == 0 && a.kv_sb % 8 == 0 && a.kv_sh >= (int64_t)a.d && (a.B == 1 || a.kv_sb > 0);
}

void launch_attention_tc(const AttnArgs &a, cudaStream_t s) {
  FG_REQUIRE(attn_tc_supported(a), FG_ERR_SHAPE, "tensor-core attention: unsupported shape or layout");
  if (a.B == 0 || a.Nq == 0 || a.H == 0) return;
  if (a.d == 64)
    launch_tc_d<64>(a, s);
  else
    launch_tc_d<128>(a, s);
}

}  // namespace fg
