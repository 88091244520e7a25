// Flash attention on the 5th-generation tensor cores (tcgen05, sm_100a) for
// fp16 K/V (fp32 or fp16 Q) and head_dim 64 or 128, with the reference
// semantics (packages/forge/src/tensor/kernels/flash_attention.wgsl.ts:13-178):
//   GQA kv_head = h / (H / H_kv); causal: key j visible iff
//   j < N_kv - N_q + i + 1; running max starts at -1e30; out = acc / max(l, 1e-12).
//
// A CTA owns 128 query rows of one (batch, head) and walks the visible keys in
// blocks of 128:
//  * a loader thread brings K and V blocks into two-slot rings with 4-D TMA
//    boxes [128 keys][64 head columns] (128-byte swizzle, rows past the cache
//    extent read as zero);
//  * one thread of the MMA warp issues S = Q K^T (M = 128 queries, N = 128
//    keys, K = head_dim) into one of two TMEM score buffers, so the tensor
//    core computes block j + 1's scores while block j is in softmax, and
//    O += P V (N = head_dim, K = 128 keys, V read MN-major) into a TMEM
//    accumulator;
//  * eight softmax warps own the TMEM lanes = query rows, two warps per
//    32-lane quadrant, each taking 64 of the block's 128 keys (both read the
//    whole row for its maximum, so they agree on m without exchanging it):
//    they read S
//    (tcgen05.ld), apply the scale and the causal/extent mask, update the
//    running max m and sum l (exp2 domain), and write P as fp16 into one of
//    two swizzled shared tiles.  m moves only when a row's maximum grows by
//    more than 2^8 (P then stays <= 256, exact in fp16 range); only then is
//    the O row rescaled in TMEM, so most blocks need no O round trip and the
//    softmax of block j overlaps P V of block j - 1;
//  * the same warps finish with out = O / max(l, 1e-12) in fp32, each warp of
//    a pair storing half of the head columns.
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

constexpr int kFaRows = 128;  // queries per CTA: UMMA M, TMEM lanes
constexpr int kFaKeys = 128;  // keys per block: N of S = Q K^T, K of O += P V
constexpr int kFaSoftmaxWarps = 8;
constexpr int kFaMmaWarp = 9;  // warp 8 loads K/V
constexpr int kFaThreads = 10 * 32;
constexpr int kFaTmemCols = 512;  // S0 [0, 128), S1 [128, 256), O [256, 256 + head_dim)
constexpr int kFaOCol = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazy = 8.f;  // log2 of the largest P before the reference max moves

template <int D>
struct FaGeo {
  static constexpr int Atoms = D / 64;                  // 64-column swizzle atoms along head_dim
  static constexpr int AtomBytes = 128 * 128;           // [128 rows][64] fp16
  static constexpr int QBytes = Atoms * AtomBytes;      // Q tile, K-major
  static constexpr int KVBytes = Atoms * AtomBytes;     // one K or V block
  static constexpr int PTile = 2 * AtomBytes;           // P tile [2 atoms of 64 keys][128 rows][64]
  static constexpr int PBytes = 2 * PTile;              // two P tiles
  static constexpr size_t KOff = QBytes, VOff = KOff + 2 * (size_t)KVBytes, POff = VOff + 2 * (size_t)KVBytes;
  // + 1 KB for the 1024-byte alignment; at least 120 KB, so that one CTA
  // holds an SM (it allocates 512 TMEM columns)
  static constexpr size_t Need = 1024 + POff + PBytes;
  static constexpr size_t Smem = Need > 122880 ? Need : 122880;
  static_assert(Smem + 512 <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

template <int D>
__global__ void __launch_bounds__(kFaThreads, 1)
    k_attn_tc(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, AttnArgs a) {
  using G = FaGeo<D>;
  extern __shared__ __align__(1024) unsigned char fa_smem_raw[];
  unsigned char *sm = fa_smem_raw + ((1024 - (smem_u32(fa_smem_raw) & 1023)) & 1023);
  unsigned char *qs = sm, *ks = sm + G::KOff, *vs = sm + G::VOff, *ps = sm + G::POff;
  __shared__ __align__(8) uint64_t kfull[2], kempty[2], vfull[2], vempty[2], sfull[2], pvdone[2], pfull, qready;
  __shared__ uint32_t s_taddr;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qb = gridDim.x - 1 - blockIdx.x;  // the longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z, hk = h / (a.H / a.Hkv);
  const int i0 = qb * kFaRows;

  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int nkv = a.n_kv_dev ? a.n_kv_dev[b] + a.n_kv_add : a.n_kv;
  int kend = nkv;  // keys any row of the block can see
  if (a.causal) kend = min(kend, nkv - a.Nq + i0 + kFaRows);
  const int nblk = kend > 0 ? (kend + kFaKeys - 1) / kFaKeys : 0;

  if (nblk == 0) {  // no row of the block sees a key: acc = 0, l = 0, out = 0
    if (tid < kFaRows && i0 + tid < a.Nq) {
      float *o = a.o + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + (int64_t)(i0 + tid) * a.o_si;
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
      mbar_init(&sfull[s], 1);
      mbar_init(&pvdone[s], 1);  // P V of the blocks using P tile s
    }
    mbar_init(&pfull, kFaSoftmaxWarps);
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
    // ================= softmax warps: thread = query row = TMEM lane, warp half hh of the keys =========
    const int quad = warp & 3, hh = warp >> 2, r = 32 * quad + lane, qi = i0 + r;
    {  // this row's half of Q, fp16, into the K-major swizzled tile (row r at r * 128, chunk c at c ^ (r & 7))
      const int64_t qoff = (int64_t)b * a.q_sb + (int64_t)h * a.q_sh + (int64_t)qi * a.q_si;
#pragma unroll 4
      for (int c = hh * (D / 16); c < (hh + 1) * (D / 16); ++c) {  // 16-byte chunk c: head columns 8c .. 8c+7
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (qi < a.Nq) {
          if (a.q_f16) {
            v = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __half *>(a.q) + qoff + 8 * c);
          } else {
            const float *qf = reinterpret_cast<const float *>(a.q) + qoff + 8 * c;
            const float4 x0 = *reinterpret_cast<const float4 *>(qf), x1 = *reinterpret_cast<const float4 *>(qf + 4);
            v = make_uint4(pack_f16x2(x0.x, x0.y), pack_f16x2(x0.z, x0.w), pack_f16x2(x1.x, x1.y),
                           pack_f16x2(x1.z, x1.w));
          }
        }
        *reinterpret_cast<uint4 *>(qs + (c >> 3) * G::AtomBytes + r * 128 + (((c & 7) ^ (r & 7)) * 16)) = v;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&qready);

    const float sl2 = a.scale * kLog2e;  // scores in log2 units
    const int lim = a.causal ? min(nkv - a.Nq + qi + 1, nkv) : nkv;  // keys [0, lim) visible to this row
    float m = -1e30f * kLog2e, l = 0.f;  // l: this warp's half of the row sum
    const uint32_t trow = taddr + ((uint32_t)(32 * quad) << 16), to = trow + kFaOCol + hh * (D / 2);
    for (int j = 0; j < nblk; ++j) {
      const int sb = j & 1, kh = j * kFaKeys + hh * 64;  // first key of this warp's half
      ok = ok && mbar_wait(&sfull[sb], (uint32_t)(j >> 1) & 1, a.err, DEVERR_ATTN_FULL);
      __syncwarp();
      tc_fence_after();
      const uint32_t ts = trow + sb * kFaKeys + hh * 64;
      const bool masked = kh + 64 > lim;
      const int ko = j * kFaKeys + (hh ^ 1) * 64;  // first key of the partner warp's half
      // the whole row in one go (own half kept for the exponentials), one wait
      uint32_t s0[32], s1[32], x0[32], x1[32];
      tmem_ld32_issue(ts, s0);
      tmem_ld32_issue(ts + 32, s1);
      tmem_ld32_issue(ts + (hh ? -64 : 64), x0);
      tmem_ld32_issue(ts + (hh ? -32 : 96), x1);
      tmem_ld_wait(s0);
      tmem_ld_wait(s1);
      tmem_ld_wait(x0);
      tmem_ld_wait(x1);
      float v[64];  // this warp's 64 scores; masked keys read as -inf (ex2(-inf) = 0)
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        v[e] = __uint_as_float(s0[e]);
        v[32 + e] = __uint_as_float(s1[e]);
      }
      if (masked) {
#pragma unroll
        for (int e = 0; e < 64; ++e)
          if (kh + e >= lim) v[e] = -INFINITY;
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < 64; ++e) mx4[e & 3] = fmaxf(mx4[e & 3], v[e]);  // four independent chains
      const bool xmasked = ko + 64 > lim;
#pragma unroll
      for (int e = 0; e < 32; ++e) {  // the partner's half: for the maximum only
        const float y0 = (xmasked && ko + e >= lim) ? -INFINITY : __uint_as_float(x0[e]);
        const float y1 = (xmasked && ko + 32 + e >= lim) ? -INFINITY : __uint_as_float(x1[e]);
        mx4[e & 3] = fmaxf(mx4[e & 3], fmaxf(y0, y1));
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      // the reference max moves only when this row's maximum grew by more than kLazy
      const float mc = fmaxf(m, mx * sl2);
      const bool grow = mc - m > kLazy;
      const bool rescale = __any_sync(0xffffffffu, grow && j > 0);  // same rows, same decision in both warps
      float alpha = 1.f;
      if (grow) {
        alpha = ex2(m - mc);
        m = mc;
      }
      const int pb = j & 1;
      if (j >= 2) {  // P tile pb is free once P V of block j - 2 has completed
        ok = ok && mbar_wait(&pvdone[pb], (uint32_t)((j >> 1) - 1) & 1, a.err, DEVERR_ATTN_EMPTY);
        __syncwarp();
      }
      float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 sl2x2 = make_float2(sl2, sl2), negm = make_float2(-m, -m);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 x = ffma2(make_float2(v[32 * c + e], v[32 * c + e + 1]), sl2x2, negm);
          const float2 p = make_float2(ex2(x.x), ex2(x.y));
          sum2[(e >> 1) & 1] = fadd2(sum2[(e >> 1) & 1], p);
          pk[e >> 1] = pack_f16x2(p.x, p.y);
        }
        // keys 64 hh + 32c .. +31 of the row: atom hh, 16-byte chunks 4c .. 4c+3
        unsigned char *prow = ps + pb * G::PTile + hh * G::AtomBytes + r * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int cc = 4 * c + q;
          *reinterpret_cast<uint4 *>(prow + ((cc ^ (r & 7)) * 16)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      if (rescale) {  // O *= alpha (this warp's half of the columns) once P V of block j - 1 is in
        ok = ok && mbar_wait(&pvdone[pb ^ 1], (uint32_t)((j - 1) >> 1) & 1, a.err, DEVERR_ATTN_EMPTY);
        __syncwarp();
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          float o[32];
          tmem_ld32(to + 32 * c, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= alpha;
          tmem_st32(to + 32 * c, o);
        }
      }
      fence_proxy_async_smem();  // P is read by the tensor core through the async proxy
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull);
      l = l * alpha + ((sum2[0].x + sum2[0].y) + (sum2[1].x + sum2[1].y));
    }
    ok = ok && mbar_wait(&pvdone[(nblk - 1) & 1], (uint32_t)((nblk - 1) >> 1) & 1, a.err, DEVERR_ATTN_FULL);
    __syncwarp();
    tc_fence_after();
    // row sum = the two halves; the Q tile is free once the last MMA has completed
    float *xsum = reinterpret_cast<float *>(qs);
    xsum[hh * kFaRows + r] = l;
    named_sync_id(1 + quad, 64);
    l += xsum[(hh ^ 1) * kFaRows + r];
    const float inv = 1.f / fmaxf(l, 1e-12f);
    float *orow = a.o + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + (int64_t)qi * a.o_si + hh * (D / 2);
#pragma unroll 1
    for (int c = 0; c < D / 64; ++c) {
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
  } else if (warp == kFaMmaWarp) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16_f32acc(kFaRows, kFaKeys, false);
      constexpr uint32_t idO = idesc_f16_f32acc(kFaRows, D, true);
      const uint32_t qa = smem_u32(qs), pa = smem_u32(ps);
      ok = ok && mbar_wait(&qready, 0, a.err, DEVERR_ATTN_FULL);
      auto issue_s = [&](int j) {  // S[j % 2] = Q K_j^T, K = 16 head columns per MMA
        const int sb = j & 1;
        ok = ok && mbar_wait(&kfull[sb], (uint32_t)(j >> 1) & 1, a.err, DEVERR_ATTN_FULL);
        tc_fence_after();
        const uint32_t ka = smem_u32(ks + sb * G::KVBytes);
        if (ok) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * G::AtomBytes + 32 * (kk & 3);
            umma_f16(taddr + sb * kFaKeys, smem_desc_sw128(qa + off), smem_desc_sw128(ka + off), idS,
                     kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(&sfull[sb]);
        umma_commit(&kempty[sb]);
      };
      issue_s(0);
      if (nblk > 1) issue_s(1);
      for (int j = 0; j < nblk; ++j) {
        const int sb = j & 1;
        ok = ok && mbar_wait(&pfull, (uint32_t)j & 1, a.err, DEVERR_ATTN_FULL);
        ok = ok && mbar_wait(&vfull[sb], (uint32_t)(j >> 1) & 1, a.err, DEVERR_ATTN_FULL);
        tc_fence_after();
        const uint32_t va = smem_u32(vs + sb * G::KVBytes);
        if (ok) {
#pragma unroll
          for (int kk = 0; kk < kFaKeys / 16; ++kk) {  // K = 16 keys per MMA
            const uint64_t dp = smem_desc_sw128(pa + (j & 1) * G::PTile + (kk >> 2) * G::AtomBytes + 32 * (kk & 3));
            // V block [atom of 64 head columns][128 keys][64], MN-major: 16 keys = 2048 bytes
            // per step, 8-key atoms 1024 bytes apart, the next 64 head columns one atom further
            const uint64_t dv = smem_desc_sw128(va + kk * 2048, G::AtomBytes, 1024);
            umma_f16(taddr + kFaOCol, dp, dv, idO, (j > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&pvdone[j & 1]);
        umma_commit(&vempty[sb]);
        if (j + 2 < nblk) issue_s(j + 2);  // the softmax has finished reading S[j % 2]
      }
    }
  } else if (lane == 0) {
    // ================= loader (warp 8): K and V blocks, two slots each =================
    const uint64_t pol = l2_evict_last_policy();  // re-read by the other query blocks and GQA heads
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
    int kiss = 0, viss = 0;
    for (int j = 0; j < nblk; ++j) {
      const int sb = j & 1;
      if (j >= 2) ok = ok && mbar_wait(&kempty[sb], (uint32_t)((j >> 1) - 1) & 1, a.err, DEVERR_ATTN_EMPTY);
      if (ok) {
        mbar_arrive_expect_tx(&kfull[sb], (uint32_t)G::KVBytes);
        for (int t = 0; t < G::Atoms; ++t)
          tma_load_4d(ks + sb * G::KVBytes + t * G::AtomBytes, &tmk, 64 * t, j * kFaKeys, hk, b, &kfull[sb], pol);
        kiss = j + 1;
      } else {
        mbar_arrive(&kfull[sb]);
      }
      if (j >= 2) ok = ok && mbar_wait(&vempty[sb], (uint32_t)((j >> 1) - 1) & 1, a.err, DEVERR_ATTN_EMPTY);
      if (ok) {
        mbar_arrive_expect_tx(&vfull[sb], (uint32_t)G::KVBytes);
        for (int t = 0; t < G::Atoms; ++t)
          tma_load_4d(vs + sb * G::KVBytes + t * G::AtomBytes, &tmv, 64 * t, j * kFaKeys, hk, b, &vfull[sb], pol);
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
  cfg.gridDim = dim3((unsigned)ceil_div(a.Nq, kFaRows), (unsigned)a.H, (unsigned)a.B);
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
  if (simt || !a.kv_f16 || !(a.d == 64 || a.d == 128) || a.Hkv < 1 || a.H % a.Hkv != 0) return false;
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
