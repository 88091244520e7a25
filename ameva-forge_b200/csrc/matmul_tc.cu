// fp32 matmul on the 5th-generation tensor cores (tcgen05, sm_100a):
//   C[M, N] = A[M, K] B,  B given as [K, N] row-major (the reference's matmul /
//   matmul_tiled, packages/forge/src/tensor/kernels/matmul_tiled.wgsl.ts:13-86)
//   or as [N, K] (nn.Linear's W under the graph's transpose fold, forge-py
//   nn.py:248-259),
// with fp32-level accuracy from tf32 operands by a three-term split:
//   A = Ah + Al, B = Bh + Bl, where Ah, Bh are the fp32 values with the low 13
//   mantissa bits cleared (exact in tf32) and Al, Bl the exact fp32
//   remainders; A B ~ Ah Bh + Ah Bl + Al Bh.  The dropped Al Bl term and the
//   tf32 reading of Al, Bl are ~2^-20 relative, below the reference suite's
//   atol 1e-4 at its shapes (matmul_tiled.test.ts:146-212).
//
//  * k_tf32_split writes Ah, Al [M][Kp] and Bh, Bl [N][Kp] (K-major, zero for
//    k >= K, Kp = K rounded up to 32 columns), transposing a row-major B
//    through a shared tile, so the GEMM reads every operand with 2-D TMA boxes
//    of [rows][32] fp32: 128-byte rows with the 128-byte swizzle;
//  * k_matmul_tc: a CTA owns a 128 x kMmN tile of C.  K advances 32 columns per
//    stage through a ring of kMmStages stages (Ah, Al, Bh, Bl boxes); one thread
//    issues 3 x 4 tcgen05.mma.kind::tf32 (K = 8 each) per stage into a TMEM
//    accumulator (128 lanes x kMmN fp32 columns) and commits each stage to its
//    "empty" barrier; warps 0-3 read the accumulator with tcgen05.ld and store
//    C with bounds checks.
// Every wait is bounded (tma.cuh); on a timeout the device error word is set,
// the CTA skips its stores, drains its copies and frees its TMEM.
#include <cstdlib>
#include <cstring>

#include "runtime.cuh"
#include "tcgen05.cuh"
#include "tmap.cuh"

namespace fg {
namespace {

constexpr int kMmM = 128;      // UMMA M: rows of C per CTA (TMEM lanes)
constexpr int kMmN = 128;      // UMMA N: columns of C per CTA
constexpr int kMmK = 32;       // K per stage: one 128-byte swizzle row of fp32
constexpr int kMmStages = 3;
constexpr int kMmThreads = 6 * 32;  // warps 0-3 epilogue, warp 4 loads, warp 5 issues the MMAs
constexpr int kMmTileA = kMmM * kMmK * 4;  // 16 KB
constexpr int kMmTileB = kMmN * kMmK * 4;  // 16 KB
constexpr int kMmStage = 2 * kMmTileA + 2 * kMmTileB;
constexpr size_t kMmSmem = 1024 + (size_t)kMmStages * kMmStage;
static_assert(kMmSmem + 256 <= 232448, "shared memory per CTA");

// Instruction descriptor of kind::tf32: tf32 A and B, fp32 D, both K-major, shape M x N.
constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void split_tf32(float v, float &hi, float &lo) {
  if (isfinite(v)) {
    hi = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    lo = v - hi;  // exact: the cleared bits
  } else {
    hi = v;
    lo = 0.0f;
  }
}

// src [rows][K] (trans = false) or [K][rows] (trans = true) -> hi, lo [rows][Kp], zero for k >= K.
// 32 x 32 tiles through shared memory so both the read and the write are coalesced.
__global__ void __launch_bounds__(256) k_tf32_split(const float *__restrict__ src, int64_t rows, int64_t K, int trans,
                                                    int64_t Kp, float *__restrict__ hi, float *__restrict__ lo) {
  __shared__ float tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, k0 = (int64_t)blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int j = ty; j < 32; j += 8) {
    float v = 0.0f;
    if (trans) {  // row k0 + j of src, column r0 + tx
      const int64_t k = k0 + j, r = r0 + tx;
      if (k < K && r < rows) v = src[k * rows + r];
      tile[tx][j] = v;  // tile[r][k]
    } else {
      const int64_t r = r0 + j, k = k0 + tx;
      if (k < K && r < rows) v = src[r * K + k];
      tile[j][tx] = v;
    }
  }
  __syncthreads();
  for (int j = ty; j < 32; j += 8) {
    const int64_t r = r0 + j, k = k0 + tx;
    if (r < rows && k < Kp) {
      float h, l;
      split_tf32(tile[j][tx], h, l);
      hi[r * Kp + k] = h;
      lo[r * Kp + k] = l;
    }
  }
}

__global__ void __launch_bounds__(kMmThreads, 1)
    k_matmul_tc(const __grid_constant__ CUtensorMap tah, const __grid_constant__ CUtensorMap tal,
                const __grid_constant__ CUtensorMap tbh, const __grid_constant__ CUtensorMap tbl, float *__restrict__ C,
                int M, int N, int nk, int *err) {
  extern __shared__ __align__(1024) unsigned char mm_smem_raw[];
  unsigned char *sm = mm_smem_raw + ((1024 - (smem_u32(mm_smem_raw) & 1023)) & 1023);
  __shared__ __align__(8) uint64_t full[kMmStages], empty[kMmStages], accum;
  __shared__ uint32_t s_taddr;
  __shared__ int s_ok;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.y * kMmM, n0 = blockIdx.x * kMmN;

  if (tid == 0) {
    for (int s = 0; s < kMmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accum, 1);
    s_ok = 1;
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(&s_taddr, kMmN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = s_taddr;
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 4) {
    // ---------------- loads: Ah, Al (rows m0..), Bh, Bl (rows n0..) of K columns [32 t, 32 t + 32)
    if (lane == 0) {
      tma_prefetch_desc(&tah);
      tma_prefetch_desc(&tal);
      tma_prefetch_desc(&tbh);
      tma_prefetch_desc(&tbl);
      const uint64_t pol = l2_evict_last_policy();  // every tile is read by the other CTAs of its row / column
      int t = 0;
      for (; t < nk; ++t) {
        const int s = t % kMmStages;
        if (t >= kMmStages && !mbar_wait(&empty[s], (uint32_t)(t / kMmStages - 1) & 1, err, DEVERR_GEMV_EMPTY)) {
          s_ok = 0;
          break;
        }
        unsigned char *st = sm + (size_t)s * kMmStage;
        mbar_arrive_expect_tx(&full[s], (uint32_t)kMmStage);
        tma_load_2d(st, &tah, t * kMmK, m0, &full[s], pol);
        tma_load_2d(st + kMmTileA, &tal, t * kMmK, m0, &full[s], pol);
        tma_load_2d(st + 2 * kMmTileA, &tbh, t * kMmK, n0, &full[s], pol);
        tma_load_2d(st + 2 * kMmTileA + kMmTileB, &tbl, t * kMmK, n0, &full[s], pol);
      }
      // no copy may still be landing when the CTA exits
      for (int j = t > kMmStages ? t - kMmStages : 0; j < t; ++j)
        mbar_wait(&full[j % kMmStages], (uint32_t)(j / kMmStages) & 1, err, DEVERR_DRAIN);
    }
  } else if (warp == 5) {
    // ---------------- MMA issue: Ah Bh + Ah Bl + Al Bh, K = 8 per instruction
    if (lane == 0) {
      constexpr uint32_t id = idesc_tf32(kMmM, kMmN);
      bool ok = true;
      for (int t = 0; t < nk; ++t) {
        const int s = t % kMmStages;
        ok = ok && mbar_wait(&full[s], (uint32_t)(t / kMmStages) & 1, err, DEVERR_GEMV_FULL);
        tc_fence_after();
        if (ok) {
          const uint32_t a_h = smem_u32(sm + (size_t)s * kMmStage), a_l = a_h + kMmTileA;
          const uint32_t b_h = a_h + 2 * kMmTileA, b_l = b_h + kMmTileB;
#pragma unroll
          for (int kk = 0; kk < kMmK / 8; ++kk) {
            const uint32_t off = 32 * kk;  // 8 tf32 = 32 bytes along the swizzled 128-byte row
            umma_tf32(taddr, smem_desc_sw128(a_h + off), smem_desc_sw128(b_h + off), id, (t > 0 || kk > 0) ? 1u : 0u);
            umma_tf32(taddr, smem_desc_sw128(a_h + off), smem_desc_sw128(b_l + off), id, 1u);
            umma_tf32(taddr, smem_desc_sw128(a_l + off), smem_desc_sw128(b_h + off), id, 1u);
          }
        }
        umma_commit(&empty[s]);
      }
      if (!ok) s_ok = 0;
      umma_commit(&accum);
    }
  } else {
    // ---------------- epilogue: warp w reads TMEM lanes 32 w .. 32 w + 31 = rows m0 + 32 w + lane
    const bool ok = mbar_wait(&accum, 0, err, DEVERR_GEMV_FULL);
    __syncwarp();
    tc_fence_after();
    const int r = m0 + 32 * warp + lane;
    const uint32_t trow = taddr + ((uint32_t)(32 * warp) << 16);
    const bool vec = (N & 3) == 0;
#pragma unroll 1
    for (int c0 = 0; c0 < kMmN; c0 += 32) {
      float v[32];
      tmem_ld32(trow + c0, v);
      if (!ok || !s_ok || r >= M || n0 + c0 >= N) continue;
      float *crow = C + (int64_t)r * N + n0 + c0;
      if (vec && n0 + c0 + 32 <= N) {
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4 *>(crow + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (n0 + c0 + e < N) crow[e] = v[e];
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(taddr, kMmN);
  }
}

// Operand of the GEMM: hi / lo [rows][Kp] fp32.
CUtensorMap split_map(const float *p, int64_t rows, int64_t Kp, int box_rows) {
  return make_tmap_2d(p, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)rows, (uint64_t)Kp, (uint64_t)Kp * 4,
                      (uint32_t)box_rows, kMmK, CU_TENSOR_MAP_SWIZZLE_128B);
}

void launch_split(const float *src, int64_t rows, int64_t K, bool trans, int64_t Kp, float *hi, float *lo,
                  cudaStream_t s) {
  dim3 grid((unsigned)ceil_div(Kp, 32), (unsigned)ceil_div(rows, 32));
  k_tf32_split<<<grid, 256, 0, s>>>(src, rows, K, trans ? 1 : 0, Kp, hi, lo);
  FG_LAUNCH_CHECK();
}

}  // namespace

uint64_t matmul_tc_scratch_bytes(int64_t M, int64_t K, int64_t N) {
  const int64_t Kp = align_up((uint64_t)std::max<int64_t>(K, 1), kMmK);
  return 2 * align_up((uint64_t)(M * Kp * 4), 256) + 2 * align_up((uint64_t)(N * Kp * 4), 256);
}

void launch_matmul_tc(const float *A, const float *B, float *C, int64_t M, int64_t K, int64_t N, bool b_trans,
                      void *scratch, int *err, cudaStream_t s) {
  if (M == 0 || N == 0) return;
  FG_REQUIRE(M <= INT32_MAX && N <= INT32_MAX, FG_ERR_SHAPE, "matmul: dimensions above 2^31");
  const int64_t Kp = align_up((uint64_t)std::max<int64_t>(K, 1), kMmK);
  unsigned char *p = (unsigned char *)scratch;
  float *ah = (float *)p;
  float *al = (float *)(p += align_up((uint64_t)(M * Kp * 4), 256));
  float *bh = (float *)(p += align_up((uint64_t)(M * Kp * 4), 256));
  float *bl = (float *)(p += align_up((uint64_t)(N * Kp * 4), 256));
  launch_split(A, M, K, false, Kp, ah, al, s);
  launch_split(B, N, K, !b_trans, Kp, bh, bl, s);  // B [K, N] is transposed into [N][Kp]
  const CUtensorMap tah = split_map(ah, M, Kp, kMmM), tal = split_map(al, M, Kp, kMmM);
  const CUtensorMap tbh = split_map(bh, N, Kp, kMmN), tbl = split_map(bl, N, Kp, kMmN);
  static unsigned long long attr_set = 0;
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << dev))) {
    FG_CUDA(cudaFuncSetAttribute(k_matmul_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMmSmem));
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ceil_div(N, kMmN), (unsigned)ceil_div(M, kMmM));
  cfg.blockDim = dim3(kMmThreads);
  cfg.dynamicSmemBytes = kMmSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FG_CUDA(cudaLaunchKernelEx(&cfg, k_matmul_tc, tah, tal, tbh, tbl, C, (int)M, (int)N, (int)(Kp / kMmK), err));
}

// The tensor-core path for products of at least 2^20 multiply-adds (smaller ones are launch-bound and
// keep the SIMT kernel); FORGE_B200_MATMUL=tc / simt forces one path.
bool matmul_use_tc(int64_t M, int64_t K, int64_t N) {
  const char *force = std::getenv("FORGE_B200_MATMUL");
  if (force && !std::strcmp(force, "tc")) return M > 0 && N > 0;
  if (force && !std::strcmp(force, "simt")) return false;
  return M > 0 && N > 0 && K > 0 && (double)M * (double)N * (double)K >= 1048576.0;
}

void launch_matmul(Ctx &c, const float *A, const float *B, float *C, int64_t M, int64_t K, int64_t N, bool b_trans) {
  if (!matmul_use_tc(M, K, N)) {
    launch_matmul_f32(A, B, C, M, K, N, c.stream, b_trans);
    return;
  }
  const uint64_t bytes = matmul_tc_scratch_bytes(M, K, N);
  void *scratch = c.alloc(bytes);
  try {
    launch_matmul_tc(A, B, C, M, K, N, b_trans, scratch, c.gemv.err, c.stream);
  } catch (...) {
    c.free_async(scratch, bytes);
    throw;
  }
  c.free_async(scratch, bytes);
}

}  // namespace fg
