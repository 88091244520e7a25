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
#include "q4_gemv.cuh"
#include "tmap.cuh"

namespace fg {
namespace {

constexpr int kRows = 32;        // Q8_0 rows per row group (one TMA box high)
constexpr int kConsumers = 8;    // consumer warps (two CTAs share an SM)
constexpr int kCThreads = kConsumers * 32;
constexpr int kThreads = kCThreads + 32;  // + producer warp
constexpr int kTileBytes = 512;  // code bytes per row per chunk (one TMA box wide)
constexpr int kStages = 3;

// Q8_0 stage geometry: ROWS rows x TB code bytes (CB blocks) per TMA tile.
template <int ROWS, int TB, int CB>
struct Geo {
  static constexpr int SQ = ROWS * TB;            // code bytes per stage
  static constexpr int SB = SQ + ROWS * CB * 2;   // + scales
};

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

// ---------------------------------------------------------------------------
// Q4_0 tensor-core GEMV (q4_gemv.cuh): a CTA owns consecutive 16-row strips.
// ---------------------------------------------------------------------------
// Ring depth: 4 stages, or 3 where 4 would keep the x staging of a long K from fitting two CTAs per
// SM (108 KB in flight per SM still streams at full HBM speed).
template <int MV, int kQ4Stages>
__global__ void __launch_bounds__(kThreads, 2)
    k_qgemv_q4(QMat w, const float *__restrict__ x, int64_t ldx, const float *__restrict__ gamma, float eps, int do_norm,
               Epilogue ep, GemvScratch scr) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *ring = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
  __shared__ __align__(8) uint64_t full[kQ4Stages], empty[kQ4Stages];
  __shared__ float s_sum[kConsumers * MV];
  __shared__ float s_inv[MV];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = (int)(w.K >> 5), nq = (int)w.row_words;
  const Sched sc = make_sched(w.N, kQ4StripRows, 1, blockIdx.x, gridDim.x);  // units = strips
  Q4X<MV> X;
  X.carve(ring + kQ4Stages * kQ4TileBytes, nb, nq * 4);
  float *red = reinterpret_cast<float *>(ring + kQ4Stages * kQ4TileBytes + Q4X<MV>::bytes(X.nbx));  // [2][8][16][MV]

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
    if (lane == 0) {
      int i = 0;
      produce_q4_strips<kQ4Stages>(w, sc.u0, sc.u1, ring, full, empty, i, l2_evict_first_policy(), scr.err);
      drain_ring<kQ4Stages>(full, i, scr.err);
    }
    return;
  }

  // ---------------- stage x (after the producer of x has finished)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  q4_stage_x<MV>(X, x, ldx, do_norm ? gamma : nullptr, tid, kCThreads, s_sum);
  named_sync(kCThreads);
  if (tid < MV) s_inv[tid] = rms_inv(s_sum, kConsumers, MV, tid, w.K, eps, do_norm);

  // ---------------- consume
  Q4Lane<MV> L;
  L.init(X, lane);
  float2 acc[Q4X<MV>::NM];
#pragma unroll
  for (int im = 0; im < Q4X<MV>::NM; ++im) acc[im] = make_float2(0.0f, 0.0f);
  bool ok = true;
  int i = 0;
  for (int u = sc.u0; u < sc.u1; ++u) {
    for (int q0 = 0; q0 < nq; q0 += kQ4TileQuads, ++i) {
      const int s = i % kQ4Stages;
      ok = ok && mbar_wait(&full[s], (uint32_t)(i / kQ4Stages) & 1, scr.err, DEVERR_GEMV_FULL);
      if (ok) q4_tile<MV>(ring + s * kQ4TileBytes, q0, min(kQ4TileQuads, nq - q0), warp, L, acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // two partial buffers in turn: a warp refills this one two strips later, after the next strip's
    // barrier, which the finishing threads reach only once they have read it
    float *rb = red + ((u - sc.u0) & 1) * (kGroupWarps * kQ4StripRows * MV);
    q4_group_red<MV>(rb, acc, warp, lane);
    named_sync(kCThreads);
    if (ok) finish_strip<MV>(w, ep, u, rb, s_inv, tid, kCThreads);
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
  const Sched sc = make_sched(w.N, kRows, (nb + CB - 1) / CB, blockIdx.x, gridDim.x);
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
      finish_group<kRows, MV>(w, ep, scr, sc, g, red, nullptr, &s_last, ok, tid, kCThreads, 1);
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
size_t q4_smem(int64_t K, int MV, int stages = 4) {
  const int nbx = (int)q4_quads(K) * 4;
  size_t xbytes = 0;
  switch (MV) {
    case 1: xbytes = Q4X<1>::bytes(nbx); break;
    case 2: xbytes = Q4X<2>::bytes(nbx); break;
    case 3: xbytes = Q4X<3>::bytes(nbx); break;
    default: xbytes = Q4X<4>::bytes(nbx); break;
  }
  return 128 + (size_t)stages * kQ4TileBytes + xbytes + (size_t)2 * kGroupWarps * kQ4StripRows * MV * 4;
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
  const int CB = 16, ROWS = kRows, TB = kTileBytes;  // Q8_0 tiles
  // units: Q4_0 16-row strips; Q8_0 (32-row group, 16-block chunk) pairs
  const int64_t nb = w.K / 32, nc = q4 ? 1 : ceil_div(nb, CB), G = q4 ? q4_strips(w.N) : ceil_div(w.N, ROWS);
  const int64_t U = G * nc;
  FG_REQUIRE(U < (1ll << 31), FG_ERR_SHAPE, "gemv: matrix too large");
  // Q4_0: a 3-stage ring where only that keeps two CTAs per SM
  const int stages = q4 && q4_smem(w.K, MV, 4) > kSmemTwo && q4_smem(w.K, MV, 3) <= kSmemTwo ? 3 : 4;
  const size_t smem = q4 ? q4_smem(w.K, MV, stages) : q8_smem(w.K, MV);
  const int P = (int)std::min<int64_t>((smem <= kSmemTwo ? 2LL : 1LL) * num_sms, U);
  GemvScratch scx = sc;
  if (!q4) {  // stream-K fix-up slots of the Q8_0 kernel
    int maxc = 1;
    for (int64_t g = 0; g < G; ++g)
      maxc = std::max(maxc, cta_of((int)(g * nc + nc - 1), (int)U, P) - cta_of((int)(g * nc), (int)U, P) + 1);
    FG_REQUIRE((uint64_t)G * maxc * ROWS * MV <= sc.part_floats && G <= sc.n_tickets, FG_ERR_SHAPE,
               "gemv: workspace too small for N=%lld K=%lld", (long long)w.N, (long long)w.K);
    scx.maxc = maxc;
  }
  static unsigned long long attr_set[3] = {0, 0, 0};  // per instantiation, one bit per device
  const int inst = q4 ? (stages == 3 ? 2 : 1) : 0;
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set[inst] & (1ull << dev))) {
    if (inst == 1)
      FG_CUDA(cudaFuncSetAttribute(k_qgemv_q4<MV, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOne));
    else if (inst == 2)
      FG_CUDA(cudaFuncSetAttribute(k_qgemv_q4<MV, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOne));
    else
      FG_CUDA(cudaFuncSetAttribute(k_qgemv_q8<MV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOne));
    attr_set[inst] |= 1ull << dev;
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
    if (stages == 3)
      FG_CUDA(cudaLaunchKernelEx(&cfg, k_qgemv_q4<MV, 3>, w, x, ldx, gamma, eps, do_norm ? 1 : 0, ep, scx));
    else
      FG_CUDA(cudaLaunchKernelEx(&cfg, k_qgemv_q4<MV, 4>, w, x, ldx, gamma, eps, do_norm ? 1 : 0, ep, scx));
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
