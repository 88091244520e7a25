// Q4_0 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a):
//   Y[m, n] = sum_k X[m, k] W[n, k]   (+ the fused epilogues of epilogue.cuh)
// for more than 4 token rows (prefill chunks, batched decode).
//
// The weight matrix is the UMMA A operand: a CTA owns 128 weight rows (8 of
// the 16-row strips of the Q4_0 layout, common.cuh) and NT tokens (16..256,
// the UMMA N), so D = W_tile X_tile^T sits in TMEM as 128 lanes x NT fp32
// columns.  Per 64-wide K step:
//  * 8 producer warps write the stage in the canonical K-major, 128-byte
//    swizzled layout (row r at r * 128 bytes, 16-byte chunk c at c ^ (r & 7);
//    8-row atoms 1024 bytes apart): warps 0-3 dequantise the Q4_0 codes of
//    two blocks per row, (q - 8) * d in one rounding (the fp16 pair 1024 + q,
//    one exact add, one multiply); warps 4-7 convert X to fp16.  Both operands
//    are fp16: a Q4_0 weight (q - 8) * d carries 15 significant bits, which
//    fp16 keeps to 2^-12 (bf16 would lose 2^-9 and sit at the GEMM tolerance);
//  * one thread of warp 8 issues four tcgen05.mma.kind::f16 (K = 16 each)
//    with shared-memory descriptors and commits them to the stage's "empty"
//    mbarrier, so the producers refill the stage once the tensor core has
//    read it; after the last step it commits to the "accumulator" mbarrier;
//  * warps 0-3 (TMEM lanes 0..127) read D with tcgen05.ld and run the
//    epilogue on row pairs (RoPE / SwiGLU partners are neighbouring lanes).
// When the (weight tile, token tile) grid is smaller than the GPU, K is split
// over several CTAs: each writes its partial tile and the last one of a tile
// to arrive sums them in split order (deterministic) and runs the epilogue.
//
// Every wait is bounded (tma.cuh): on a timeout the device error word is set,
// the CTA skips the remaining work, still frees its TMEM and returns.
#include "q4_gemv.cuh"

namespace fg {
namespace {

constexpr int kTcRows = 128;                 // UMMA M: weight rows per CTA
constexpr int kTcK = 64;                     // K per stage (one 128-byte swizzle atom of fp16)
constexpr int kTcStages = 4;
constexpr int kTcProducerWarps = 8;
constexpr int kTcThreads = (kTcProducerWarps + 1) * 32;
constexpr int kTcABytes = kTcRows * kTcK * 2;  // 16 KB per stage

template <int NT>
struct TcGeo {
  static constexpr int BBytes = NT * kTcK * 2;
  static constexpr int Stage = kTcABytes + BBytes;
  static constexpr int TmemCols = NT < 32 ? 32 : NT;  // allocation: a power of two >= 32
  static constexpr size_t Smem = 1024 + (size_t)kTcStages * Stage;  // + 1 KB for the 1024-byte alignment
};

// ---- tcgen05 / UMMA helpers (PTX ISA 8.7, sm_100a) ----
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[32]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 bytes apart (stride byte offset), version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: fp16 A and B, fp32 D, both K-major, M = 128, N = NT.
template <int NT>
__device__ __forceinline__ uint32_t idesc_f16() {
  return (1u << 4) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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

template <int NT>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_qgemm_tc(QMat w, const float *__restrict__ x, int64_t ldx, int M, Epilogue ep, GemvScratch scr, int splits) {
  using Geo = TcGeo<NT>;
  extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
  unsigned char *sm = tc_smem_raw + ((1024 - (smem_u32(tc_smem_raw) & 1023)) & 1023);
  __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], accum;
  __shared__ uint32_t s_taddr;
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tile_n = blockIdx.x, tile_m = blockIdx.y, split = blockIdx.z;
  const int nq = (int)w.row_words;
  const int nstage = nq * 2;  // 64-wide K steps (quads of 128, zero-padded)
  const int ks0 = (int)((int64_t)split * nstage / splits), ks1 = (int)((int64_t)(split + 1) * nstage / splits);
  const int64_t nstrips = q4_strips(w.N);
  const int m0 = tile_m * NT;

  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], kTcProducerWarps);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accum, 1);
    fence_barrier_init();
  }
  if (warp == kTcProducerWarps) tmem_alloc(&s_taddr, Geo::TmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = s_taddr;
  asm volatile("griddepcontrol.wait;" ::: "memory");

  bool ok = true;
  if (warp < kTcProducerWarps) {
    // ================= producers =================
    for (int ks = ks0, i = 0; ks < ks1; ++ks, ++i) {
      const int s = i % kTcStages;
      if (i >= kTcStages) ok = ok && mbar_wait(&empty[s], (uint32_t)(i / kTcStages - 1) & 1, scr.err, DEVERR_GEMV_EMPTY);
      unsigned char *st = sm + s * Geo::Stage;
      if (ok) {
        if (warp < 4) {
          // A: weight row r = tid, blocks 2h, 2h+1 of quad Q
          const int r = tid;
          const int64_t strip = (int64_t)tile_n * (kTcRows / kQ4StripRows) + r / kQ4StripRows;
          const int rr = r % kQ4StripRows, Q = ks >> 1, h = ks & 1;
          if (strip < nstrips) {
            const unsigned char *qb =
                reinterpret_cast<const unsigned char *>(w.qs) + (strip * nq + Q) * (int64_t)kQ4QuadBytes;
            uint2 wd[4];  // lane-word t of blocks 2h (.x) and 2h+1 (.y)
#pragma unroll
            for (int t = 0; t < 4; ++t) wd[t] = __ldg(reinterpret_cast<const uint2 *>(qb + (rr * 4 + t) * 16 + 8 * h));
            const uint32_t dd = __ldg(reinterpret_cast<const uint32_t *>(qb + kQ4QuadCodeBytes + (rr * 4 + 2 * h) * 2));
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)(b ? (dd >> 16) : (dd & 0xFFFFu))));
              // chunk j = block elements 8j..8j+7: lane-words 2(j & 1), 2(j & 1) + 1, low nibbles
              // for j < 2 (elements 0..15), high nibbles for j >= 2 (elements 16..31)
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t wa = b ? wd[2 * (j & 1)].y : wd[2 * (j & 1)].x;
                const uint32_t wb = b ? wd[2 * (j & 1) + 1].y : wd[2 * (j & 1) + 1].x;
                const uint32_t p0 = __byte_perm(wa, 0u, 0x4140), p1 = __byte_perm(wa, 0u, 0x4342);
                const uint32_t p2 = __byte_perm(wb, 0u, 0x4140), p3 = __byte_perm(wb, 0u, 0x4342);
                uint4 chunk;
                if (j < 2)
                  chunk = make_uint4(dq_lo(p0, d2), dq_lo(p1, d2), dq_lo(p2, d2), dq_lo(p3, d2));
                else
                  chunk = make_uint4(dq_hi(p0, d2), dq_hi(p1, d2), dq_hi(p2, d2), dq_hi(p3, d2));
                const int cidx = b * 4 + j;  // 16-byte chunk of the 128-byte row
                *reinterpret_cast<uint4 *>(st + r * 128 + ((cidx ^ (r & 7)) * 16)) = chunk;
              }
            }
          } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4 *>(st + r * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
        } else {
          // B: token rows m0 .. m0 + NT - 1, fp32 -> fp16
          unsigned char *sb = st + kTcABytes;
          const int k0 = ks * kTcK;
          for (int idx = tid - 128; idx < NT * 8; idx += 128) {
            const int row = idx >> 3, c = idx & 7;
            const int m = m0 + row, k = k0 + 8 * c;
            uint4 chunk = make_uint4(0u, 0u, 0u, 0u);
            if (m < M && k < w.K) {
              const float4 a = *reinterpret_cast<const float4 *>(x + (int64_t)m * ldx + k);
              const float4 b = *reinterpret_cast<const float4 *>(x + (int64_t)m * ldx + k + 4);
              const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
              const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
              chunk = make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                                 *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
            }
            *reinterpret_cast<uint4 *>(sb + row * 128 + ((c ^ (row & 7)) * 16)) = chunk;
          }
        }
      }
      fence_proxy_async_smem();  // the tensor core reads these bytes through the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    }
  } else if (lane == 0) {
    // ================= MMA issuer =================
    const uint32_t idesc = idesc_f16<NT>();
    for (int ks = ks0, i = 0; ks < ks1; ++ks, ++i) {
      const int s = i % kTcStages;
      ok = ok && mbar_wait(&full[s], (uint32_t)(i / kTcStages) & 1, scr.err, DEVERR_GEMV_FULL);
      tc_fence_after();
      if (ok) {
        const uint32_t a = smem_u32(sm + s * Geo::Stage), b = a + kTcABytes;
#pragma unroll
        for (int kk = 0; kk < kTcK / 16; ++kk)  // K = 16 per MMA: 32 bytes further into the swizzle atom
          umma_f16(taddr, smem_desc_sw128(a + 32 * kk), smem_desc_sw128(b + 32 * kk), idesc,
                   (ks > ks0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(&empty[s]);  // frees the stage once the MMAs above have read it
    }
    umma_commit(&accum);
  }

  // ================= epilogue: warps 0..3 own TMEM lanes 0..127 =================
  if (warp < 4) {
    ok = ok && mbar_wait(&accum, 0, scr.err, DEVERR_GEMV_FULL);
    tc_fence_after();
    const int row = 32 * warp + lane;                      // weight row within the tile = TMEM lane
    const int64_t n = (int64_t)tile_n * kTcRows + row;     // output column
    const uint32_t tw = taddr + ((uint32_t)(32 * warp) << 16);
    float *part = nullptr;
    if (splits > 1) part = scr.part + (((int64_t)(tile_m * gridDim.x + tile_n) * splits) * kTcRows) * NT;
    constexpr int CW = NT < 32 ? 16 : 32;
    for (int c0 = 0; c0 < NT; c0 += CW) {
      float v[32];
      if (CW == 32)
        tmem_ld32(tw + c0, v);
      else
        tmem_ld16(tw + c0, v);
      if (splits > 1) {
#pragma unroll
        for (int j = 0; j < CW; ++j) part[((int64_t)split * kTcRows + row) * NT + c0 + j] = v[j];
      } else if (ok) {
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          const float partner = __shfl_xor_sync(0xffffffffu, v[j], 1);
          const int m = m0 + c0 + j;
          if ((lane & 1) == 0 && m < M) {
            if (n + 1 < w.N)
              epi_store_pair(ep, n, m, v[j], partner);
            else if (n < w.N && ep.mode == EPI_PLAIN)
              epi_store_one(ep, n, m, v[j]);
          }
        }
      }
    }
    if (splits > 1) {
      // the last split of this tile to arrive sums the partials in split order
      __threadfence();
      named_sync_id(1, 128);
      if (tid == 0) s_last = atomicAdd(scr.tickets + tile_m * gridDim.x + tile_n, 1) == splits - 1;
      named_sync_id(1, 128);
      if (s_last) {
        __threadfence();
        if (tid == 0) scr.tickets[tile_m * gridDim.x + tile_n] = 0;
        for (int j = 0; j < NT; ++j) {
          float acc = 0.0f;
          for (int q = 0; q < splits; ++q) acc += __ldcg(part + ((int64_t)q * kTcRows + row) * NT + j);
          const float partner = __shfl_xor_sync(0xffffffffu, acc, 1);
          const int m = m0 + j;
          if (ok && (lane & 1) == 0 && m < M) {
            if (n + 1 < w.N)
              epi_store_pair(ep, n, m, acc, partner);
            else if (n < w.N && ep.mode == EPI_PLAIN)
              epi_store_one(ep, n, m, acc);
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == kTcProducerWarps) {
    tc_fence_after();
    tmem_dealloc(taddr, Geo::TmemCols);
  }
}

template <int NT>
void launch_tc_t(const QMat &w, const float *x, int M, int64_t ldx, const Epilogue &ep, const GemvScratch &sc,
                 int num_sms, cudaStream_t s) {
  using Geo = TcGeo<NT>;
  const int tiles_n = (int)ceil_div(w.N, kTcRows), tiles_m = (int)ceil_div(M, NT);
  const int nstage = (int)w.row_words * 2;
  int splits = 1;
  const int tiles = tiles_n * tiles_m;
  if (tiles < num_sms) splits = (int)std::min<int64_t>(ceil_div(num_sms, tiles), std::max(1, nstage / 4));
  if (splits > 1) {
    const uint64_t need = (uint64_t)tiles * splits * kTcRows * NT;
    if (need > sc.part_floats || tiles > sc.n_tickets) splits = 1;
  }
  static unsigned long long attr_set = 0;
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << dev))) {
    FG_CUDA(cudaFuncSetAttribute(k_qgemm_tc<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Geo::Smem));
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)tiles_n, (unsigned)tiles_m, (unsigned)splits);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = Geo::Smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FG_CUDA(cudaLaunchKernelEx(&cfg, k_qgemm_tc<NT>, w, x, ldx, M, ep, sc, splits));
}

}  // namespace

bool qgemm_tc_supported(const QMat &w, int M) {
  return w.qtype == FG_Q4_0 && M >= 1 && w.K % 32 == 0 && w.K >= 32 && w.N >= 1;
}

void launch_qgemm_tc(const QMat &w, const float *x, int M, int64_t ldx, const Epilogue &ep, const GemvScratch &sc,
                     int num_sms, cudaStream_t s) {
  FG_REQUIRE(qgemm_tc_supported(w, M), FG_ERR_SHAPE, "tensor-core GEMM: unsupported matrix");
  FG_REQUIRE(ldx % 4 == 0 && ((uintptr_t)x & 15) == 0, FG_ERR_VALIDATION, "GEMM: x must be 16-byte aligned rows");
  if (M == 0 || w.N == 0) return;
  // token tile: the smallest UMMA N that covers M, up to 256 tokens per CTA
  if (M <= 16)
    launch_tc_t<16>(w, x, M, ldx, ep, sc, num_sms, s);
  else if (M <= 32)
    launch_tc_t<32>(w, x, M, ldx, ep, sc, num_sms, s);
  else if (M <= 64)
    launch_tc_t<64>(w, x, M, ldx, ep, sc, num_sms, s);
  else if (M <= 128)
    launch_tc_t<128>(w, x, M, ldx, ep, sc, num_sms, s);
  else
    launch_tc_t<256>(w, x, M, ldx, ep, sc, num_sms, s);
}

}  // namespace fg
