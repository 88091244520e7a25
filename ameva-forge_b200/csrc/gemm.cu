// GEMM paths for more than 4 token rows (prefill, batched decode) and the
// dense fp32 gpuCore.matmul.
//
// k_qgemm_simt: dequantised fp32 FFMA GEMM, 64x64 output tile, one 32-value
// quant block per K step.  The tile's weights are dequantised exactly as the
// reference unpack ((code - zero) * scale) into shared memory and consumed by
// a 4x4 register tile per thread.  It is the portable GEMM of this library;
// the tensor-core GEMM (gemm_tc.cu) takes the shapes it supports.
#include <cstdlib>
#include <string>

#include "epilogue.cuh"

namespace fg {
namespace {

constexpr int BM = 64, BN = 64, BK = 32;

__global__ void __launch_bounds__(256) k_qgemm_simt(QMat w, const float *__restrict__ x, int64_t ldx, int M,
                                                    Epilogue ep) {
  __shared__ __align__(16) float xs[BK][BM + 4];
  __shared__ __align__(16) float ws[BK][BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t n0 = (int64_t)blockIdx.x * BN;
  const int m0 = blockIdx.y * BM;
  const int nb = (int)(w.K >> 5);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  for (int kb = 0; kb < nb; ++kb) {
    // x tile [BM][32] -> xs[k][m]
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int idx = tid + it * 256;  // 512 float4
      const int r = idx >> 3, q = idx & 7;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m0 + r < M) v = *reinterpret_cast<const float4 *>(x + (int64_t)(m0 + r) * ldx + kb * 32 + 4 * q);
      xs[4 * q + 0][r] = v.x;
      xs[4 * q + 1][r] = v.y;
      xs[4 * q + 2][r] = v.z;
      xs[4 * q + 3][r] = v.w;
    }
    // weight tile [BN][32]: thread -> (row tid/4, word tid%4), exact dequant
    {
      const int r = tid >> 2, t = tid & 3;
      const int64_t n = n0 + r;
      const float sc = n < w.N ? __half2float(w.d[qmat_scale_at(w, n, kb)]) : 0.0f;
      if (w.qtype == FG_Q4_0) {
        const uint32_t word = n < w.N ? w.qs[q4_word_at(w, n, kb, t)] : 0x88888888u;
#pragma unroll
        for (int p = 0; p < 8; ++p)
          ws[q4_elem(t, p)][r] = __fmul_rn(__fsub_rn((float)((word >> (4 * p)) & 0xFu), 8.0f), sc);
      } else {
        const uint2 wd = n < w.N ? reinterpret_cast<const uint2 *>(w.qs + n * w.row_words)[kb * 4 + t]
                                 : make_uint2(0x80808080u, 0x80808080u);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ws[8 * t + k][r] = __fmul_rn(__fsub_rn((float)((wd.x >> (8 * k)) & 0xFFu), 128.0f), sc);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ws[8 * t + 4 + k][r] = __fmul_rn(__fsub_rn((float)((wd.y >> (8 * k)) & 0xFFu), 128.0f), sc);
      }
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < BK; ++k) {
      const float4 a = *reinterpret_cast<const float4 *>(&xs[k][ty * 4]);
      const float4 b = *reinterpret_cast<const float4 *>(&ws[k][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  asm volatile("griddepcontrol.launch_dependents;");
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      const int64_t n = n0 + tx * 4 + j;
      if (n + 1 < w.N) {
        epi_store_pair(ep, n, m, acc[i][j], acc[i][j + 1]);
      } else if (n < w.N) {
        epi_store_one(ep, n, m, acc[i][j]);
      }
    }
  }
}

// Dense fp32 C = A B (matmul_tiled.wgsl.ts semantics, edges zero-padded).  BT: B is stored
// transposed, [N, K] row-major (nn.Linear's x W^T without materialising W^T).
template <bool BT>
__global__ void __launch_bounds__(256) k_matmul_f32(const float *__restrict__ A, const float *__restrict__ B,
                                                    float *__restrict__ C, int64_t M, int64_t K, int64_t N) {
  __shared__ __align__(16) float as[16][BM + 4];
  __shared__ __align__(16) float bs[16][BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t n0 = (int64_t)blockIdx.x * BN, m0 = (int64_t)blockIdx.y * BM;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += 16) {
    for (int idx = tid; idx < BM * 16; idx += 256) {
      const int r = idx / 16, k = idx % 16;
      as[k][r] = (m0 + r < M && k0 + k < K) ? A[(m0 + r) * K + k0 + k] : 0.0f;
    }
    for (int idx = tid; idx < BN * 16; idx += 256) {
      if constexpr (BT) {  // consecutive threads walk K: coalesced rows of B^T
        const int c = idx / 16, k = idx % 16;
        bs[k][c] = (n0 + c < N && k0 + k < K) ? B[(n0 + c) * K + k0 + k] : 0.0f;
      } else {
        const int k = idx / BN, c = idx % BN;
        bs[k][c] = (n0 + c < N && k0 + k < K) ? B[(k0 + k) * N + n0 + c] : 0.0f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = as[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = bs[k][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < M && n < N) C[m * N + n] = acc[i][j];
    }
}

}  // namespace

void launch_qgemm(const QMat &w, const float *x, int M, int64_t ldx, const Epilogue &ep, const GemvScratch &sc,
                  int num_sms, cudaStream_t s) {
  if (M == 0 || w.N == 0) return;
  // Q4_0 and Q8_0 run on the tensor cores; FORGE_B200_GEMM=simt keeps the CUDA-core kernel (for comparison)
  static const bool force_simt = [] {
    const char *e = std::getenv("FORGE_B200_GEMM");
    return e && std::string(e) == "simt";
  }();
  if (!force_simt && qgemm_tc_supported(w, M)) {
    launch_qgemm_tc(w, x, M, ldx, ep, sc, num_sms, s);
    return;
  }
  dim3 grid((unsigned)ceil_div(w.N, BN), (unsigned)ceil_div(M, BM));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FG_CUDA(cudaLaunchKernelEx(&cfg, k_qgemm_simt, w, x, ldx, M, ep));
}

void launch_matmul_f32(const float *A, const float *B, float *C, int64_t M, int64_t K, int64_t N, cudaStream_t s,
                       bool b_trans) {
  if (M == 0 || N == 0) return;
  dim3 grid((unsigned)ceil_div(N, BN), (unsigned)ceil_div(M, BM));
  if (b_trans)
    k_matmul_f32<true><<<grid, 256, 0, s>>>(A, B, C, M, K, N);
  else
    k_matmul_f32<false><<<grid, 256, 0, s>>>(A, B, C, M, K, N);
  FG_LAUNCH_CHECK();
}

}  // namespace fg
