// Fused dequant-GEMV for batch-1..4 decode: y[m, n] = sum_k x[m, k] W[n, k],
// W in Q4_0 / Q8_0 (device layout: reference unpack packing + fp16 scales).
//
// Roofline: HBM-bound.  Algorithmic bytes per launch = N*K/32 blocks *
// (18 B Q4_0 | 34 B Q8_0) + 4*M*(K + N); each weight byte is read once.
//
// Design (sm_100a):
//  * a warp owns R rows; lane l takes 32-value block l of each 1024-value
//    chunk of those rows: one 16-byte streaming load per row per block (Q4_0,
//    two for Q8_0), so a warp-load is 512 contiguous bytes;
//  * x is staged once per CTA in shared memory, pre-scaled for the magic-
//    number unpack below and stored with a 16-byte XOR swizzle (slot q of
//    block b at q ^ (b & 7)) so the per-lane float4 reads are conflict-free;
//    the RMSNorm that precedes every projection is fused into this staging;
//  * nibbles become fp32 without I2F: (w & 0xF<<4p) | 0x4B000000 is the float
//    2^23 + n*16^p; one packed FADD2 removes 2^23 + 8*16^p exactly, leaving
//    (n - 8) * 16^p, whose 16^p is cancelled by the pre-scaled x.  Products
//    accumulate with packed FFMA2 in fp32 and are scaled by the block's fp16 d
//    once per block.  Q8_0 bytes go through PRMT into 2^23 + byte the same way;
//  * optional split-K across the warps of a CTA fills the GPU for short N;
//  * next-chunk loads are issued before the current chunk's math.
#include "epilogue.cuh"

namespace fg {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// 2^23 + 8 * 16^p for nibble positions p = 0..7 (positions 5..7 are read
// after a 12-bit shift, so their scale is 16^(p-3)).
#define FG_M1 (-8388616.0f)
#define FG_M16 (-8388736.0f)
#define FG_M256 (-8390656.0f)
#define FG_M4096 (-8421376.0f)
#define FG_M65536 (-8912896.0f)


// Word of 8 nibbles -> 4 pairs (p0,p1) (p2,p3) (p4,p5) (p6,p7), each value
// (n_p - 8) * 16^p' exactly.
__device__ __forceinline__ void unpack_q4(uint32_t w, float2 v[4]) {
  const uint32_t M = 0x4B000000u;
  const uint32_t w12 = w >> 12;
  v[0] = fadd2(make_float2(__uint_as_float((w & 0xFu) | M), __uint_as_float((w & 0xF0u) | M)),
               make_float2(FG_M1, FG_M16));
  v[1] = fadd2(make_float2(__uint_as_float((w & 0xF00u) | M), __uint_as_float((w & 0xF000u) | M)),
               make_float2(FG_M256, FG_M4096));
  v[2] = fadd2(make_float2(__uint_as_float((w & 0xF0000u) | M), __uint_as_float((w12 & 0xF00u) | M)),
               make_float2(FG_M65536, FG_M256));
  v[3] = fadd2(make_float2(__uint_as_float((w12 & 0xF000u) | M), __uint_as_float((w12 & 0xF0000u) | M)),
               make_float2(FG_M4096, FG_M65536));
}

// Word of 4 offset-binary bytes -> 2 pairs of exact int8 values.
__device__ __forceinline__ void unpack_q8(uint32_t w, float2 v[2]) {
  const uint32_t M = 0x4B000000u;
  const float2 off = make_float2(-8388736.0f, -8388736.0f);  // 2^23 + 128
  v[0] = fadd2(make_float2(__uint_as_float(__byte_perm(w, M, 0x7540)), __uint_as_float(__byte_perm(w, M, 0x7541))),
               off);
  v[1] = fadd2(make_float2(__uint_as_float(__byte_perm(w, M, 0x7542)), __uint_as_float(__byte_perm(w, M, 0x7543))),
               off);
}

template <int QT>
struct QTraits;
template <>
struct QTraits<FG_Q4_0> {
  static constexpr int kU4 = 1;     // 16-byte loads per block
  static constexpr int kWords = 4;  // u32 words per block
};
template <>
struct QTraits<FG_Q8_0> {
  static constexpr int kU4 = 2;
  static constexpr int kWords = 8;
};

template <int QT, int MV, int R>
__global__ void __launch_bounds__(kThreads) k_qgemv(QMat w, const float *__restrict__ x, int64_t ldx,
                                                      const float *__restrict__ gamma, float eps, int do_norm,
                                                      int ksplit, Epilogue ep) {
  using T = QTraits<QT>;
  extern __shared__ float4 smem4[];
  __shared__ float s_red[kWarps][R * MV];
  __shared__ float s_norm[kWarps][MV];
  __shared__ float s_inv[MV];

  const int nb = (int)(w.K >> 5);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float4 *xs = smem4;  // [MV][nb][8] float4, swizzled

  // Wait for the producer of x (programmatic dependent launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- fused RMSNorm statistics (rmsnorm.wgsl.ts:44-66) ----
  if (do_norm) {
    float ss[MV];
#pragma unroll
    for (int m = 0; m < MV; ++m) ss[m] = 0.0f;
    for (int i = tid; i < nb * 8; i += kThreads) {
#pragma unroll
      for (int m = 0; m < MV; ++m) {
        float4 v = *reinterpret_cast<const float4 *>(x + m * ldx + 4 * i);
        ss[m] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
    }
#pragma unroll
    for (int m = 0; m < MV; ++m) {
      float s = warp_sum(ss[m]);
      if (lane == 0) s_norm[warp][m] = s;
    }
    __syncthreads();
    if (tid < MV) {
      float s = 0.0f;
      for (int i = 0; i < kWarps; ++i) s += s_norm[i][tid];
      s_inv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)w.K), eps)));
    }
    __syncthreads();
  }

  // ---- stage x: normalise, pre-scale, swizzle ----
  for (int idx = tid; idx < MV * nb * 8; idx += kThreads) {
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
        const float4 g = *reinterpret_cast<const float4 *>(gamma + 32 * b + 4 * q);
        v.x = __fmul_rn(v.x, g.x);
        v.y = __fmul_rn(v.y, g.y);
        v.z = __fmul_rn(v.z, g.z);
        v.w = __fmul_rn(v.w, g.w);
      }
    }
    if (QT == FG_Q4_0) {
      // element 4q+i sits at nibble position (4q+i) & 7, unpacked with scale
      // 1, 16, 256, 4096, 65536, 256, 4096, 65536 for positions 0..7
      if ((q & 1) == 0) {
        v.y *= 0x1p-4f;
        v.z *= 0x1p-8f;
        v.w *= 0x1p-12f;
      } else {
        v.x *= 0x1p-16f;
        v.y *= 0x1p-8f;
        v.z *= 0x1p-12f;
        v.w *= 0x1p-16f;
      }
    }
    xs[(m * nb + b) * 8 + (q ^ (b & 7))] = v;
  }
  __syncthreads();

  const int gpc = kWarps / ksplit;  // row groups per CTA
  const int64_t row0 = ((int64_t)blockIdx.x * gpc + warp / ksplit) * R;
  const int kp = warp % ksplit;
  const int nchunks = (nb + 31) >> 5;

  float2 acc[R][MV];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MV; ++m) acc[r][m] = make_float2(0.0f, 0.0f);

  if (row0 < w.N) {
    const uint4 *qrow[R];
    const __half *drow[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      qrow[r] = reinterpret_cast<const uint4 *>(w.qs) + (row0 + r) * nb * T::kU4;
      drow[r] = w.d + (row0 + r) * nb;
    }
    uint4 qn[R][T::kU4];
    __half dn[R];
    int c = kp;
    int b = c * 32 + lane;
    if (c < nchunks && b < nb) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int u = 0; u < T::kU4; ++u) qn[r][u] = ld_stream_u4(qrow[r] + b * T::kU4 + u);
        dn[r] = drow[r][b];
      }
    }
    for (; c < nchunks; c += ksplit) {
      uint4 qc[R][T::kU4];
      float dc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int u = 0; u < T::kU4; ++u) qc[r][u] = qn[r][u];
        dc[r] = __half2float(dn[r]);
      }
      const int bc = b;
      // prefetch the next chunk of this warp
      b = (c + ksplit) * 32 + lane;
      if (c + ksplit < nchunks && b < nb) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
          for (int u = 0; u < T::kU4; ++u) qn[r][u] = ld_stream_u4(qrow[r] + b * T::kU4 + u);
          dn[r] = drow[r][b];
        }
      }
      if (bc < nb) {
        float2 part[R][MV];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int m = 0; m < MV; ++m) part[r][m] = make_float2(0.0f, 0.0f);
        const int sw = bc & 7;
#pragma unroll
        for (int t = 0; t < T::kWords; ++t) {
          if (QT == FG_Q4_0) {
            float4 xa[MV], xb[MV];
#pragma unroll
            for (int m = 0; m < MV; ++m) {
              const float4 *xbk = xs + (m * nb + bc) * 8;
              xa[m] = xbk[(2 * t) ^ sw];
              xb[m] = xbk[(2 * t + 1) ^ sw];
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const uint32_t word = t == 0 ? qc[r][0].x : t == 1 ? qc[r][0].y : t == 2 ? qc[r][0].z : qc[r][0].w;
              float2 v[4];
              unpack_q4(word, v);
#pragma unroll
              for (int m = 0; m < MV; ++m) {
                part[r][m] = ffma2(v[0], make_float2(xa[m].x, xa[m].y), part[r][m]);
                part[r][m] = ffma2(v[1], make_float2(xa[m].z, xa[m].w), part[r][m]);
                part[r][m] = ffma2(v[2], make_float2(xb[m].x, xb[m].y), part[r][m]);
                part[r][m] = ffma2(v[3], make_float2(xb[m].z, xb[m].w), part[r][m]);
              }
            }
          } else {
            float4 xa[MV];
#pragma unroll
            for (int m = 0; m < MV; ++m) xa[m] = xs[(m * nb + bc) * 8 + (t ^ sw)];
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const uint4 &q4 = qc[r][t >> 2];
              const int tt = t & 3;
              const uint32_t word = tt == 0 ? q4.x : tt == 1 ? q4.y : tt == 2 ? q4.z : q4.w;
              float2 v[2];
              unpack_q8(word, v);
#pragma unroll
              for (int m = 0; m < MV; ++m) {
                part[r][m] = ffma2(v[0], make_float2(xa[m].x, xa[m].y), part[r][m]);
                part[r][m] = ffma2(v[1], make_float2(xa[m].z, xa[m].w), part[r][m]);
              }
            }
          }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int m = 0; m < MV; ++m) acc[r][m] = ffma2(part[r][m], make_float2(dc[r], dc[r]), acc[r][m]);
      }
    }
  }

  // Let the next kernel in the stream get resident while this one drains.
  asm volatile("griddepcontrol.launch_dependents;");

  // ---- reduce: lanes, then the ksplit warps of a row group ----
  float tot[R * MV];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MV; ++m) tot[r * MV + m] = warp_sum(acc[r][m].x + acc[r][m].y);
  if (ksplit > 1) {
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < R * MV; ++j) s_red[warp][j] = tot[j];
    }
    __syncthreads();
    if (kp == 0) {
#pragma unroll
      for (int j = 0; j < R * MV; ++j) {
        float s = 0.0f;
        for (int k = 0; k < ksplit; ++k) s += s_red[warp + k][j];
        tot[j] = s;
      }
    }
  }
  if (kp != 0 || row0 >= w.N) return;

  // ---- epilogue: lane (r, m) owns one output, pairs handled by even r ----
  if (lane < R * MV) {
    const int r = lane / MV, m = lane % MV;
    float v = 0.0f, vn = 0.0f;
#pragma unroll
    for (int j = 0; j < R * MV; ++j) {
      if (j == lane) v = tot[j];
      if (j == lane + MV) vn = tot[j];
    }
    if (R % 2 == 0) {
      if ((r & 1) == 0) epi_store_pair(ep, row0 + r, m, v, vn);
    } else {
      epi_store_one(ep, row0 + r, m, v);
    }
  }
}

template <int QT, int MV, int R>
void launch_t(const QMat &w, const float *x, int64_t ldx, const float *gamma, float eps, bool do_norm,
              const Epilogue &ep, int num_sms, cudaStream_t s) {
  const int64_t nb = w.K / 32;
  const int64_t groups = w.N / R;
  const int64_t nchunks = ceil_div(nb, 32);
  int ksplit = 1;
  while (ksplit < 8 && groups * ksplit < (int64_t)num_sms * 16 && nchunks >= 2 * ksplit) ksplit *= 2;
  const int gpc = kWarps / ksplit;
  const int grid = (int)ceil_div(groups, gpc);
  const size_t smem = (size_t)MV * nb * 8 * sizeof(float4);
  static unsigned long long attr_set = 0;  // per instantiation, one bit per device
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << dev))) {
    FG_CUDA(cudaFuncSetAttribute(k_qgemv<QT, MV, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_set |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FG_CUDA(cudaLaunchKernelEx(&cfg, k_qgemv<QT, MV, R>, w, x, ldx, gamma, eps, do_norm ? 1 : 0, ksplit, ep));
}

template <int QT, int MV>
void launch_r(const QMat &w, const float *x, int64_t ldx, const float *gamma, float eps, bool do_norm,
              const Epilogue &ep, int num_sms, cudaStream_t s) {
  if (w.N % 4 == 0)
    launch_t<QT, MV, 4>(w, x, ldx, gamma, eps, do_norm, ep, num_sms, s);
  else if (w.N % 2 == 0)
    launch_t<QT, MV, 2>(w, x, ldx, gamma, eps, do_norm, ep, num_sms, s);
  else {
    FG_REQUIRE(ep.mode == EPI_PLAIN, FG_ERR_SHAPE, "paired epilogue needs an even row count (N=%lld)", (long long)w.N);
    launch_t<QT, MV, 1>(w, x, ldx, gamma, eps, do_norm, ep, num_sms, s);
  }
}

template <int QT>
void launch_m(const QMat &w, const float *x, int M, int64_t ldx, const float *gamma, float eps, bool do_norm,
              const Epilogue &ep, int num_sms, cudaStream_t s) {
  switch (M) {
    case 1: launch_r<QT, 1>(w, x, ldx, gamma, eps, do_norm, ep, num_sms, s); break;
    case 2: launch_r<QT, 2>(w, x, ldx, gamma, eps, do_norm, ep, num_sms, s); break;
    case 3: launch_r<QT, 3>(w, x, ldx, gamma, eps, do_norm, ep, num_sms, s); break;
    default: launch_r<QT, 4>(w, x, ldx, gamma, eps, do_norm, ep, num_sms, s); break;
  }
}

}  // namespace

bool gemv_supported(const QMat &w, int M) {
  return M >= 1 && M <= 4 && (uint64_t)M * w.K * 4 <= 200 * 1024 && w.K % 32 == 0;
}

void launch_qgemv_ld(const QMat &w, const float *x, int M, int64_t ldx, const float *norm_gamma, float norm_eps,
                     bool do_norm, const Epilogue &ep, int num_sms, cudaStream_t s) {
  FG_REQUIRE(gemv_supported(w, M), FG_ERR_SHAPE, "gemv: unsupported M=%d K=%lld", M, (long long)w.K);
  if (w.qtype == FG_Q4_0)
    launch_m<FG_Q4_0>(w, x, M, ldx, norm_gamma, norm_eps, do_norm, ep, num_sms, s);
  else
    launch_m<FG_Q8_0>(w, x, M, ldx, norm_gamma, norm_eps, do_norm, ep, num_sms, s);
}

void launch_qgemv(const QMat &w, const float *x, int M, const float *norm_gamma, float norm_eps, bool do_norm,
                  const Epilogue &ep, int num_sms, cudaStream_t s) {
  launch_qgemv_ld(w, x, M, w.K, norm_gamma, norm_eps, do_norm, ep, num_sms, s);
}

}  // namespace fg
