// Attention kernels with the reference flash-attention semantics
// (packages/forge/src/tensor/kernels/flash_attention.wgsl.ts:13-178):
//   GQA kv_head = h / (H / H_kv)                          (:58-59)
//   causal: key j visible iff j < N_kv - N_q + i + 1      (:92-96, KV offset)
//   running max starts at -1e30, out = acc / max(l, 1e-12) (:72, :160)
//
// k_attn_simt   -- fp32 (or fp16-in) online-softmax attention for any
//                  N_q, d <= 256: a 32-query tile per CTA, 32-key tiles in
//                  shared memory, 4 threads per query row.
// k_attn_decode -- split-KV decode (N_q = 1) over the fp16 KV cache: each
//                  CTA streams one slice of one KV head for all of its G query
//                  heads with a three-stage ring of cp.async tiles per warp
//                  (two 32-key tiles in flight while one is computed); the last CTA of a
//                  head (atomic ticket) merges the slices, so no second launch.
#include "runtime.cuh"

namespace fg {
namespace {

constexpr float kMaskInit = -1e30f;

__device__ __forceinline__ int kv_len(const AttnArgs &a, int b) {
  return a.n_kv_dev ? a.n_kv_dev[b] + a.n_kv_add : a.n_kv;
}

__device__ __forceinline__ float load_any(const void *p, int64_t i, int f16) {
  return f16 ? __half2float(reinterpret_cast<const __half *>(p)[i]) : reinterpret_cast<const float *>(p)[i];
}

// ------------------------------------------------------------------------
// Generic fp32 attention.  Thread (r, sub): query row r of the tile, keys
// sub, sub+4, ... of each key tile, output columns sub, sub+4, ...
// ------------------------------------------------------------------------
template <int D, int BQ>
__global__ void __launch_bounds__(BQ * 4) k_attn_simt(AttnArgs a) {
  constexpr int BKV = 32;
  constexpr int DP = D + 4;  // padded row (bank spread)
  constexpr int CPT = D / 4; // output columns per thread
  extern __shared__ float sm[];
  float *Qs = sm;                 // [BQ][DP]
  float *Ks = Qs + BQ * DP;       // [BKV][DP]
  float *Vs = Ks + BKV * DP;      // [BKV][DP]
  float *Ps = Vs + BKV * DP;      // [BQ][BKV+1]

  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.z, h = blockIdx.y;
  const int i0 = blockIdx.x * BQ;
  const int tid = threadIdx.x, r = tid >> 2, sub = tid & 3;
  const int d = a.d;
  const int hk = h / (a.H / a.Hkv);
  const int nkv = kv_len(a, b);
  const int64_t qbase = (int64_t)b * a.q_sb + (int64_t)h * a.q_sh;
  const int64_t kvbase = (int64_t)b * a.kv_sb + (int64_t)hk * a.kv_sh;

  for (int idx = tid; idx < BQ * D; idx += BQ * 4) {
    const int rr = idx / D, c = idx % D;
    float v = 0.0f;
    if (i0 + rr < a.Nq && c < d) v = load_any(a.q, qbase + (int64_t)(i0 + rr) * a.q_si + c, a.q_f16);
    Qs[rr * DP + c] = v;
  }
  const int i = i0 + r;  // this thread's query
  int lim = nkv;
  if (a.causal) lim = min(nkv, nkv - a.Nq + i + 1);
  int lim_tile = nkv;  // keys any row of the tile may see
  if (a.causal) lim_tile = min(nkv, nkv - a.Nq + min(i0 + BQ, a.Nq));
  float m = kMaskInit, l = 0.0f;
  float o[CPT];
#pragma unroll
  for (int c = 0; c < CPT; ++c) o[c] = 0.0f;

  for (int j0 = 0; j0 < lim_tile; j0 += BKV) {
    __syncthreads();
    for (int idx = tid; idx < BKV * D; idx += BQ * 4) {
      const int jj = idx / D, c = idx % D;
      float kv = 0.0f, vv = 0.0f;
      if (j0 + jj < nkv && c < d) {
        const int64_t off = kvbase + (int64_t)(j0 + jj) * d + c;
        kv = load_any(a.k, off, a.kv_f16);
        vv = load_any(a.v, off, a.kv_f16);
      }
      Ks[jj * DP + c] = kv;
      Vs[jj * DP + c] = vv;
    }
    __syncthreads();
    float s[BKV / 4];
    float tmax = -INFINITY;
#pragma unroll
    for (int t = 0; t < BKV / 4; ++t) {
      const int jj = t * 4 + sub;
      float acc = 0.0f;
      const float4 *qr = reinterpret_cast<const float4 *>(Qs + r * DP);
      const float4 *kr = reinterpret_cast<const float4 *>(Ks + jj * DP);
#pragma unroll 8
      for (int c4 = 0; c4 < D / 4; ++c4) {
        const float4 qv = qr[c4], kv = kr[c4];
        acc = fmaf(qv.x, kv.x, acc);
        acc = fmaf(qv.y, kv.y, acc);
        acc = fmaf(qv.z, kv.z, acc);
        acc = fmaf(qv.w, kv.w, acc);
      }
      const bool ok = (j0 + jj) < lim && i < a.Nq;
      s[t] = ok ? acc * a.scale : -INFINITY;
      tmax = fmaxf(tmax, s[t]);
    }
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
    const float mn = fmaxf(m, tmax);
    const float alpha = expf(m - mn);
    float ps = 0.0f;
#pragma unroll
    for (int t = 0; t < BKV / 4; ++t) {
      const float p = expf(s[t] - mn);
      ps += p;
      Ps[r * (BKV + 1) + t * 4 + sub] = p;
    }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l = l * alpha + ps;
    m = mn;
    __syncwarp();
#pragma unroll
    for (int c = 0; c < CPT; ++c) o[c] *= alpha;
    for (int jj = 0; jj < BKV; ++jj) {
      const float p = Ps[r * (BKV + 1) + jj];
      const float *vr = Vs + jj * DP + sub;  // columns sub, sub+4, ...: 4 threads hit 4 banks
#pragma unroll
      for (int c = 0; c < CPT; ++c) o[c] = fmaf(p, vr[4 * c], o[c]);
    }
  }
  asm volatile("griddepcontrol.launch_dependents;");
  if (i < a.Nq) {
    const float inv = 1.0f / fmaxf(l, 1e-12f);
    float *orow = a.o + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + (int64_t)i * a.o_si;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      const int col = 4 * c + sub;
      if (col < d) orow[col] = o[c] * inv;
    }
  }
}

// ------------------------------------------------------------------------
// Split-KV decode.  Warp w of a CTA owns a contiguous run of 32-key tiles;
// lane l owns key l of a tile for Q.K (K rows stored with a 16-byte XOR
// swizzle) and output columns [l*D/32, (l+1)*D/32) for P.V.
// ------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, int src_bytes) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kDecodeStages = 3;  // cp.async ring depth per warp of k_attn_decode

template <int D, int G>
__global__ void __launch_bounds__(128) k_attn_decode(AttnArgs a, int splits, float *__restrict__ part,
                                                     int *__restrict__ counters) {
  constexpr int W = 4, T = 32, NS = kDecodeStages;
  constexpr int CH = D / 8;            // 16-byte chunks per row
  constexpr int RPI = 32 / CH;         // rows per warp-instruction in the tile copy
  constexpr int CPL = D / 32;          // output columns per lane
  extern __shared__ __align__(16) unsigned char smraw[];
  __half *kv = reinterpret_cast<__half *>(smraw);           // [W][NS][2][T][D]
  float *qs = reinterpret_cast<float *>(kv + W * NS * 2 * T * D);  // [G][D]
  float *ps = qs + G * D;                                   // [W][G][T]
  __shared__ int s_last;

  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.z, hk = blockIdx.y, split = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nkv = kv_len(a, b);
  const int per = (nkv + splits - 1) / splits;
  const int s0 = min(nkv, split * per), s1 = min(nkv, s0 + per);
  // warp sub-range, in whole tiles
  const int ntile = (s1 - s0 + T - 1) / T;
  const int tpw = (ntile + W - 1) / W;
  const int t0 = min(ntile, warp * tpw), t1 = min(ntile, t0 + tpw);

  for (int idx = tid; idx < G * D; idx += 128) {
    const int g = idx / D, c = idx % D;
    const int h = hk * G + g;
    qs[idx] = load_any(a.q, (int64_t)b * a.q_sb + (int64_t)h * a.q_sh + c, a.q_f16) * a.scale;
  }
  __syncthreads();

  const __half *kbase = reinterpret_cast<const __half *>(a.k) + (int64_t)b * a.kv_sb + (int64_t)hk * a.kv_sh;
  const __half *vbase = reinterpret_cast<const __half *>(a.v) + (int64_t)b * a.kv_sb + (int64_t)hk * a.kv_sh;
  __half *wk = kv + warp * NS * 2 * T * D;  // this warp's stages

  auto issue = [&](int t, int stage) {
    const int key0 = s0 + t * T;
    __half *ks = wk + stage * 2 * T * D;
    __half *vs = ks + T * D;
#pragma unroll
    for (int it = 0; it < T / RPI; ++it) {
      const int row = it * RPI + lane / CH, ch = lane % CH;
      const int key = key0 + row;
      const bool ok = key < s1;
      const int64_t src = (int64_t)(ok ? key : s0) * D + ch * 8;
      cp_async16(ks + row * D + ((ch ^ (row & 7)) * 8), kbase + src, ok ? 16 : 0);
      cp_async16(vs + row * D + ch * 8, vbase + src, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  float m[G], lsum[G], o[G][CPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = kMaskInit;
    lsum[g] = 0.0f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) o[g][c] = 0.0f;
  }

  static_assert(NS == 3, "the waits below assume three stages");
  if (t0 < t1) issue(t0, 0);
  if (t0 + 1 < t1) issue(t0 + 1, 1);
  for (int t = t0; t < t1; ++t) {
    const int stage = (t - t0) % NS;
    if (t + 2 < t1) {  // the stage of tile t + 2 held tile t - 1, finished before the last __syncwarp
      issue(t + 2, (t - t0 + 2) % NS);
      cp_async_wait<2>();
    } else if (t + 1 < t1) {
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();
    const __half *ks = wk + stage * 2 * T * D;
    const __half *vs = ks + T * D;
    const bool valid = s0 + t * T + lane < s1;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.0f;
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
      const uint4 kk = *reinterpret_cast<const uint4 *>(ks + lane * D + ((ch ^ (lane & 7)) * 8));
      const float2 k01 = __half22float2(*reinterpret_cast<const __half2 *>(&kk.x));
      const float2 k23 = __half22float2(*reinterpret_cast<const __half2 *>(&kk.y));
      const float2 k45 = __half22float2(*reinterpret_cast<const __half2 *>(&kk.z));
      const float2 k67 = __half22float2(*reinterpret_cast<const __half2 *>(&kk.w));
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 qa = *reinterpret_cast<const float4 *>(qs + g * D + ch * 8);
        const float4 qb = *reinterpret_cast<const float4 *>(qs + g * D + ch * 8 + 4);
        float acc = s[g];
        acc = fmaf(qa.x, k01.x, acc);
        acc = fmaf(qa.y, k01.y, acc);
        acc = fmaf(qa.z, k23.x, acc);
        acc = fmaf(qa.w, k23.y, acc);
        acc = fmaf(qb.x, k45.x, acc);
        acc = fmaf(qb.y, k45.y, acc);
        acc = fmaf(qb.z, k67.x, acc);
        acc = fmaf(qb.w, k67.y, acc);
        s[g] = acc;
      }
    }
    float *pw = ps + warp * G * T;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sv = valid ? s[g] : -INFINITY;
      const float tmax = warp_max(sv);
      const float mn = fmaxf(m[g], tmax);
      const float alpha = expf(m[g] - mn);
      const float p = expf(sv - mn);
      lsum[g] = lsum[g] * alpha + p;
      m[g] = mn;
      pw[g * T + lane] = p;
#pragma unroll
      for (int c = 0; c < CPL; ++c) o[g][c] *= alpha;
    }
    __syncwarp();
#pragma unroll 4
    for (int j = 0; j < T; ++j) {
      float vf[CPL];
      if (CPL == 4) {
        const uint2 vv = *reinterpret_cast<const uint2 *>(vs + j * D + lane * 4);
        const float2 a01 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
        const float2 a23 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
        vf[0] = a01.x;
        vf[1] = a01.y;
        vf[2] = a23.x;
        vf[3] = a23.y;
      } else {
        const float2 a01 = __half22float2(*reinterpret_cast<const __half2 *>(vs + j * D + lane * 2));
        vf[0] = a01.x;
        vf[1] = a01.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float p = pw[g * T + j];
#pragma unroll
        for (int c = 0; c < CPL; ++c) o[g][c] = fmaf(p, vf[c], o[g][c]);
      }
    }
    __syncwarp();
  }
  asm volatile("griddepcontrol.launch_dependents;");

  // ---- merge the 4 warps (reuse the tile buffers) ----
  __syncthreads();
  float *cm = reinterpret_cast<float *>(smraw);  // [W][G]
  float *cl = cm + W * G;                         // [W][G]
  float *co = cl + W * G;                         // [W][G][D]
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float lt = warp_sum(lsum[g]);
    if (lane == 0) {
      cm[warp * G + g] = m[g];
      cl[warp * G + g] = lt;
    }
#pragma unroll
    for (int c = 0; c < CPL; ++c) co[(warp * G + g) * D + lane * CPL + c] = o[g][c];
  }
  __syncthreads();
  const int64_t head_slot = (int64_t)b * a.Hkv + hk;
  for (int idx = tid; idx < G * D; idx += 128) {
    const int g = idx / D, c = idx % D;
    float M = kMaskInit;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, cm[w * G + g]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const float e = expf(cm[w * G + g] - M);
      L += cl[w * G + g] * e;
      O += co[(w * G + g) * D + c] * e;
    }
    if (splits == 1) {
      const int h = hk * G + g;
      a.o[(int64_t)b * a.o_sb + (int64_t)h * a.o_sh + c] = O / fmaxf(L, 1e-12f);
    } else {
      float *pp = part + ((head_slot * splits + split) * G + g) * (D + 2);
      if (c == 0) {
        pp[0] = M;
        pp[1] = L;
      }
      pp[2 + c] = O;
    }
  }
  if (splits == 1) return;

  // ---- last CTA of this head merges all splits ----
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int ticket = atomicAdd(counters + head_slot, 1);
    s_last = ticket == splits - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = tid; idx < G * D; idx += 128) {
    const int g = idx / D, c = idx % D;
    const float *base = part + (head_slot * splits * G + g) * (D + 2);
    const int64_t stride = (int64_t)G * (D + 2);
    float M = kMaskInit;
    for (int sp = 0; sp < splits; ++sp) M = fmaxf(M, __ldcg(base + sp * stride));
    float L = 0.0f, O = 0.0f;
    for (int sp = 0; sp < splits; ++sp) {
      const float e = expf(__ldcg(base + sp * stride) - M);
      L += __ldcg(base + sp * stride + 1) * e;
      O += __ldcg(base + sp * stride + 2 + c) * e;
    }
    const int h = hk * G + g;
    a.o[(int64_t)b * a.o_sb + (int64_t)h * a.o_sh + c] = O / fmaxf(L, 1e-12f);
  }
  if (tid == 0) counters[head_slot] = 0;  // ready for the next launch
}

template <int D, int BQ>
void launch_simt_t(const AttnArgs &a, cudaStream_t s) {
  const size_t smem = (size_t)(BQ * (D + 4) + 2 * 32 * (D + 4) + BQ * 33) * sizeof(float);
  static unsigned long long attr_set = 0;
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << dev))) {
    FG_CUDA(cudaFuncSetAttribute(k_attn_simt<D, BQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set |= 1ull << dev;
  }
  dim3 grid((unsigned)ceil_div(a.Nq, BQ), a.H, a.B);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(BQ * 4);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FG_CUDA(cudaLaunchKernelEx(&cfg, k_attn_simt<D, BQ>, a));
}

template <int D, int G>
void launch_decode_t(const AttnArgs &a, int splits, void *scratch, cudaStream_t s) {
  const size_t smem =
      (size_t)4 * kDecodeStages * 2 * 32 * D * sizeof(__half) + (size_t)(G * D + 4 * G * 32) * sizeof(float);
  static unsigned long long attr_set = 0;
  int dev = 0;
  FG_CUDA(cudaGetDevice(&dev));
  if (!(attr_set & (1ull << dev))) {
    FG_CUDA(cudaFuncSetAttribute(k_attn_decode<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set |= 1ull << dev;
  }
  float *part = nullptr;
  int *counters = nullptr;
  if (splits > 1) {
    const int sb = a.scratch_batch > 0 ? a.scratch_batch : a.B;
    FG_REQUIRE(a.B <= sb && scratch, FG_ERR_VALIDATION, "decode attention: scratch too small");
    counters = (int *)scratch;
    part = (float *)((char *)scratch + align_up((uint64_t)sb * a.Hkv * sizeof(int), 256));
  }
  dim3 grid(splits, a.Hkv, a.B);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FG_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<D, G>, a, splits, part, counters));
}

template <int D>
void launch_decode_d(const AttnArgs &a, int splits, void *scratch, cudaStream_t s) {
  switch (a.H / a.Hkv) {
    case 1: launch_decode_t<D, 1>(a, splits, scratch, s); break;
    case 2: launch_decode_t<D, 2>(a, splits, scratch, s); break;
    case 4: launch_decode_t<D, 4>(a, splits, scratch, s); break;
    case 8: launch_decode_t<D, 8>(a, splits, scratch, s); break;
    default: raise(FG_ERR_SHAPE, "decode attention: GQA group %d not in {1,2,4,8}", a.H / a.Hkv);
  }
}

}  // namespace

void launch_attention(const AttnArgs &a, int num_sms, cudaStream_t s) {
  (void)num_sms;
  FG_REQUIRE(a.d >= 1 && a.d <= 256, FG_ERR_SHAPE, "HeadDim %d exceeds max supported dimension 256", a.d);
  FG_REQUIRE(a.H % a.Hkv == 0, FG_ERR_SHAPE, "Query heads %d must be divisible by KV heads %d", a.H, a.Hkv);
  if (a.B == 0 || a.Nq == 0 || a.H == 0) return;
  if (a.Nq >= 16 && attn_tc_supported(a)) {  // prefill: tensor cores (fewer query rows use the SIMT tile)
    launch_attention_tc(a, s);
    return;
  }
  if (a.d <= 64)
    launch_simt_t<64, 32>(a, s);
  else if (a.d <= 128)
    launch_simt_t<128, 32>(a, s);
  else
    launch_simt_t<256, 16>(a, s);
}

bool attn_decode_supported(const AttnArgs &a) {
  const int g = a.Hkv > 0 ? a.H / a.Hkv : 0;
  return a.Nq == 1 && a.kv_f16 && !a.q_f16 && (a.d == 64 || a.d == 128) && (g == 1 || g == 2 || g == 4 || g == 8);
}

int attn_decode_splits(const AttnArgs &a, int max_kv, int num_sms, uint64_t max_scratch) {
  const int64_t heads = (int64_t)a.B * a.Hkv;
  const int G = a.H / a.Hkv;
  // resident CTAs per SM from k_attn_decode's shared memory (+ 1 KB the runtime reserves per CTA)
  const int64_t smem = (int64_t)4 * kDecodeStages * 2 * 32 * a.d * 2 + (int64_t)(G * a.d + 4 * G * 32) * 4 + 1024;
  const int64_t slots = (int64_t)std::max(1, num_sms) * std::max<int64_t>(1, std::min<int64_t>(16, 233472 / smem));
  // cost of s splits: waves of equal CTAs x (keys per split + ~64 keys of per-CTA latency); at least 128
  // keys per split
  const int cap = (int)std::max<int64_t>(1, ceil_div(max_kv, 128));
  int best = 1;
  double best_cost = 0.0;
  for (int sp = 1; sp <= cap; ++sp) {
    if (sp > 1 && attn_decode_scratch_bytes(a, sp) > max_scratch) break;
    const double cost = (double)ceil_div(heads * sp, slots) * (double)(ceil_div(max_kv, sp) + 64);
    if (sp == 1 || cost < best_cost) {
      best = sp;
      best_cost = cost;
    }
  }
  return best;
}

uint64_t attn_decode_scratch_bytes(const AttnArgs &a, int splits) {
  const int G = a.H / a.Hkv;
  if (splits <= 1) return 0;
  const int sb = a.scratch_batch > 0 ? a.scratch_batch : a.B;
  return align_up((uint64_t)sb * a.Hkv * sizeof(int), 256) +
         (uint64_t)sb * a.Hkv * splits * G * (a.d + 2) * sizeof(float);
}

void launch_attention_decode(const AttnArgs &a, int splits, void *scratch, cudaStream_t s) {
  FG_REQUIRE(attn_decode_supported(a), FG_ERR_SHAPE, "decode attention: unsupported shape");
  if (a.d == 64)
    launch_decode_d<64>(a, splits, scratch, s);
  else
    launch_decode_d<128>(a, splits, scratch, s);
}

}  // namespace fg
