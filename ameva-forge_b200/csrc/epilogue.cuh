// Fused epilogues of the quantized GEMV / GEMM kernels.  Row n of W gives
// output column n for token m; rows come in adjacent pairs (2i, 2i+1) so a
// RoPE pair or a (gate, up) pair is finished by the thread holding both.
#pragma once
#include "runtime.cuh"

namespace fg {

// Interleaved-pair RoPE of one (v0, v1) pair: rope.wgsl.ts:45-59 (theta in fp32).
__device__ inline float rope_theta(float inv_freq, int pos) { return __fmul_rn(inv_freq, (float)pos); }
__device__ inline void rope_rot(float v0, float v1, float c, float s, float &o0, float &o1) {
  o0 = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
  o1 = __fadd_rn(__fmul_rn(v1, c), __fmul_rn(v0, s));
}
__device__ inline void rope_pair(float v0, float v1, float inv_freq, int pos, float &o0, float &o1) {
  float s, c;
  sincosf(rope_theta(inv_freq, pos), &s, &c);
  rope_rot(v0, v1, c, s, o0, o1);
}
// RoPE of frequency i: from the epilogue's table when it has one (same theta, same sincosf).
__device__ inline void rope_pair_ep(const Epilogue &ep, float v0, float v1, int i, int pos, float &o0, float &o1) {
  if (ep.rope_cs)
    rope_rot(v0, v1, ep.rope_cs[i], ep.rope_cs[(ep.head_dim >> 1) + i], o0, o1);
  else
    rope_pair(v0, v1, ep.inv_freq[i], pos, o0, o1);
}

// SwiGLU: swiglu.wgsl.ts:38-40, gate / (1 + exp(-gate)) * up.
__device__ inline float swiglu1(float g, float u) { return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u); }

// Store a finished pair of columns (n even, n+1) for token m.
// XCHG (tensor-parallel o_proj / down_proj partial sums): the value of column n to every rank's
// slot, a peer store over NVLink for the other ranks.  Only kernels instantiated for tensor
// parallelism reach it (finish_strip<MV, true>).
__device__ inline void epi_xchg_one(const Epilogue &ep, int64_t n, int m, float v) {
  for (int r = 0; r < ep.nx; ++r) ep.xdst[r][ep.xoff + (int64_t)m * ep.ldy + n] = v;
}
__device__ inline void epi_xchg_pair(const Epilogue &ep, int64_t n, int m, float v0, float v1) {
  for (int r = 0; r < ep.nx; ++r) {
    float *y = ep.xdst[r] + ep.xoff + (int64_t)m * ep.ldy + n;
    y[0] = v0;
    y[1] = v1;
  }
}

__device__ inline void epi_store_pair(const Epilogue &ep, int64_t n, int m, float v0, float v1) {
  if (ep.mode == EPI_PLAIN) {
    float *y = ep.y + (int64_t)m * ep.ldy + n;
    if (ep.resid) {  // read through L2: other SMs of a persistent kernel may have written it
      const float *r = ep.resid + (int64_t)m * ep.ldy + n;
      v0 = __fadd_rn(__ldcg(r), v0);
      v1 = __fadd_rn(__ldcg(r + 1), v1);
    }
    y[0] = v0;
    y[1] = v1;
  } else if (ep.mode == EPI_SWIGLU) {
    ep.y[(int64_t)m * ep.ldy + (n >> 1)] = swiglu1(v0, v1);
  } else {  // EPI_QKV
    const int d = ep.head_dim;
    const int b = m / ep.tokens_per_seq;
    const int pos = ep.rope_cs ? ep.pos0 : ep.pos[b] + (m - b * ep.tokens_per_seq);
    if (n < ep.n_q) {
      float o0, o1;
      rope_pair_ep(ep, v0, v1, (int)((n % d) >> 1), pos, o0, o1);
      float *q = ep.q_out + (int64_t)m * ep.n_q + n;
      q[0] = o0;
      q[1] = o1;
    } else {
      const int64_t nk = n - ep.n_q;
      const bool is_v = nk >= ep.n_kv;
      const int64_t nn = is_v ? nk - ep.n_kv : nk;
      const int hkv = ep.n_kv / d;
      const int64_t hk = nn / d, c = nn % d;
      const int64_t idx = (((int64_t)b * hkv + hk) * ep.cap + pos) * d + c;
      if (is_v) {
        *reinterpret_cast<__half2 *>(ep.v_cache + idx) = __halves2half2(__float2half_rn(v0), __float2half_rn(v1));
      } else {
        float o0, o1;
        rope_pair_ep(ep, v0, v1, (int)(c >> 1), pos, o0, o1);
        *reinterpret_cast<__half2 *>(ep.k_cache + idx) = __halves2half2(__float2half_rn(o0), __float2half_rn(o1));
      }
    }
  }
}

// Single column (PLAIN only; used when a kernel's row group is odd-sized).
__device__ inline void epi_store_one(const Epilogue &ep, int64_t n, int m, float v) {
  float *y = ep.y + (int64_t)m * ep.ldy + n;
  if (ep.resid) v = __fadd_rn(__ldcg(ep.resid + (int64_t)m * ep.ldy + n), v);
  *y = v;
}

// Four consecutive columns n..n+3 (n even) of token m, of a matrix with N
// columns: one 16-byte store where the row allows it, else two pairs (and a
// single column at an odd end, PLAIN only).
__device__ inline void epi_store_quad(const Epilogue &ep, int64_t n, int64_t N, int m, float4 v) {
  if (ep.mode == EPI_PLAIN && n + 3 < N) {
    float *y = ep.y + (int64_t)m * ep.ldy + n;
    const float *r = ep.resid ? ep.resid + (int64_t)m * ep.ldy + n : nullptr;
    if ((((uintptr_t)y | (uintptr_t)r) & 15) == 0) {
      if (r) {
        const float4 a = __ldcg(reinterpret_cast<const float4 *>(r));
        v = make_float4(__fadd_rn(a.x, v.x), __fadd_rn(a.y, v.y), __fadd_rn(a.z, v.z), __fadd_rn(a.w, v.w));
      }
      *reinterpret_cast<float4 *>(y) = v;
      return;
    }
  }
  const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; k += 2) {
    if (n + k + 1 < N)
      epi_store_pair(ep, n + k, m, e[k], e[k + 1]);
    else if (n + k < N && ep.mode == EPI_PLAIN)
      epi_store_one(ep, n + k, m, e[k]);
  }
}

}  // namespace fg
