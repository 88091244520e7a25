// Standalone elementwise / row kernels of the op API: RMSNorm, RoPE, SwiGLU,
// embedding gather, residual add, greedy argmax, dtype casts.  All are HBM-
// bound and small next to the quantized GEMV; inside the Llama step most are
// fused into the GEMV prologue/epilogue instead (epilogue.cuh).
#include "epilogue.cuh"

namespace fg {
namespace {

inline int grid_for(int64_t n, int per_block = 256) { return (int)std::min<int64_t>(ceil_div(n, per_block), 148 * 32); }

// RMSNORM_WGSL (packages/forge/src/tensor/kernels/rmsnorm.wgsl.ts:10-74): one
// CTA per token; inv_rms = 1 / sqrt(mean(x^2) + eps); out = x * inv_rms * gamma.
__global__ void __launch_bounds__(256) k_rmsnorm(const float *__restrict__ x, int64_t ldx,
                                                 const float *__restrict__ gamma, float eps, int64_t dim,
                                                 float *__restrict__ out) {
  __shared__ float red[8];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float *row = x + blockIdx.x * ldx;
  float ss = 0.0f;
  for (int64_t i = threadIdx.x; i < dim; i += 256) ss += row[i] * row[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)dim), eps)));
  float *orow = out + blockIdx.x * dim;
  for (int64_t i = threadIdx.x; i < dim; i += 256) {
    float v = __fmul_rn(row[i], inv);
    if (gamma) v = __fmul_rn(v, gamma[i]);
    orow[i] = v;
  }
}

// ROPE_WGSL (rope.wgsl.ts:11-62): interleaved pair p of row (b, h, n) rotated
// by theta = inv_freq[p] * (n + offset).  One thread per pair.
__global__ void k_rope(const float *__restrict__ x, int64_t rows, int64_t N, int64_t d,
                       const float *__restrict__ inv_freq, int64_t offset, float *__restrict__ out) {
  const int64_t half = d / 2;
  const int64_t total = rows * N * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i % half;
    const int64_t tok = i / half;  // (row, n)
    const int64_t n = tok % N;
    const float2 v = *reinterpret_cast<const float2 *>(x + tok * d + 2 * p);
    float o0, o1;
    rope_pair(v.x, v.y, inv_freq[p], (int)(n + offset), o0, o1);
    *reinterpret_cast<float2 *>(out + tok * d + 2 * p) = make_float2(o0, o1);
  }
}

__global__ void k_swiglu(const float *__restrict__ g, const float *__restrict__ u, int64_t n,
                         float *__restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = swiglu1(g[i], u[i]);
}

// EMBEDDING_WGSL (embedding.wgsl.ts:20-63): one CTA per token; an id that is
// NaN (f32 ids), negative or >= vocab yields a zero row.
__global__ void k_embedding(const void *__restrict__ table, int f16, int64_t vocab, int64_t dim,
                            const void *__restrict__ ids, int ids_f32, float *__restrict__ out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t t = blockIdx.x;
  int64_t id = -1;
  if (ids_f32) {
    const float raw = reinterpret_cast<const float *>(ids)[t];
    const float rd = rintf(raw);  // WGSL round(): half to even
    if (raw == raw && rd >= 0.0f && rd < (float)vocab) id = (int64_t)rd;
  } else {
    const int32_t raw = reinterpret_cast<const int32_t *>(ids)[t];
    if (raw >= 0 && raw < vocab) id = raw;
  }
  float *o = out + t * dim;
  for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) {
    float v = 0.0f;
    if (id >= 0)
      v = f16 ? __half2float(reinterpret_cast<const __half *>(table)[id * dim + c])
              : reinterpret_cast<const float *>(table)[id * dim + c];
    o[c] = v;
  }
}

__global__ void k_add(const float *__restrict__ a, const float *__restrict__ b, int64_t n, float *__restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __fadd_rn(a[i], b[i]);
}

// Greedy pick with the sampler's rule (sampling.ts:45-55): start at index 0
// and take i only if logits[i] > best, so ties keep the lowest index and NaN
// entries never win (a NaN at index 0 keeps index 0, as the reference does).
struct Best {
  float v;
  int64_t i;
};
__device__ inline Best better(Best a, Best b) {
  // a and b cover disjoint index ranges; prefer the strictly larger value,
  // on ties the lower index; NaN never compares larger.
  if (b.v > a.v || (b.v == a.v && b.i < a.i) || (a.v != a.v && b.i < a.i)) return b;
  return a;
}

__global__ void __launch_bounds__(256) k_argmax(const float *__restrict__ logits, int64_t n, int64_t ld,
                                                int64_t index_base, int32_t *__restrict__ out,
                                                unsigned long long *__restrict__ keys) {
  __shared__ float sv[8];
  __shared__ long long si[8];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float *row = logits + blockIdx.x * ld;
  const bool nan0 = index_base == 0 && row[0] != row[0];  // only global index 0 is special
  Best best{-INFINITY, n};
  for (int64_t i = threadIdx.x; i < n; i += 256) {
    const float v = row[i];
    if (v > best.v || (v == best.v && i < best.i)) best = Best{v, i};
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best other{__shfl_xor_sync(0xffffffffu, best.v, o), (int64_t)__shfl_xor_sync(0xffffffffu, (long long)best.i, o)};
    best = better(best, other);
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best.v;
    si[threadIdx.x >> 5] = best.i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    Best b{sv[0], si[0]};
    for (int w = 1; w < 8; ++w) b = better(b, Best{sv[w], si[w]});
    if (nan0 || b.i >= n) b = Best{nan0 ? INFINITY : -INFINITY, 0};
    if (out) out[blockIdx.x] = (int32_t)(b.i + index_base);
    if (keys) {
      // order by value (monotone map of the float bits), then by lower index
      uint32_t bits = __float_as_uint(b.v);
      bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
      keys[blockIdx.x] = ((unsigned long long)bits << 32) | (0xFFFFFFFFull - (unsigned long long)(b.i + index_base));
    }
  }
}

__global__ void k_keys_to_ids(const unsigned long long *__restrict__ keys, int64_t rows, int32_t *__restrict__ ids) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x)
    ids[r] = (int32_t)(0xFFFFFFFFull - (keys[r] & 0xFFFFFFFFull));
}

__global__ void k_cast(const void *__restrict__ in, int in_f16, void *__restrict__ out, int out_f16, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = in_f16 ? __half2float(reinterpret_cast<const __half *>(in)[i]) : reinterpret_cast<const float *>(in)[i];
    if (out_f16)
      reinterpret_cast<__half *>(out)[i] = __float2half_rn(v);
    else
      reinterpret_cast<float *>(out)[i] = v;
  }
}

__global__ void k_check_finite(const float *__restrict__ x, int64_t n, int *__restrict__ flag) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    if (!isfinite(x[i])) {
      *flag = 1;
      return;
    }
}

// End of a decode step: every sequence advanced by `by` positions; the step's
// greedy ids are logged for device-resident generation.
__global__ void k_advance_pos(int *pos, int batch, int by, int32_t *log, const int32_t *ids, int *step,
                              int log_steps) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = threadIdx.x;
  if (b < batch) {
    if (log) {
      const int st = *step;
      if (st < log_steps) log[(int64_t)st * batch + b] = ids[b];
    }
    pos[b] += by;
  }
  __syncthreads();
  if (b == 0 && log) *step += 1;
}

}  // namespace

void launch_advance_pos(int *pos, int batch, int by, int32_t *log, const int32_t *ids, int *step, int log_steps,
                        cudaStream_t s) {
  k_advance_pos<<<1, ((batch + 31) / 32) * 32, 0, s>>>(pos, batch, by, log, ids, step, log_steps);
  FG_LAUNCH_CHECK();
}

void launch_rmsnorm(const float *x, int64_t ldx, const float *gamma, float eps, int64_t tokens, int64_t dim,
                    float *out, cudaStream_t s) {
  if (tokens == 0) return;
  k_rmsnorm<<<(unsigned)tokens, 256, 0, s>>>(x, ldx, gamma, eps, dim, out);
  FG_LAUNCH_CHECK();
}

void launch_rope(const float *x, int64_t rows, int64_t N, int64_t d, const float *inv_freq, int64_t offset,
                 float *out, cudaStream_t s) {
  const int64_t total = rows * N * (d / 2);
  if (total == 0) return;
  k_rope<<<grid_for(total), 256, 0, s>>>(x, rows, N, d, inv_freq, offset, out);
  FG_LAUNCH_CHECK();
}

void launch_swiglu(const float *g, const float *u, int64_t n, float *out, cudaStream_t s) {
  if (n == 0) return;
  k_swiglu<<<grid_for(n), 256, 0, s>>>(g, u, n, out);
  FG_LAUNCH_CHECK();
}

void launch_embedding(const void *table, int table_f16, int64_t vocab, int64_t dim, const void *ids, int ids_f32,
                      int64_t n, float *out, cudaStream_t s) {
  if (n == 0) return;
  k_embedding<<<(unsigned)n, 256, 0, s>>>(table, table_f16, vocab, dim, ids, ids_f32, out);
  FG_LAUNCH_CHECK();
}

void launch_add(const float *a, const float *b, int64_t n, float *out, cudaStream_t s) {
  if (n == 0) return;
  k_add<<<grid_for(n), 256, 0, s>>>(a, b, n, out);
  FG_LAUNCH_CHECK();
}

void launch_argmax(const float *logits, int64_t rows, int64_t n, int64_t ld, int32_t *out, cudaStream_t s) {
  if (rows == 0) return;
  k_argmax<<<(unsigned)rows, 256, 0, s>>>(logits, n, ld, 0, out, nullptr);
  FG_LAUNCH_CHECK();
}

void launch_argmax_keys(const float *logits, int64_t rows, int64_t n, int64_t ld, int64_t index_base,
                        unsigned long long *keys, cudaStream_t s) {
  if (rows == 0) return;
  k_argmax<<<(unsigned)rows, 256, 0, s>>>(logits, n, ld, index_base, nullptr, keys);
  FG_LAUNCH_CHECK();
}

void launch_keys_to_ids(const unsigned long long *keys, int64_t rows, int32_t *ids, cudaStream_t s) {
  if (rows == 0) return;
  k_keys_to_ids<<<1, 256, 0, s>>>(keys, rows, ids);
  FG_LAUNCH_CHECK();
}

void launch_cast(const void *in, int in_dtype, void *out, int out_dtype, int64_t n, cudaStream_t s) {
  if (n == 0) return;
  k_cast<<<grid_for(n), 256, 0, s>>>(in, in_dtype == FG_F16, out, out_dtype == FG_F16, n);
  FG_LAUNCH_CHECK();
}

void launch_check_finite(const float *x, int64_t n, int *flag, cudaStream_t s) {
  if (n == 0) return;
  k_check_finite<<<grid_for(n), 256, 0, s>>>(x, n, flag);
  FG_LAUNCH_CHECK();
}

}  // namespace fg
