// On-device token sampler with the semantics of LLMSampler.sample
// (packages/forge/src/tensor/sampling.ts:35-128):
//   temperature <= 1e-5            -> first maximum (greedy, :45-55)
//   K = top_k if 0 < top_k < V else V
//   K < V and K <= 128             -> partial selection sort with swaps (:62-76):
//                                     K passes, each takes the first maximum of
//                                     positions [i, V) and swaps it to i (ties are
//                                     ordered as those swaps leave them)
//   otherwise                      -> stable sort by value, descending (:78-80)
//   p_i = exp(l_i / T - l_0 / T) in double, stored as float32, normalised by
//   1 / max(sum, 1e-12) (:82-96); top-p keeps the shortest prefix whose
//   cumulative probability reaches top_p (:98-109); the pick is the first
//   candidate whose cumulative renormalised probability reaches r (:113-124),
//   r = the first Xorshift32 output of the seed / 2^32 (:20-28; each call
//   seeds a fresh generator).
// One CTA of 1024 threads per row.  The sums run over per-thread chunks in a
// fixed order (deterministic; they may round differently from a strictly
// sequential sum, in the last bits of a double).
#include <random>

#include "runtime.cuh"

namespace fg {
namespace {

constexpr int kSampThreads = 1024;

struct SampleOpts {
  double temperature, top_p;
  int top_k;
  uint32_t seed;
};

__device__ __forceinline__ uint32_t ord_bits(float v) {  // ascending unsigned order of the float; NaN lowest
  if (v != v) return 0u;
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Block-wide max of a 64-bit key (all threads get it).
__device__ unsigned long long block_max_u64(unsigned long long v, unsigned long long *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kSampThreads / 32 ? red[lane] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
      v = w > v ? w : v;
    }
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// Block-wide sum of doubles over threads in thread order (fixed tree: deterministic).
__device__ double block_sum_f64(double v, double *red) {
  __syncthreads();
  red[threadIdx.x] = v;
  __syncthreads();
  for (int s = kSampThreads / 2; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  return red[0];
}

// Exclusive prefix of per-thread values, in thread order (thread 0 scans).
__device__ double block_excl_f64(double v, double *red) {
  __syncthreads();
  red[threadIdx.x] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double run = 0.0;
    for (int t = 0; t < kSampThreads; ++t) {
      const double x = red[t];
      red[t] = run;
      run += x;
    }
  }
  __syncthreads();
  return red[threadIdx.x];
}

// Block-wide min of an int (all threads get it).
__device__ int block_min_i32(int v, int *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < kSampThreads / 32 ? red[threadIdx.x] : INT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// keys: [rows][np2] u64 scratch (the sorted candidate order), cand: [rows][V] f32 scratch.
__global__ void __launch_bounds__(kSampThreads) k_sample(const float *__restrict__ logits, int V, int64_t ld,
                                                          SampleOpts o, int np2, unsigned long long *__restrict__ keys,
                                                          float *__restrict__ cand, int32_t *__restrict__ out) {
  __shared__ unsigned long long s_u64[32];
  __shared__ double s_f64[kSampThreads];
  __shared__ int s_i32[32];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.x, tid = threadIdx.x;
  const float *l = logits + (int64_t)row * ld;
  unsigned long long *key = keys + (int64_t)row * np2;
  float *cp = cand + (int64_t)row * V;

  if (o.temperature <= 1e-5) {  // greedy: the first maximum; a NaN at index 0 keeps index 0
    unsigned long long best = 0;
    for (int j = tid; j < V; j += kSampThreads) {
      const float v = l[j];
      const unsigned long long k =
          v != v ? (j == 0 ? ~0ull : 0ull) : ((unsigned long long)ord_bits(v) << 32) | (0xFFFFFFFFull - (unsigned)j);
      best = k > best ? k : best;
    }
    best = block_max_u64(best, s_u64);
    if (tid == 0) out[row] = (int32_t)(0xFFFFFFFFull - (best & 0xFFFFFFFFull));
    return;
  }

  const int K = (o.top_k > 0 && o.top_k < V) ? o.top_k : V;
  if (K < V && K <= 128) {
    // the reference's partial selection sort: position order in the low word of key[]
    for (int j = tid; j < V; j += kSampThreads) key[j] = (unsigned)j;
    __syncthreads();
    for (int i = 0; i < K; ++i) {
      unsigned long long best = 0;
      for (int p = i + tid; p < V; p += kSampThreads) {
        const float v = l[(uint32_t)key[p]];
        const unsigned long long k = ((unsigned long long)ord_bits(v) << 32) | (0xFFFFFFFFull - (unsigned)p);
        best = k > best ? k : best;
      }
      best = block_max_u64(best, s_u64);
      if (tid == 0) {
        int mp = (int)(0xFFFFFFFFull - (best & 0xFFFFFFFFull));
        if (l[(uint32_t)key[i]] != l[(uint32_t)key[i]]) mp = i;  // a NaN at position i is kept (nothing is > NaN)
        const unsigned long long t = key[i];
        key[i] = key[mp];
        key[mp] = t;
      }
      __syncthreads();
    }
  } else {
    // stable descending sort: ascending order of (descending value, ascending index) keys
    for (int j = tid; j < np2; j += kSampThreads)
      key[j] = j < V ? ((unsigned long long)(0xFFFFFFFFu - ord_bits(l[j])) << 32) | (unsigned)j : ~0ull;
    __syncthreads();
    for (int k = 2; k <= np2; k <<= 1) {
      for (int jj = k >> 1; jj > 0; jj >>= 1) {
        for (int i = tid; i < np2; i += kSampThreads) {
          const int p = i ^ jj;
          if (p > i) {
            const unsigned long long a = key[i], b = key[p];
            const bool up = (i & k) == 0;
            if ((a > b) == up) {
              key[i] = b;
              key[p] = a;
            }
          }
        }
        __syncthreads();
      }
    }
  }
  // candidates 0..K-1 of the sorted order: this thread's chunk [c0, c1)
  const int chunk = (K + kSampThreads - 1) / kSampThreads;
  const int c0 = min(K, tid * chunk), c1 = min(K, c0 + chunk);
  const double T = o.temperature;
  const double mx = (double)l[(uint32_t)key[0]] / T;
  double s = 0.0;
  for (int i = c0; i < c1; ++i) {
    const double p = exp((double)l[(uint32_t)key[i]] / T - mx);
    cp[i] = (float)p;
    s += p;
  }
  const double inv = 1.0 / fmax(block_sum_f64(s, s_f64), 1e-12);
  for (int i = c0; i < c1; ++i) cp[i] = (float)((double)cp[i] * inv);
  // top-p: the shortest prefix whose cumulative probability reaches top_p
  int cutoff = K;
  if (o.top_p < 1.0) {
    double cs = 0.0;
    for (int i = c0; i < c1; ++i) cs += (double)cp[i];
    double run = block_excl_f64(cs, s_f64);
    int mine = INT_MAX;
    for (int i = c0; i < c1; ++i) {
      run += (double)cp[i];
      if (run >= o.top_p) {
        mine = i + 1;
        break;
      }
    }
    cutoff = min(K, block_min_i32(mine, s_i32));
  }
  double fs = 0.0;
  for (int i = c0; i < min(c1, cutoff); ++i) fs += (double)cp[i];
  const double invf = 1.0 / fmax(block_sum_f64(fs, s_f64), 1e-12);
  // r = the first Xorshift32 output of the seed
  uint32_t x = o.seed ? o.seed : 1u;
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  const double r = (double)x / 4294967296.0;
  double as = 0.0;
  for (int i = c0; i < min(c1, cutoff); ++i) as += (double)cp[i] * invf;
  double acc = block_excl_f64(as, s_f64);
  int pick = INT_MAX;
  for (int i = c0; i < min(c1, cutoff); ++i) {
    acc += (double)cp[i] * invf;
    if (r <= acc) {
      pick = i;
      break;
    }
  }
  pick = block_min_i32(pick, s_i32);
  if (tid == 0) out[row] = (int32_t)(uint32_t)key[pick == INT_MAX ? cutoff - 1 : pick];
}

}  // namespace

uint64_t sample_scratch_bytes(int64_t rows, int64_t V) {
  int64_t np2 = 1;
  while (np2 < V) np2 <<= 1;
  return (uint64_t)rows * (np2 * 8 + align_up((uint64_t)V * 4, 256));
}

void launch_sample(const float *logits, int64_t rows, int64_t V, int64_t ld, double temperature, int top_k,
                   double top_p, bool has_seed, uint32_t seed, void *scratch, int32_t *out, cudaStream_t s) {
  FG_REQUIRE(V > 0 && V < (1ll << 30), FG_ERR_VALIDATION, "Logits array cannot be empty");
  if (rows == 0) return;
  if (!has_seed) {  // the reference draws from Math.random without a seed
    std::random_device rd;
    seed = rd();
  }
  int np2 = 1;
  while (np2 < V) np2 <<= 1;
  SampleOpts o{temperature, top_p, top_k, seed};
  unsigned long long *keys = (unsigned long long *)scratch;
  float *cand = (float *)((char *)scratch + (uint64_t)rows * np2 * 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)rows);
  cfg.blockDim = dim3(kSampThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FG_CUDA(cudaLaunchKernelEx(&cfg, k_sample, logits, (int)V, ld, o, np2, keys, cand, out));
}

}  // namespace fg
