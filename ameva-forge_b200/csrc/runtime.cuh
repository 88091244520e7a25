// Context, tensor registry, allocator and kernel launcher declarations.
#pragma once

#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "common.cuh"

struct ncclComm;

namespace fg {

struct Ctx;

// A float32 [B, H, cap, d] buffer of the graph front-end's key/value tensors: the first `tip`
// positions of every (b, h) are written; tensors over it see their first `len` positions.  An
// append to the tensor whose len == tip writes in place (the reference re-concatenates the
// whole cache every step).  Freed through the context when the last tensor over it goes.
struct KVStore {
  Ctx *ctx = nullptr;
  float *ptr = nullptr;
  uint64_t bytes = 0;
  int64_t B = 0, H = 0, cap = 0, d = 0, tip = 0;
  ~KVStore();
};

// A tensor of the graph front-end that is not materialised yet: its value is a pure function of the
// tensor `src` (kept readable by the context: disposing `src` first materialises its lazy users),
// or of a key/value store.
struct LazyView {
  enum Kind { T2D = 1, HEADS = 2, KVCAP = 3 } kind = T2D;
  uint64_t src = 0;            // handle of the source tensor (T2D, HEADS)
  std::vector<int32_t> heads;  // HEADS: head j of this [B, H, S, d] tensor is head heads[j] of src
  std::shared_ptr<KVStore> store;  // KVCAP: this tensor is positions [0, len) of the store
  int64_t len = 0;
};

struct Tensor {
  std::shared_ptr<LazyView> lazy;  // set: ptr is null until the first get()
  void *ptr = nullptr;
  uint64_t bytes = 0;
  int32_t dtype = FG_F32;
  int32_t ndim = 0;
  int64_t shape[FG_MAX_DIMS] = {0};
  int64_t numel() const {
    int64_t n = 1;
    for (int i = 0; i < ndim; ++i) n *= shape[i];
    return n;
  }
  QMat qmat() const {  // valid for FG_Q4_0 / FG_Q8_0 tensors of shape [N, K]
    return qmat_at(ptr, dtype, shape[0], shape[1]);
  }
};

// Workspace of the stream-K GEMV (gemv.cu): partial sums of row groups cut
// between CTAs, arrival tickets (zero between launches) and the device error
// word that bounded waits write on timeout.
struct GemvScratch {
  float *part = nullptr;
  uint64_t part_floats = 0;
  int *tickets = nullptr;
  int64_t n_tickets = 0;
  int *err = nullptr;
  int maxc = 1;
  __half *xh = nullptr;  // fp16 copy of a GEMM's activations (tensor-core GEMM B operand)
  uint64_t xh_elems = 0;
};

// Graph limits of configureRuntime (graphExecutor.ts:98-116, defaults as there).
struct GraphLimits {
  int64_t max_instructions = 10000;
  int max_shape_dim = 8;
  int64_t max_elements = 256ll * 1024 * 1024;
};

// One context = one device, one stream, one handle namespace (the reference's
// _globalRegistry + QuotaManager + device singleton, per GPU).
struct Ctx {
  int device = 0;
  int tp_rank = 0, tp_size = 1;
  cudaStream_t stream = nullptr;
  cudaMemPool_t pool = nullptr;
  ncclComm *nccl = nullptr;
  std::recursive_mutex mu;
  std::unordered_map<uint64_t, Tensor> tensors;
  uint64_t next_id = 1;
  uint64_t epoch = 1;  // bumped on context loss; handles of an old epoch are stale
  uint64_t limit = 0, active = 0, pending = 0, peak = 0;
  bool allow_non_finite = false;
  GraphLimits graph;
  bool lost = false;
  // Pinned staging ring for host <-> device copies (buffers.ts:70-140 keeps a
  // pow-2 staging pool; here two pinned halves alternate so the host copy of
  // one chunk overlaps the DMA of the other).
  void *staging[2] = {nullptr, nullptr};
  cudaEvent_t staging_ev[2] = {nullptr, nullptr};
  uint64_t staging_bytes = 0;
  int num_sms = 148;
  GemvScratch gemv;  // allocated at init, shared by every GEMV launch of the stream

  // allocation with quota accounting (quota.ts:65-313)
  void *alloc(uint64_t bytes);
  void free_async(void *p, uint64_t bytes);
  fg_handle add(const Tensor &t);
  Tensor &get(fg_handle h);   // materialises a lazy tensor
  Tensor &peek(fg_handle h);  // the registry entry as it is (graph front-end)
  void materialize(fg_handle h, Tensor &t);  // graph.cu
  std::unordered_multimap<uint64_t, uint64_t> lazy_users;  // source handle -> lazy tensors reading it
  fg_handle make(const int64_t *shape, int ndim, int dtype, Tensor **out = nullptr);
  void dispose(fg_handle h);
  void h2d(void *dst, const void *src, uint64_t bytes);
  void d2h(void *dst, const void *src, uint64_t bytes);
  void sync();
  void check_device_error();  // raises if a kernel's bounded wait timed out
  // d2h of a small result and the device error word in one stream synchronisation, then check_device_error's
  // test on the word (falls back to the two steps when the result does not fit the staging buffer)
  void d2h_checked(void *dst, const void *src, uint64_t bytes);
  void ensure_xh(uint64_t elems);  // grow gemv.xh (never during stream capture)
};

uint64_t dtype_bytes(int dtype, int64_t numel, const int64_t *shape, int ndim);

// ------------------------------------------------------------------ launchers
// quant.cu
void launch_unpack_quant(const uint32_t *packed, const float *scales, const float *zeros, int bits, int64_t gs,
                         int64_t n, float *out, cudaStream_t s);
// GGUF blocks of an [N, K] matrix into rows r * dst_rs + dst_ro of dst.
void launch_gguf_to_device(const uint8_t *blocks, int qtype, int64_t N, int64_t K, const QMat &dst, int64_t dst_rs,
                           int64_t dst_ro, cudaStream_t s);
void launch_device_to_gguf(const QMat &w, uint8_t *blocks, cudaStream_t s);
void launch_dequant(const QMat &w, float *out, cudaStream_t s);
// q4k.cu: GGUF Q4_K / Q6_K (blocks in GGUF order, [N][K / 256] x 144 / 210 bytes)
void launch_dequant_q4k(const void *blocks, int64_t n_blocks, float *out, cudaStream_t s);
void launch_qmatmul_q4k(const void *w, int64_t N, int64_t K, const float *x, int64_t M, float *y, float *scratch,
                        int *err, cudaStream_t s);
void launch_dequant_q6k(const void *blocks, int64_t n_blocks, float *out, cudaStream_t s);
void launch_qmatmul_q6k(const void *w, int64_t N, int64_t K, const float *x, int64_t M, float *y, float *scratch,
                        cudaStream_t s);
// Epilogue pass over k-quant GEMV outputs (q4k.cu): mode 0 = QKV from s0 (q, n0 columns), s1 (k, n1),
// s2 (v, n1); mode 1 = pair p from (s0[m][p], s1[m][p]) (gate, up); mode 2 = the columns of s0.
// npairs = output columns / 2.
struct Epilogue;
void launch_kq_post(const Epilogue &ep, int M, int64_t npairs, const float *s0, int64_t n0, const float *s1,
                    int64_t n1, const float *s2, int mode, cudaStream_t s);
void launch_synth_normal(uint64_t seed, uint64_t offset, int64_t n, float mean, float stdv, int dtype, void *out,
                         cudaStream_t s);
// Synthetic [N, K] block of a [*, k_full] matrix starting at (row0, col0),
// written into rows r * dst_rs + dst_ro of dst.
void launch_synth_quant(int qtype, int64_t N, int64_t K, uint64_t seed, int64_t row0, int64_t col0, int64_t k_full,
                        float stdv, const QMat &dst, int64_t dst_rs, int64_t dst_ro, cudaStream_t s);

// Fused epilogues shared by the GEMV and GEMM kernels.  Row n of the weight
// produces column n of y for token m.
enum EpiMode { EPI_PLAIN = 0, EPI_SWIGLU = 1, EPI_QKV = 2, EPI_XCHG = 3 };
struct Epilogue {
  int mode = EPI_PLAIN;
  float *y = nullptr;            // PLAIN: [M][ldy]; SWIGLU: [M][ldy] (N/2 columns used)
  const float *resid = nullptr;  // PLAIN only: y = resid + acc (may alias y)
  int64_t ldy = 0;
  // QKV: rows [0,n_q) -> q_out (rope), [n_q, n_q+n_kv) -> k cache (rope, fp16),
  // [n_q+n_kv, n_q+2 n_kv) -> v cache (fp16).
  float *q_out = nullptr;  // [M][n_q]
  __half *k_cache = nullptr, *v_cache = nullptr;  // [B][Hkv][cap][d]
  int n_q = 0, n_kv = 0, head_dim = 0, cap = 0;
  int tokens_per_seq = 1;        // token m belongs to sequence m / tokens_per_seq
  const int *pos = nullptr;      // [B] cache length before this forward
  const float *inv_freq = nullptr;  // [head_dim/2]
  // single-token QKV (the persistent decode step): cos / sin of every frequency at position pos0,
  // cos at [i], sin at [head_dim/2 + i], computed once per launch (null: sincosf per pair)
  const float *rope_cs = nullptr;
  int pos0 = 0;
  // XCHG (tensor-parallel partial sums): column n goes to xdst[r] + xoff + n for every rank r < nx
  float *const *xdst = nullptr;
  int64_t xoff = 0;
  int nx = 0;
};

// gemv.cu: y = x W^T for up to 4 rows of x (the batch-1 decode path).
// x [M][ldx] fp32; optional fused RMSNorm of x (gamma may be null).
bool gemv_supported(const QMat &w, int M);
void launch_qgemv_ld(const QMat &w, const float *x, int M, int64_t ldx, const float *norm_gamma, float norm_eps,
                     bool do_norm, const Epilogue &ep, const GemvScratch &sc, int num_sms, cudaStream_t s);
// gemm.cu: the same contract without the fused norm, any M (prefill / batched decode).
void launch_qgemm(const QMat &w, const float *x, int M, int64_t ldx, const Epilogue &ep, const GemvScratch &sc,
                  int num_sms, cudaStream_t s);
// gemm_tc.cu: the Q4_0 GEMM on tcgen05 tensor cores (launch_qgemm picks it).
bool qgemm_tc_supported(const QMat &w, int M);
// fp16 scratch elements the tensor-core GEMM needs for M tokens of K columns
// (rows padded to whole 128-column quads).
inline uint64_t tc_xh_elems(int64_t M, int64_t K) { return (uint64_t)M * (uint64_t)(q4_quads(K) * 128); }
void launch_qgemm_tc(const QMat &w, const float *x, int M, int64_t ldx, const Epilogue &ep, const GemvScratch &sc,
                     int num_sms, cudaStream_t s);
// C[M, N] = A[M, K] B[K, N]; b_trans: B stored as [N, K].
void launch_matmul_f32(const float *A, const float *B, float *C, int64_t M, int64_t K, int64_t N, cudaStream_t s,
                       bool b_trans = false);
// matmul_tc.cu: the same product on tcgen05 (tf32 with a three-term split, fp32-level accuracy); `scratch`
// holds matmul_tc_scratch_bytes(M, K, N).  launch_matmul picks it (or the SIMT kernel for small
// products) and takes the scratch from the context's pool.
uint64_t matmul_tc_scratch_bytes(int64_t M, int64_t K, int64_t N);
void launch_matmul_tc(const float *A, const float *B, float *C, int64_t M, int64_t K, int64_t N, bool b_trans,
                      void *scratch, int *err, cudaStream_t s);
bool matmul_use_tc(int64_t M, int64_t K, int64_t N);
void launch_matmul(Ctx &c, const float *A, const float *B, float *C, int64_t M, int64_t K, int64_t N, bool b_trans);

// attention.cu
struct AttnArgs {
  const void *q;  // fp32 or fp16
  const void *k, *v;
  float *o;
  int q_f16 = 0, kv_f16 = 0;
  int B = 1, H = 1, Hkv = 1, Nq = 1, d = 64;
  int64_t q_sb = 0, q_sh = 0, q_si = 0;  // element strides of Q (batch, head, token)
  int64_t o_sb = 0, o_sh = 0, o_si = 0;
  int64_t kv_sb = 0, kv_sh = 0;          // element strides of K/V (batch, head); token stride = d
  const int *n_kv_dev = nullptr;         // per-sequence live KV length on the device (or null)
  int n_kv = 0;                          // used when n_kv_dev is null
  int n_kv_add = 0;                      // n_kv = n_kv_dev[b] + n_kv_add
  float scale = 1.0f;
  int causal = 0;
  int scratch_batch = 0;                 // decode scratch was sized for this batch (0 = B)
  int *err = nullptr;                    // device error word of bounded waits (tensor-core path)
};
void launch_attention(const AttnArgs &a, int num_sms, cudaStream_t s);
// attention_tc32.cu: fp32 K/V on the tensor cores (fp16 hi/lo splits of Q and K, range-scaled per head
// and query row, in scratch from the context pool) where the shape allows, else launch_attention above.
bool attn_tc32_supported(const AttnArgs &a);
void launch_attention(Ctx &c, const AttnArgs &a, cudaStream_t s);
// attention_tc.cu: tcgen05 flash attention (fp16 K/V, head_dim 64 or 128,
// 16-byte aligned rows).  K/V past the live length up to the cache extent
// (kv_sh / d tokens) are read in whole 128-key blocks and masked, so they must
// hold finite values.
bool attn_tc_supported(const AttnArgs &a);
void launch_attention_tc(const AttnArgs &a, cudaStream_t s);
bool attn_decode_supported(const AttnArgs &a);
// Split-KV decode attention (Nq == 1, fp16 cache, fp32 q).  Needs a scratch
// area of attn_decode_scratch_bytes() bytes: per-head arrival counters first
// (sized for scratch_batch, zero on entry and left zero on exit), then the
// per-split partial results.
// Split count for k_attn_decode: the fewest waves of resident CTAs, weighed
// against per-CTA latency, within `max_scratch` bytes of scratch.
int attn_decode_splits(const AttnArgs &a, int max_kv, int num_sms, uint64_t max_scratch = ~0ull);
uint64_t attn_decode_scratch_bytes(const AttnArgs &a, int splits);
void launch_attention_decode(const AttnArgs &a, int splits, void *scratch, cudaStream_t s);

// decode_step.cu: the persistent batch-1 decode step (one launch per token).
struct StepLayer {
  QMat qkv, o, gateup, down;
  const float *attn_norm, *ffn_norm;
  __half *k, *v;  // [Hkv][cap][d] fp16 (batch 1)
};
struct StepArgs {
  const StepLayer *layers;  // [L], device memory
  int L;
  QMat lm_head;
  const float *norm;
  const __half *embed;      // [vocab][H]
  int vocab, H, d, Hq, Hkv, I, cap;
  float eps, scale;
  const float *inv_freq;
  float *h, *q, *att, *ffn, *logits;
  int32_t *ids;             // [1] token in / out
  int *pos;                 // [1] cache length
  int32_t *token_log;
  int *step;
  int log_steps;
  unsigned long long *argkey;  // 0 between launches
  GemvScratch gs;              // error word
  float *attn_part;            // [Hkv][2 SMs / Hkv][G][d + 2]
  unsigned long long *attn_cnt;  // [Hkv] arrivals of the head's attention splits (never reset)
  unsigned long long *bar;     // grid barrier arrivals, launches; attention arrivals per head so far (never reset)
  int *err;
  uint64_t xarea_bytes;
  // [L][2] CUtensorMap of every layer's K and V cache ([Hkv][cap][d] fp16, boxes of 32 keys x 64 dims, 128-byte
  // swizzle): the attention phases' tile copies
  const void *kv_maps = nullptr;
  // tensor parallelism (tp > 1): rank r's exchange region at xr[r] (a peer mapping for r != rank):
  // float part[2][tp][H] (partial sums of o_proj / down_proj by source rank, by exchange parity),
  // then at byte xflags the u64 flag words: key[8] at word 8, kflag[8] at word 16 (the greedy pick across
  // vocabulary shards) and at word 24 the exchange counter (one add per CTA of every rank per exchange).
  int tp = 1, rank = 0;
  float *xr[8] = {};
  int64_t xflags = 0;
  unsigned long long *xep = nullptr;  // exchange epoch of this rank (launches; never reset)
  int vocab_l = 0, vbase = 0;         // logits of this rank: vocab_l rows from global index vbase
  float *h2 = nullptr;                // the residual's second buffer (tensor parallelism: h alternates)
};
// Bytes of the step kernel's grid-barrier words (zeroed at setup and reset).
constexpr uint64_t kStepBarBytes = 2048;
bool decode_step_supported(int d, int G, int qtype, int64_t H, int64_t I, int64_t qdim);
size_t decode_step_xarea(int d, int G, int64_t H, int64_t I, int64_t qdim);
size_t decode_step_smem(int d, int G, int64_t H, int64_t I, int64_t qdim);
int decode_step_vctas(int num_sms);
void launch_decode_step(const StepArgs &A, int num_sms, cudaStream_t s);

// misc.cu
void launch_rmsnorm(const float *x, int64_t ldx, const float *gamma, float eps, int64_t tokens, int64_t dim,
                    float *out, cudaStream_t s);
void launch_rope(const float *x, int64_t rows, int64_t N, int64_t d, const float *inv_freq, int64_t offset,
                 float *out, cudaStream_t s);
void launch_swiglu(const float *g, const float *u, int64_t n, float *out, cudaStream_t s);
void launch_embedding(const void *table, int table_f16, int64_t vocab, int64_t dim, const void *ids, int ids_f32,
                      int64_t n, float *out, cudaStream_t s);
void launch_add(const float *a, const float *b, int64_t n, float *out, cudaStream_t s);
void launch_argmax(const float *logits, int64_t rows, int64_t n, int64_t ld, int32_t *out, cudaStream_t s);
// sample.cu: LLMSampler.sample per row (temperature, top-k, top-p, Xorshift32 seed);
// scratch of sample_scratch_bytes(rows, V) bytes.
uint64_t sample_scratch_bytes(int64_t rows, int64_t V);
void launch_sample(const float *logits, int64_t rows, int64_t V, int64_t ld, double temperature, int top_k,
                   double top_p, bool has_seed, uint32_t seed, void *scratch, int32_t *out, cudaStream_t s);
// per-row (value, index) keys for a cross-rank greedy pick: key orders by value
// then by lower global index; index_base = first global column of this shard.
void launch_argmax_keys(const float *logits, int64_t rows, int64_t n, int64_t ld, int64_t index_base,
                        unsigned long long *keys, cudaStream_t s);
void launch_keys_to_ids(const unsigned long long *keys, int64_t rows, int32_t *ids, cudaStream_t s);
void launch_cast(const void *in, int in_dtype, void *out, int out_dtype, int64_t n, cudaStream_t s);
void launch_check_finite(const float *x, int64_t n, int *flag, cudaStream_t s);
void launch_advance_pos(int *pos, int batch, int by, int32_t *log, const int32_t *ids, int *step, int log_steps,
                        cudaStream_t s);

}  // namespace fg
