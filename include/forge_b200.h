/*
 * forge_b200.h -- C ABI of the B200-native quantized-LLM inference path of
 * AMEVA-Forge (uno-km/ameva-forge).
 *
 * The library replaces the reference's WebGPU backend (device, buffer pool,
 * staging ring, pipeline cache, quota: packages/forge/src/webgpu/) and the
 * encode/submit halves of gpuCore.dispatchKernel (packages/forge/src/tensor/
 * gpuCore.ts:500-600) and executeGraph (packages/forge/src/tensor/
 * graphExecutor.ts:517-1979).  Its op entry points mirror gpuCore's op API
 * (gpuCore.ts:1448-1467) and the model entry points mirror
 * LlamaForCausalLM.forward/generate (packages/forge-py/src/forge/models/
 * llama.py:199-248).  Every citation below is relative to the reference
 * project root.
 *
 * Conventions
 *   - Every function returns an int status: FG_OK (0) or one FG_ERR_* code,
 *     one per typed error class of packages/forge/src/errors.ts:12-111.
 *     fg_last_error() returns the thread-local message of the last failure.
 *   - Tensors are opaque 64-bit handles owned by the library.  Host buffers
 *     are borrowed for the duration of a call only.
 *   - Calls on one context are serialised; all device work of a context runs
 *     on one CUDA stream (plus NCCL on the same stream under tensor
 *     parallelism).  Calls enqueue and return; fg_read / fg_synchronize wait.
 *   - No PyTorch, Triton or CPU fallback: without a CUDA device fg_init
 *     fails with FG_ERR_UNAVAILABLE.
 */
#ifndef FORGE_B200_H
#define FORGE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes: errors.ts:12-111 --------------------------------------- */
enum {
  FG_OK = 0,
  FG_ERR_SHAPE = 1,          /* AMEVAForgeShapeError            errors.ts:32  */
  FG_ERR_DTYPE = 2,          /* AMEVAForgeDTypeError            errors.ts:39  */
  FG_ERR_DEVICE = 3,         /* AMEVAForgeDeviceError           errors.ts:46  */
  FG_ERR_DISPOSED = 4,       /* AMEVAForgeDisposedError         errors.ts:53  */
  FG_ERR_QUOTA_EXCEEDED = 5, /* AMEVAForgeQuotaExceededError    errors.ts:60  */
  FG_ERR_UNAVAILABLE = 6,    /* AMEVAForgeWebGPUUnavailableError errors.ts:67 (no CUDA device) */
  FG_ERR_SECURITY = 7,       /* AMEVAForgeSecurityError         errors.ts:74  */
  FG_ERR_UNSUPPORTED_OP = 8, /* AMEVAForgeUnsupportedOpError    errors.ts:81  */
  FG_ERR_VALIDATION = 9,     /* AMEVAForgeValidationError       errors.ts:87  */
  FG_ERR_OUT_OF_MEMORY = 10, /* AMEVAForgeOutOfMemoryError      errors.ts:93  */
  FG_ERR_INTERNAL_GPU = 11,  /* AMEVAForgeInternalGPUError      errors.ts:99  */
  FG_ERR_DEVICE_LOST = 12,   /* AMEVAForgeDeviceLostError       errors.ts:105 */
  FG_ERR_STALE_HANDLE = 13   /* AMEVAForgeStaleHandleError      errors.ts:111 */
};

/* ---- element types ---------------------------------------------------------
 * The reference is fp32-only (packages/forge/src/types.ts:26).  fp16 is added
 * for Q/K/V and the KV cache; Q4_0 / Q8_0 are GGUF block formats (32 values
 * per block with one fp16 scale) stored on the device in the reference's
 * unpack layout (unpack_quant.wgsl.ts:38-51) plus an fp16 scale plane.    */
enum {
  FG_F32 = 0,
  FG_F16 = 1,
  FG_I32 = 3,
  FG_U8 = 4,
  FG_U32 = 5,
  FG_Q4_0 = 16,
  FG_Q8_0 = 17,
  FG_Q4_K = 18, /* GGUF k-quant super-blocks (256 values: Q4_K 144 bytes, Q6_K 210 bytes),   */
  FG_Q6_K = 19  /* kept in GGUF order; cols % 256 == 0.  fg_upload_quant / fg_read_quant_gguf /
                   fg_dequant / fg_qmatmul take them (GEMV for up to 8 rows of x, else dequant +
                   GEMM); the graph front-end's transpose -> matmul fold too. */
};

typedef struct fg_ctx fg_ctx;
typedef struct fg_llama fg_llama;
typedef uint64_t fg_handle; /* 0 is never a valid handle */

#define FG_MAX_DIMS 8

typedef struct fg_init_opts {
  int32_t device;            /* CUDA ordinal */
  int32_t tp_rank;           /* tensor-parallel rank (0 when tp_size == 1) */
  int32_t tp_size;           /* 1 = single GPU, no NCCL */
  int32_t reserved;
  uint64_t vram_limit_bytes; /* quota; 0 = 92% of the free device memory
                                (gpuCore.init({vramLimitBytes}), gpuCore.ts:236-307) */
  uint8_t nccl_id[128];      /* fg_nccl_unique_id() of rank 0 when tp_size > 1 */
} fg_init_opts;

typedef struct fg_tensor_info { /* getTensorInfo (pyodideBridge.ts:31-58) */
  int32_t dtype;
  int32_t ndim;
  int64_t shape[FG_MAX_DIMS];
  uint64_t bytes;
  uint64_t device_ptr;
} fg_tensor_info;

typedef struct fg_quota { /* getQuotaSnapshot (packages/forge/src/webgpu/quota.ts:315-336) */
  uint64_t limit_bytes;
  uint64_t active_bytes;
  uint64_t pending_bytes; /* disposed, waiting for the stream to pass them */
  uint64_t peak_bytes;
  uint64_t live_tensors;
} fg_quota;

/* ---- library / context ------------------------------------------------------ */
const char *fg_version(void);
/* Thread-local message of the last failing call (errors.ts messages). */
const char *fg_last_error(void);
/* "AMEVAForgeShapeError" etc. -- the JS class name the N-API shim throws,
 * which forge-py maps back to exceptions by name (forge-py bridge.py:206-226). */
const char *fg_status_name(int status);
int fg_device_count(int32_t *out);
/* Replaces gpuCore.init / initWebGPU (gpuCore.ts:236-312, device.ts:77-134). */
int fg_init(const fg_init_opts *opts, fg_ctx **out);
int fg_shutdown(fg_ctx *ctx);
/* NCCL unique id for fg_init_opts.nccl_id (new: the reference has no
 * multi-GPU path). */
int fg_nccl_unique_id(uint8_t out[128]);
int fg_synchronize(fg_ctx *ctx);
/* The context's CUDA stream (cudaStream_t), for callers that interleave
 * their own work. */
int fg_get_stream(fg_ctx *ctx, void **stream);
int fg_quota_snapshot(fg_ctx *ctx, fg_quota *out);

/* ---- tensor lifecycle: tensorRegistry.ts:24-255, buffers.ts:24-242 ---------- */
/* uploadFloat32Array / graph "upload" (graphExecutor.ts:652-700): copies
 * `bytes` from host into a new device tensor of the given shape and dtype.
 * Non-finite f32 values are rejected (FG_ERR_VALIDATION) unless the context
 * allows them, as the reference's upload does (graphExecutor.ts:667-681). */
int fg_upload(fg_ctx *ctx, const void *host, uint64_t bytes, const int64_t *shape, int32_t ndim,
              int32_t dtype, fg_handle *out);
/* GGUF loader weight upload (new; the reference's loader is an open TODO,
 * JIRA_RELEASE_TASKS_MATRIX.md:70): takes raw Q4_0 (18 B) or Q8_0 (34 B)
 * blocks of a row-major [rows, cols] matrix and repacks them on the device. */
int fg_upload_quant(fg_ctx *ctx, int32_t qtype, const void *gguf_blocks, uint64_t bytes, int64_t rows,
                    int64_t cols, fg_handle *out);
/* Uninitialised device tensor. */
int fg_empty(fg_ctx *ctx, const int64_t *shape, int32_t ndim, int32_t dtype, fg_handle *out);
/* read / mapBufferAsync+readMappedInto (gpuCore.ts:372-471): copies the whole
 * tensor into `host` (`bytes` must equal the tensor size); waits. */
int fg_read(fg_ctx *ctx, fg_handle h, void *host, uint64_t bytes);
/* Reads a quantized tensor back as GGUF blocks (inverse of fg_upload_quant). */
int fg_read_quant_gguf(fg_ctx *ctx, fg_handle h, void *host, uint64_t bytes);
int fg_info(fg_ctx *ctx, fg_handle h, fg_tensor_info *out);
/* dispose (tensorRegistry.ts:136-152): deferred until the stream has passed
 * every use; a second dispose of the same handle is a no-op. */
int fg_dispose(fg_ctx *ctx, fg_handle h);
int fg_dispose_batch(fg_ctx *ctx, const fg_handle *hs, int32_t n);
/* configureRuntime({allowNonFinite}) (graphExecutor.ts:118-127). */
int fg_set_allow_non_finite(fg_ctx *ctx, int32_t allow);

/* ---- ops: gpuCore op API (gpuCore.ts:1448-1467); each allocates its output --- */
/* gpuCore.unpackQuant (gpuCore.ts:1123-1152) with the graph path's semantics
 * (graphExecutor.ts:1313-1323): out[i] = (code_i - zeros[i/gs]) * scales[i/gs],
 * code_i = nibble i%8 of u32 word i/8 (bits 4) or byte i%4 of word i/4
 * (bits 8).  packed: U32 (or F32 bit patterns), scales/zeros: F32. */
int fg_unpack_quant(fg_ctx *ctx, fg_handle packed, fg_handle scales, fg_handle zeros, int32_t bits,
                    int64_t group_size, int64_t num_elements, fg_handle *out);
/* Q4_0/Q8_0 tensor -> F32 [rows, cols], bit-identical to the unpack above. */
int fg_dequant(fg_ctx *ctx, fg_handle w, fg_handle *out);
/* Quantized nn.Linear (forge-py nn.py:248-259): y[..., N] = x[..., K] W^T with
 * W a Q4_0/Q8_0 [N, K] tensor, fp32 accumulation.  Dequantisation is fused
 * into the GEMV (up to 4 rows of x) or GEMM that consumes it. */
int fg_qmatmul(fg_ctx *ctx, fg_handle x, fg_handle w, fg_handle *out);
/* fg_qmatmul into an existing F32 tensor `out` of x's shape with the last
 * dimension N (no allocation, so a caller can capture it in a CUDA graph on
 * the context stream). */
int fg_qmatmul_into(fg_ctx *ctx, fg_handle x, fg_handle w, fg_handle out);
/* gpuCore.matmul (gpuCore.ts:713-761): C[M,N] = A[M,K] B[K,N], fp32. */
int fg_matmul(fg_ctx *ctx, fg_handle a, fg_handle b, fg_handle *out);
/* gpuCore.flashAttention (gpuCore.ts:949-1017): Q [B,H,Nq,d], K/V
 * [B,Hkv,Nkv,d], H % Hkv == 0, d <= 256; scale = 1/sqrt(d) unless has_scale.
 * F32 inputs use an fp32 kernel; F16 inputs use the tensor-core kernel
 * (fp32 softmax statistics).  Output dtype = F32. */
int fg_flash_attention(fg_ctx *ctx, fg_handle q, fg_handle k, fg_handle v, float scale,
                       int32_t has_scale, int32_t causal, fg_handle *out);
/* Decode attention (one query token per sequence) that allocates nothing.
 * No counterpart in the reference: it serves hosts that cannot allocate at
 * call time (device memory fully committed to their own KV cache under a hard
 * quota, latency-critical threads where cudaMalloc/cudaFree would synchronise
 * the device, hosts without an fg_ctx).  Raw device pointers: q and out F32
 * [batch, heads, head_dim]; k_cache and v_cache F16 [batch, kv_heads,
 * cache_capacity, head_dim], of which the first n_kv positions are attended.
 * head_dim 64 or 128, heads / kv_heads in {1, 2, 4, 8}.  k_cache and
 * v_cache must be 16-byte aligned (the kernel copies 16-byte chunks of them)
 * and q and out 4-byte aligned; other pointers give FG_ERR_VALIDATION.
 * Runs on `stream`
 * (a cudaStream_t; NULL = legacy default stream) of the current device.
 * Split-KV scratch comes from a 2 MiB static device array: shapes whose
 * partials would need more run with fewer splits (one split needs none).
 * Calls on one device must not overlap in
 * time (they share the array); calls queued on one stream are safe.  The
 * first call on each device looks up the array's address and must not be
 * made during stream capture. */
int fg_attention_decode_static(const float *q, const void *k_cache, const void *v_cache, float *out,
                               int32_t batch, int32_t heads, int32_t kv_heads, int32_t head_dim,
                               int64_t cache_capacity, int32_t n_kv, float scale, void *stream);
/* gpuCore.rmsNorm (rmsnorm.wgsl.ts:10-74); gamma 0 = none. */
int fg_rmsnorm(fg_ctx *ctx, fg_handle x, fg_handle gamma, float eps, fg_handle *out);
/* gpuCore.rope (rope.wgsl.ts:11-62): interleaved pairs, x [B,H,N,d]. */
int fg_rope(fg_ctx *ctx, fg_handle x, float base, int64_t offset, fg_handle *out);
/* gpuCore.swiglu (swiglu.wgsl.ts:11-42), graph-path semantics. */
int fg_swiglu(fg_ctx *ctx, fg_handle gate, fg_handle up, fg_handle *out);
/* gpuCore.embedding (embedding.wgsl.ts:20-63): table F32/F16 [V, D], ids
 * I32 (or F32, rounded half to even); out-of-range ids give a zero row. */
int fg_embedding(fg_ctx *ctx, fg_handle table, fg_handle ids, fg_handle *out);
/* gpuCore.add for equal shapes (residual add). */
int fg_add(fg_ctx *ctx, fg_handle a, fg_handle b, fg_handle *out);
/* Greedy pick per row (LLMSampler.sample, sampling.ts:45-55): I32 [rows]
 * index of the first maximum of each row of logits [rows, n]. */
int fg_argmax(fg_ctx *ctx, fg_handle logits, fg_handle *out);
/* LLMSampler.sample (sampling.ts:35-128) on the device, per row of logits
 * [rows, V] -> I32 [rows]: greedy at temperature <= 1e-5, else top-k (the
 * reference's partial selection sort for k <= 128, a stable sort otherwise),
 * softmax at the temperature, top-p cutoff, and a categorical pick with the
 * first Xorshift32 output of `seed`.  has_seed = 0 draws the seed from the
 * host's random device (the reference uses Math.random). */
int fg_sample(fg_ctx *ctx, fg_handle logits, double temperature, int32_t top_k, double top_p, int32_t has_seed,
              uint32_t seed, fg_handle *out);
/* Element-type conversion F32 <-> F16 (round to nearest even). */
int fg_cast(fg_ctx *ctx, fg_handle x, int32_t dtype, fg_handle *out);

/* ---- graph front-end: executeGraph (graphExecutor.ts:487-1979) -------------
 * Runs the JSON instruction list of forge-py's GraphBuilder (graph.py:26-203):
 * [{"op", "id", "shape", "in"?, "params"?, "handle"?}, ...].  Validation
 * follows validateInstruction (graphExecutor.ts:310-478) with its messages
 * and error classes; the k-th "upload" node takes inputs[k] (float32, exactly
 * prod(shape) * 4 = input_bytes[k] bytes; non-finite values rejected unless
 * allowed); a "load" node names an existing tensor as "tensor_<hex handle>"
 * (or the decimal handle) and may also name F16 / Q4_0 / Q8_0 tensors, which
 * the Llama path consumes directly (a Q4_0 weight W under transpose -> matmul
 * runs the fused dequant GEMV / GEMM).  On success out_ids[i] / out_handles[i]
 * hold every node's id and tensor handle in instruction order (n_out = node
 * count; out_cap must be at least that).  On failure every tensor the call
 * created is disposed (the GraphTransaction rollback, :1847-1871).  Some node
 * tensors (a transpose read only by matmul, GQA head slices / cats read only
 * by attention) are computed only when first read.  Ops implemented: upload,
 * load, reshape, transpose, permute, slice, cat, matmul, matmul_tiled,
 * add/sub/mul/div (broadcasting), relu/neg/exp/log/sigmoid/tanh, rope,
 * rmsnorm, swiglu, unpack_quant, embedding, flash_attention; the other ops of
 * the allow-list give FG_ERR_UNSUPPORTED_OP. */
int fg_execute_graph(fg_ctx *ctx, const char *instructions_json, const void *const *inputs,
                     const uint64_t *input_bytes, int32_t n_inputs, int64_t *out_ids, fg_handle *out_handles,
                     int32_t out_cap, int32_t *n_out);
/* configureRuntime({maxInstructions, maxShapeDim, maxElements})
 * (graphExecutor.ts:98-127); defaults 10000, 8, 2^28. */
int fg_configure_graph(fg_ctx *ctx, int64_t max_instructions, int32_t max_shape_dim, int64_t max_elements);

/* ---- seeded synthetic data (new; the benchmark inputs) ---------------------
 * value i = mean + std * N01(seed, offset + i), N01 = splitmix64 counter
 * generator feeding a 4-term central-limit normal; dtype F32 or F16. */
int fg_synth_normal(fg_ctx *ctx, const int64_t *shape, int32_t ndim, int32_t dtype, uint64_t seed,
                    uint64_t offset, float mean, float stdv, fg_handle *out);
/* GGUF-quantized [rows, cols] matrix of N(0, std) values (element (r, c) =
 * std * N01(seed, (row0 + r) * cols + c)), quantized on the device with the
 * ggml block recipe. */
int fg_synth_quant(fg_ctx *ctx, int32_t qtype, int64_t rows, int64_t cols, uint64_t seed, int64_t row0,
                   float stdv, fg_handle *out);

/* ---- Llama model: LlamaConfig / LlamaForCausalLM (llama.py:30-248) ---------- */
typedef struct fg_llama_config {
  int32_t vocab_size;
  int32_t hidden_size;
  int32_t intermediate_size;
  int32_t num_hidden_layers;
  int32_t num_attention_heads;
  int32_t num_key_value_heads;
  int32_t max_position_embeddings; /* KV-cache capacity per sequence */
  int32_t max_batch;               /* sequences decoded together */
  float rms_norm_eps;
  float rope_theta;
  int32_t qtype; /* FG_Q4_0 or FG_Q8_0 for every Linear incl. lm_head */
  int32_t reserved;
} fg_llama_config;

int fg_llama_create(fg_ctx *ctx, const fg_llama_config *cfg, fg_llama **out);
int fg_llama_destroy(fg_llama *m);
/* Loads one weight of the FULL (unsharded) model; under tensor parallelism
 * each rank keeps its shard.  name: "embed" (F16 [V,H]), "norm" (F32 [H]),
 * "lm_head" (GGUF blocks [V,H]), per layer "q","k","v","o","gate","up",
 * "down" (GGUF blocks, nn.Linear [out,in]) and "attn_norm","ffn_norm" (F32). */
int fg_llama_load(fg_llama *m, const char *name, int32_t layer, const void *host, uint64_t bytes);
/* Fills every weight with the seeded synthetic recipe (N(0, std) quantized
 * Linears, fp16 embedding, norm gains 1 + 0.1 N01): tensor t of layer l uses
 * seed splitmix64(seed, l*16 + t); globals use layer 0xFFFF. */
int fg_llama_synthesize(fg_llama *m, uint64_t seed, float stdv);
/* Empties the KV cache (position 0). */
int fg_llama_reset(fg_llama *m);
int fg_llama_position(fg_llama *m, int32_t *pos);
/* forward(input_ids, past_key_values, offset_pos) (llama.py:199-210): runs
 * `len` tokens of each of `batch` sequences from host ids [batch, len],
 * appends them to the cache, and returns the last position's logits
 * [batch, vocab] and/or greedy next ids [batch] (nullable outputs). */
int fg_llama_forward(fg_llama *m, const int32_t *ids, int32_t batch, int32_t len, float *logits,
                     int32_t *next_ids);
/* One decode step of generate() (llama.py:239-246): host ids [batch] in,
 * greedy next ids [batch] (and optional logits [batch, vocab]) out.  The
 * step is one CUDA graph launch. */
int fg_llama_decode(fg_llama *m, const int32_t *ids, int32_t batch, int32_t *next_ids, float *logits);
/* `steps` device-resident greedy decode steps: each step's input is the
 * previous step's argmax, kept on the device; token ids of the run are
 * retrievable with fg_llama_tokens.  Seeded from the last decode/forward. */
int fg_llama_generate_device(fg_llama *m, int32_t batch, int32_t steps);
/* Copies the ids produced by the last fg_llama_generate_device call,
 * [steps, batch] row-major. */
int fg_llama_tokens(fg_llama *m, int32_t *host, int64_t count);
/* Sets the cache length of sequences [0, batch) to `pos` without running a
 * prefill: positions [0, pos) keep whatever the cache holds (zeros after
 * creation).  For decode measurements at a given context. */
int fg_llama_set_position(fg_llama *m, int32_t batch, int32_t pos);
/* Fills positions [0, len) of every layer's KV cache for sequences
 * [0, batch) with seeded fp16 values and sets their cache length to len (a
 * context "prefilled" without running a prefill; new: the reference always
 * prefills).  Key (b, kv head h, position p, dim c) of layer l is
 * fp16(std * N01(splitmix64(seed, l*16 + 9), ((b*Hkv + h)*len + p)*d + c)),
 * values use l*16 + 10; h counts the model's KV heads, so under tensor
 * parallelism each rank writes its heads' slice of the same global cache. */
int fg_llama_synthesize_kv(fg_llama *m, uint64_t seed, int32_t batch, int32_t len, float stdv);
/* Which kernel runs a decode step of `batch` sequences: 1 = the persistent
 * one-launch step kernel, 0 = the layered per-op kernels (new; for tests and
 * tools that must know which path they measured). */
int fg_llama_decode_path(fg_llama *m, int32_t batch, int32_t *kind);
/* The configuration the model was created with. */
int fg_llama_get_config(fg_llama *m, fg_llama_config *cfg);

/* ---- GGUF files (new: the loader the reference plans, ranked first among
 * the components after the hot path) -----------------------------------------
 * GGUF v2/v3 container, memory-mapped and validated on open (lengths and
 * offsets against the file size; a malformed file gives FG_ERR_VALIDATION).
 * Tensor dims follow ggml (dims[0] innermost: a Linear [out, in] is
 * {in, out}); dtype is FG_F32 / FG_F16 / FG_Q4_0 / FG_Q8_0, or -1 for ggml
 * types this build does not read (their data pointer is null). */
typedef struct fg_gguf fg_gguf;
int fg_gguf_open(const char *path, fg_gguf **out);
int fg_gguf_close(fg_gguf *g);
int fg_gguf_tensor_count(const fg_gguf *g, int64_t *n);
int fg_gguf_tensor_info(const fg_gguf *g, int64_t i, const char **name, int32_t *dtype, int32_t *ndim,
                        int64_t *dims /* [4] */, const void **data, uint64_t *bytes);
int fg_gguf_meta_number(const fg_gguf *g, const char *key, double *value);
int fg_gguf_meta_string(const fg_gguf *g, const char *key, const char **value);
/* LlamaConfig from the llama.* metadata (general.architecture "llama"): vocab
 * from token_embd.weight, qtype from blk.0.attn_q.weight; max_position <= 0
 * takes llama.context_length. */
int fg_gguf_llama_config(const fg_gguf *g, int32_t max_position, int32_t max_batch, fg_llama_config *cfg);
/* Loads every weight of a llama.cpp-named Llama file into the model (each
 * rank keeps its shard): token_embd (F16/F32), output_norm, output, and
 * blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm, ffn_gate,
 * ffn_up, ffn_down}; the Linears must be of the model's qtype. */
int fg_llama_load_gguf(fg_llama *m, const fg_gguf *g);

#ifdef __cplusplus
}
#endif
#endif /* FORGE_B200_H */
