// Llama-shaped decoder over quantized weights: LlamaConfig / LlamaModel /
// LlamaForCausalLM (packages/forge-py/src/forge/models/llama.py:30-248).
//
// Per layer (llama.py:149-165) the step is five kernels:
//   1. qkv GEMV/GEMM: fused input RMSNorm, q/k/v projections (one fused
//      weight), interleaved RoPE and the fp16 KV-cache append in the epilogue
//      (replaces rope + cat of llama.py:102-111; the cache is written in place);
//   2. attention: split-KV decode kernel (N_q = 1) or the prefill kernel; GQA
//      is native (llama.py:116-127's head repetition is never materialised);
//   3. o_proj with the residual add in the epilogue (+ NCCL all-reduce under
//      tensor parallelism);
//   4. gate/up (rows interleaved) with fused post-attention RMSNorm and SwiGLU;
//   5. down_proj with the residual add (+ all-reduce).
// The final norm is fused into the lm_head GEMV; greedy argmax on the device.
// A decode step is captured once into a CUDA graph and replayed.
//
// Tensor parallelism (Megatron): q/k/v/gate/up are split by output rows
// (heads / FFN columns), o/down by input columns, lm_head by vocabulary rows;
// embedding and norms are replicated.  Rank 0 adds the residual before the
// in-place all-reduce, the other ranks contribute only their partial sums.
#include "nccl_dyn.cuh"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>

#include "q4_gemv.cuh"
#include "runtime.cuh"
#include "tmap.cuh"

using namespace fg;

namespace {
enum Tid { T_Q = 0, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_ATTN_NORM, T_FFN_NORM };
constexpr int kGlobal = 0xFFFF;
enum Gid { G_EMBED = 0, G_NORM = 1, G_LM_HEAD = 2 };

// One Linear of a k-quant model (GGUF Q4_K / Q6_K blocks in file order, [N][K]).
struct KQ {
  void *p = nullptr;
  int type = 0;
  int64_t N = 0, K = 0;
};
enum { KQ_Q, KQ_K, KQ_V, KQ_O, KQ_GATE, KQ_UP, KQ_DOWN, KQ_N };

struct LayerW {
  float *attn_norm = nullptr, *ffn_norm = nullptr;
  QMat qkv, o, gateup, down;
  KQ kq[KQ_N];                        // k-quant models: the Linears as loaded, each of its own type
  __half *k = nullptr, *v = nullptr;  // [max_batch][Hkv_l][cap][d]
};
}  // namespace

struct fg_llama {
  fg_ctx *ctx_handle = nullptr;
  Ctx *ctx = nullptr;
  fg_llama_config cfg;
  int tp = 1, rank = 0;
  int d = 0, Hq_l = 0, Hkv_l = 0, I_l = 0, V_l = 0, H = 0;
  int cap = 0, max_batch = 1, m_max = 1;
  std::vector<std::pair<void *, uint64_t>> allocs;
  __half *embed = nullptr;
  float *norm = nullptr;
  QMat lm_head;
  std::vector<LayerW> layers;
  float *inv_freq = nullptr;
  int *pos = nullptr;         // [max_batch]
  int32_t *ids = nullptr;     // [m_max] token ids of the current step/chunk
  unsigned long long *keys = nullptr;
  float *h = nullptr, *xn = nullptr, *q = nullptr, *att = nullptr, *ffn = nullptr, *logits = nullptr;
  float *logits_all = nullptr;  // [tp][max_batch][V_l] gather buffer
  void *attn_scratch = nullptr;
  int decode_splits = 1;
  int32_t *token_log = nullptr;
  int *step = nullptr;
  int log_steps = 0;
  int host_pos = 0;
  int last_batch = 0;
  std::map<int, cudaGraphExec_t> graphs;
  bool use_step = false;  // batch-1 decode runs the persistent step kernel
  // k-quant model (created with qtype FG_Q4_K): every Linear is Q4_K or Q6_K as loaded (a llama.cpp
  // Q4_K_M file mixes both); the layer runs the k-quant GEMVs plus an epilogue pass
  bool kq = false;
  KQ lm_kq;
  float *kq_tmp = nullptr;  // [m_max][max(q + 2 kv, 2 I, H) columns]
  StepArgs step_args{};
  // tensor-parallel exchange region of this rank (cudaMalloc, shared by IPC) and the peers' mappings
  void *xbuf = nullptr;
  void *xpeer[8] = {};

  void *dalloc(uint64_t bytes) {
    void *p = ctx->alloc(bytes);
    allocs.push_back({p, bytes});
    return p;
  }
};

namespace {

uint64_t tensor_seed(uint64_t model_seed, int layer, int tid) { return splitmix64(model_seed, (uint64_t)layer * 16 + tid); }

QMat make_qmat(fg_llama *m, int qtype, int64_t N, int64_t K) {
  const uint64_t bytes = qmat_bytes(qtype, N, K);
  void *p = m->dalloc(bytes);
  FG_CUDA(cudaMemsetAsync(p, 0, bytes, m->ctx->stream));  // defined scale padding
  return qmat_at(p, qtype, N, K);
}

void allreduce(fg_llama *m, float *buf, int64_t n) {
  if (m->tp == 1) return;
  ncclResult_t r = nccl().AllReduce(buf, buf, (size_t)n, ncclFloat32, ncclSum, (ncclComm_t)m->ctx->nccl, m->ctx->stream);
  FG_REQUIRE(r == ncclSuccess, FG_ERR_DEVICE, "ncclAllReduce: %s", nccl().GetErrorString(r));
}

// y = x W^T with optional fused RMSNorm of x; GEMV for <= 4 rows, else GEMM
// (with a separate norm pass into xn).
void linear(fg_llama *m, const QMat &w, const float *x, int M, int64_t ldx, const float *gamma, bool do_norm,
            const Epilogue &ep) {
  Ctx &c = *m->ctx;
  if (gemv_supported(w, M)) {
    launch_qgemv_ld(w, x, M, ldx, gamma, m->cfg.rms_norm_eps, do_norm, ep, c.gemv, c.num_sms, c.stream);
  } else {
    const float *xx = x;
    int64_t ld = ldx;
    if (do_norm) {
      launch_rmsnorm(x, ldx, gamma, m->cfg.rms_norm_eps, M, w.K, m->xn, c.stream);
      xx = m->xn;
      ld = w.K;
    }
    launch_qgemm(w, xx, M, ld, ep, c.gemv, c.num_sms, c.stream);
  }
}

AttnArgs attn_args(fg_llama *m, const LayerW &L, int B, int T) {
  AttnArgs a;
  a.q = m->q;
  a.k = L.k;
  a.v = L.v;
  a.o = m->att;
  a.q_f16 = 0;
  a.kv_f16 = 1;
  a.B = B;
  a.H = m->Hq_l;
  a.Hkv = m->Hkv_l;
  a.Nq = T;
  a.d = m->d;
  const int64_t qrow = (int64_t)m->Hq_l * m->d;
  a.q_sb = (int64_t)T * qrow;
  a.q_sh = m->d;
  a.q_si = qrow;
  a.o_sb = a.q_sb;
  a.o_sh = a.q_sh;
  a.o_si = a.q_si;
  a.kv_sb = (int64_t)m->Hkv_l * m->cap * m->d;
  a.kv_sh = (int64_t)m->cap * m->d;
  a.n_kv_dev = m->pos;
  a.n_kv_add = T;
  a.scale = (float)(1.0 / std::sqrt((double)m->d));
  a.causal = 1;
  a.scratch_batch = m->max_batch;
  a.err = m->ctx->gemv.err;
  return a;
}

// One forward pass of T tokens for each of B sequences whose ids are already
// in m->ids ([B][T]); leaves greedy ids of the last position in m->ids[0..B)
// and advances pos by T.  Everything is enqueued on the context stream (and is
// graph-capturable when T == 1).
// y [M][w.N] = x [M][w.K] W^T for a k-quant Linear: the k-quant GEMV for up to 8 rows, else the
// bit-exact dequantisation into a temporary and the fp32 matmul (tensor cores for large products).
void kq_linear(fg_llama *m, const KQ &w, const float *x, int M, float *y) {
  Ctx &c = *m->ctx;
  FG_REQUIRE(w.p, FG_ERR_VALIDATION, "k-quant model: a Linear of shape [%lld, %lld] was never loaded",
             (long long)w.N, (long long)w.K);
  if (M <= 8) {
    if (w.type == FG_Q4_K)
      launch_qmatmul_q4k(w.p, w.N, w.K, x, M, y, nullptr, c.gemv.err, c.stream);
    else
      launch_qmatmul_q6k(w.p, w.N, w.K, x, M, y, nullptr, c.stream);
    return;
  }
  const uint64_t bytes = 4ull * (uint64_t)(w.N * w.K);
  float *w32 = (float *)c.alloc(bytes);
  try {
    if (w.type == FG_Q4_K)
      launch_dequant_q4k(w.p, w.N * w.K / 256, w32, c.stream);
    else
      launch_dequant_q6k(w.p, w.N * w.K / 256, w32, c.stream);
    launch_matmul(c, x, w32, y, M, w.K, w.N, /*b_trans=*/true);
  } catch (...) {
    c.free_async(w32, bytes);
    throw;
  }
  c.free_async(w32, bytes);
}

// forward_tokens of a k-quant model: per Linear the k-quant GEMV (plain output), then the layered
// path's epilogues as a separate pass (RoPE + fp16 KV append, SwiGLU, residual add).
void forward_tokens_kq(fg_llama *m, int B, int T, bool log_tokens) {
  Ctx &c = *m->ctx;
  const int M = B * T, H = m->H, d = m->d, I = m->I_l;
  const int64_t nq = (int64_t)m->Hq_l * d, nkv = (int64_t)m->Hkv_l * d;
  const float eps = m->cfg.rms_norm_eps;
  launch_embedding(m->embed, 1, m->cfg.vocab_size, H, m->ids, 0, M, m->h, c.stream);
  Epilogue resid;  // h += W x
  resid.mode = EPI_PLAIN;
  resid.y = m->h;
  resid.resid = m->h;
  resid.ldy = H;
  for (size_t l = 0; l < m->layers.size(); ++l) {
    const LayerW &L = m->layers[l];
    float *tq = m->kq_tmp, *tk = tq + (int64_t)M * nq, *tv = tk + (int64_t)M * nkv;
    launch_rmsnorm(m->h, H, L.attn_norm, eps, M, H, m->xn, c.stream);
    kq_linear(m, L.kq[KQ_Q], m->xn, M, tq);
    kq_linear(m, L.kq[KQ_K], m->xn, M, tk);
    kq_linear(m, L.kq[KQ_V], m->xn, M, tv);
    Epilogue e1;
    e1.mode = EPI_QKV;
    e1.q_out = m->q;
    e1.k_cache = L.k;
    e1.v_cache = L.v;
    e1.n_q = (int)nq;
    e1.n_kv = (int)nkv;
    e1.head_dim = d;
    e1.cap = m->cap;
    e1.tokens_per_seq = T;
    e1.pos = m->pos;
    e1.inv_freq = m->inv_freq;
    launch_kq_post(e1, M, (nq + 2 * nkv) / 2, tq, nq, tk, nkv, tv, 0, c.stream);

    AttnArgs a = attn_args(m, L, B, T);
    if (T == 1 && attn_decode_supported(a))
      launch_attention_decode(a, m->decode_splits, m->attn_scratch, c.stream);
    else
      launch_attention(a, c.num_sms, c.stream);

    float *to = m->kq_tmp;
    kq_linear(m, L.kq[KQ_O], m->att, M, to);
    launch_kq_post(resid, M, H / 2, to, 0, nullptr, 0, nullptr, 2, c.stream);

    launch_rmsnorm(m->h, H, L.ffn_norm, eps, M, H, m->xn, c.stream);
    float *tg = m->kq_tmp, *tu = tg + (int64_t)M * I;
    kq_linear(m, L.kq[KQ_GATE], m->xn, M, tg);
    kq_linear(m, L.kq[KQ_UP], m->xn, M, tu);
    Epilogue e4;
    e4.mode = EPI_SWIGLU;
    e4.y = m->ffn;
    e4.ldy = I;
    launch_kq_post(e4, M, I, tg, 0, tu, 0, nullptr, 1, c.stream);
    kq_linear(m, L.kq[KQ_DOWN], m->ffn, M, to);
    launch_kq_post(resid, M, H / 2, to, 0, nullptr, 0, nullptr, 2, c.stream);
  }
  // lm_head over the last position of every sequence, after the final norm
  launch_rmsnorm(m->h + (int64_t)(T - 1) * H, (int64_t)T * H, m->norm, eps, B, H, m->xn, c.stream);
  kq_linear(m, m->lm_kq, m->xn, B, m->logits);
  launch_argmax(m->logits, B, m->V_l, m->V_l, m->ids, c.stream);
  launch_advance_pos(m->pos, B, T, log_tokens ? m->token_log : nullptr, m->ids, m->step, m->log_steps, c.stream);
}

void forward_tokens(fg_llama *m, int B, int T, bool log_tokens) {
  if (m->kq) return forward_tokens_kq(m, B, T, log_tokens);
  Ctx &c = *m->ctx;
  const int M = B * T;
  const int H = m->H;
  launch_embedding(m->embed, 1, m->cfg.vocab_size, H, m->ids, 0, M, m->h, c.stream);
  for (size_t l = 0; l < m->layers.size(); ++l) {
    const LayerW &L = m->layers[l];
    Epilogue e1;
    e1.mode = EPI_QKV;
    e1.q_out = m->q;
    e1.k_cache = L.k;
    e1.v_cache = L.v;
    e1.n_q = m->Hq_l * m->d;
    e1.n_kv = m->Hkv_l * m->d;
    e1.head_dim = m->d;
    e1.cap = m->cap;
    e1.tokens_per_seq = T;
    e1.pos = m->pos;
    e1.inv_freq = m->inv_freq;
    linear(m, L.qkv, m->h, M, H, L.attn_norm, true, e1);

    AttnArgs a = attn_args(m, L, B, T);
    if (T == 1 && attn_decode_supported(a))
      launch_attention_decode(a, m->decode_splits, m->attn_scratch, c.stream);
    else
      launch_attention(a, c.num_sms, c.stream);

    Epilogue e3;
    e3.mode = EPI_PLAIN;
    e3.y = m->h;
    e3.resid = m->rank == 0 ? m->h : nullptr;
    e3.ldy = H;
    linear(m, L.o, m->att, M, (int64_t)m->Hq_l * m->d, nullptr, false, e3);
    allreduce(m, m->h, (int64_t)M * H);

    Epilogue e4;
    e4.mode = EPI_SWIGLU;
    e4.y = m->ffn;
    e4.ldy = m->I_l;
    linear(m, L.gateup, m->h, M, H, L.ffn_norm, true, e4);

    Epilogue e5 = e3;
    linear(m, L.down, m->ffn, M, m->I_l, nullptr, false, e5);
    allreduce(m, m->h, (int64_t)M * H);
  }
  // lm_head over the last position of every sequence, final norm fused
  Epilogue el;
  el.mode = EPI_PLAIN;
  el.y = m->logits;
  el.ldy = m->V_l;
  linear(m, m->lm_head, m->h + (int64_t)(T - 1) * H, B, (int64_t)T * H, m->norm, true, el);
  if (m->tp == 1) {
    launch_argmax(m->logits, B, m->V_l, m->V_l, m->ids, c.stream);
  } else {
    launch_argmax_keys(m->logits, B, m->V_l, m->V_l, (int64_t)m->rank * m->V_l, m->keys, c.stream);
    ncclResult_t r = nccl().AllReduce(m->keys, m->keys, (size_t)B, ncclUint64, ncclMax, (ncclComm_t)c.nccl, c.stream);
    FG_REQUIRE(r == ncclSuccess, FG_ERR_DEVICE, "ncclAllReduce(argmax): %s", nccl().GetErrorString(r));
    launch_keys_to_ids(m->keys, B, m->ids, c.stream);
  }
  launch_advance_pos(m->pos, B, T, log_tokens ? m->token_log : nullptr, m->ids, m->step, m->log_steps, c.stream);
}

void read_logits(fg_llama *m, int B, float *host) {
  Ctx &c = *m->ctx;
  const int64_t V = m->cfg.vocab_size;
  if (m->tp == 1) {
    c.d2h(host, m->logits, (uint64_t)B * V * 4);
    return;
  }
  ncclResult_t r = nccl().AllGather(m->logits, m->logits_all, (size_t)B * m->V_l, ncclFloat32, (ncclComm_t)c.nccl, c.stream);
  FG_REQUIRE(r == ncclSuccess, FG_ERR_DEVICE, "nccl().AllGather(logits): %s", nccl().GetErrorString(r));
  std::vector<float> tmp((size_t)m->tp * B * m->V_l);
  c.d2h(tmp.data(), m->logits_all, tmp.size() * 4);
  for (int rk = 0; rk < m->tp; ++rk)
    for (int b = 0; b < B; ++b)
      std::memcpy(host + (int64_t)b * V + (int64_t)rk * m->V_l, tmp.data() + ((int64_t)rk * B + b) * m->V_l,
                  (size_t)m->V_l * 4);
}

int set_err(int st, const char *msg);

// Tensor-parallel exchange of the persistent decode step: every rank allocates
// part[2][tp][H] floats + flag words, shares the allocation with the other
// ranks by CUDA IPC (handles all-gathered over the NCCL communicator), and maps
// the peers' regions, so the step kernel stores its o_proj / down_proj partial
// sums straight into every rank's memory over NVLink.
void setup_exchange(fg_llama *m) {
  Ctx &c = *m->ctx;
  const int tp = m->tp;
  FG_REQUIRE(tp <= 8, FG_ERR_VALIDATION, "tensor parallel degree %d > 8", tp);
  const uint64_t part = align_up((uint64_t)2 * tp * m->H * 4, 256);
  const uint64_t bytes = part + 256;  // flag words: key[8] at 8, kflag[8] at 16, the exchange counter at 24
  FG_CUDA(cudaMalloc(&m->xbuf, bytes));
  FG_CUDA(cudaMemset(m->xbuf, 0, bytes));
  cudaIpcMemHandle_t mine;
  FG_CUDA(cudaIpcGetMemHandle(&mine, m->xbuf));
  unsigned char *dh = (unsigned char *)m->dalloc((uint64_t)tp * sizeof(mine));
  c.h2d(dh + (size_t)m->rank * sizeof(mine), &mine, sizeof(mine));
  ncclResult_t r = nccl().AllGather(dh + (size_t)m->rank * sizeof(mine), dh, sizeof(mine), ncclUint8,
                                    (ncclComm_t)c.nccl, c.stream);
  FG_REQUIRE(r == ncclSuccess, FG_ERR_DEVICE, "ncclAllGather(exchange handles): %s", nccl().GetErrorString(r));
  std::vector<cudaIpcMemHandle_t> all(tp);
  c.d2h(all.data(), dh, (uint64_t)tp * sizeof(mine));
  StepArgs &A = m->step_args;
  for (int k = 0; k < tp; ++k) {
    if (k == m->rank) {
      A.xr[k] = (float *)m->xbuf;
    } else {
      FG_CUDA(cudaIpcOpenMemHandle(&m->xpeer[k], all[k], cudaIpcMemLazyEnablePeerAccess));
      A.xr[k] = (float *)m->xpeer[k];
    }
  }
  A.xflags = (int64_t)part;
  A.h2 = (float *)m->dalloc((uint64_t)m->H * 4);
  A.xep = (unsigned long long *)m->dalloc(8);
  FG_CUDA(cudaMemsetAsync(A.xep, 0, 8, c.stream));
  // every rank has zeroed and mapped its region before any rank's step kernel writes into it
  float *one = (float *)m->dalloc(4);
  FG_CUDA(cudaMemsetAsync(one, 0, 4, c.stream));
  r = nccl().AllReduce(one, one, 1, ncclFloat32, ncclSum, (ncclComm_t)c.nccl, c.stream);
  FG_REQUIRE(r == ncclSuccess, FG_ERR_DEVICE, "ncclAllReduce(exchange barrier): %s", nccl().GetErrorString(r));
  c.sync();
}

void release_exchange(fg_llama *m) {
  for (int k = 0; k < 8; ++k)
    if (m->xpeer[k]) {
      cudaIpcCloseMemHandle(m->xpeer[k]);
      m->xpeer[k] = nullptr;
    }
  if (m->xbuf) {
    cudaFree(m->xbuf);
    m->xbuf = nullptr;
  }
}

// State of the persistent decode-step kernel (decode_step.cu).
void setup_step(fg_llama *m) {
  Ctx &c = *m->ctx;
  const int L = (int)m->layers.size(), d = m->d, G = m->Hq_l / m->Hkv_l;
  std::vector<StepLayer> sl(L);
  for (int l = 0; l < L; ++l) {
    const LayerW &w = m->layers[l];
    sl[l] = StepLayer{w.qkv, w.o, w.gateup, w.down, w.attn_norm, w.ffn_norm, w.k, w.v};
  }
  StepArgs &A = m->step_args;
  A = StepArgs{};
  StepLayer *dl = (StepLayer *)m->dalloc(sizeof(StepLayer) * std::max(L, 1));
  if (L) c.h2d(dl, sl.data(), sizeof(StepLayer) * L);
  const int P = decode_step_vctas(c.num_sms);
  const int smax = std::max(1, P / m->Hkv_l);
  A.attn_part = (float *)m->dalloc((uint64_t)m->Hkv_l * smax * G * (d + 2) * 4);
  A.attn_cnt = (unsigned long long *)m->dalloc((uint64_t)m->Hkv_l * 8);
  FG_CUDA(cudaMemsetAsync(A.attn_cnt, 0, (uint64_t)m->Hkv_l * 8, c.stream));
  A.bar = (unsigned long long *)m->dalloc(kStepBarBytes);
  FG_CUDA(cudaMemsetAsync(A.bar, 0, kStepBarBytes, c.stream));
  A.argkey = (unsigned long long *)m->dalloc(8);
  FG_CUDA(cudaMemsetAsync(A.argkey, 0, 8, c.stream));
  A.layers = dl;
  A.L = L;
  A.lm_head = m->lm_head;
  A.norm = m->norm;
  A.embed = m->embed;
  A.vocab = m->cfg.vocab_size;
  A.H = m->H;
  A.d = d;
  A.Hq = m->Hq_l;
  A.Hkv = m->Hkv_l;
  A.I = m->I_l;
  A.cap = m->cap;
  A.eps = m->cfg.rms_norm_eps;
  A.scale = (float)(1.0 / std::sqrt((double)d));
  A.inv_freq = m->inv_freq;
  A.h = m->h;
  A.q = m->q;
  A.att = m->att;
  A.ffn = m->ffn;
  A.logits = m->logits;
  A.ids = m->ids;
  A.pos = m->pos;
  A.token_log = m->token_log;
  A.step = m->step;
  A.log_steps = m->log_steps;
  A.gs = c.gemv;
  A.err = c.gemv.err;
  A.xarea_bytes = decode_step_xarea(d, G, m->H, m->I_l, (int64_t)m->Hq_l * d);
  {  // tensor maps of the K and V caches (the step kernel's attention tiles: 32 keys x 64 dims per box)
    std::vector<CUtensorMap> maps(2 * std::max(L, 1));
    for (int l = 0; l < L; ++l) {
      const LayerW &w = m->layers[l];
      for (int kv = 0; kv < 2; ++kv)
        maps[2 * l + kv] = make_tmap_3d(kv ? (const void *)w.v : (const void *)w.k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                        (uint64_t)d, (uint64_t)m->cap, (uint64_t)m->Hkv_l, (uint64_t)d * 2,
                                        (uint64_t)m->cap * d * 2, 64, 32, 1, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    void *dm = m->dalloc(sizeof(CUtensorMap) * maps.size());
    FG_REQUIRE(((uintptr_t)dm & 63) == 0, FG_ERR_DEVICE, "decode step: tensor maps must be 64-byte aligned");
    c.h2d(dm, maps.data(), sizeof(CUtensorMap) * maps.size());
    A.kv_maps = dm;
  }
  A.vocab_l = m->V_l;
  A.vbase = m->rank * m->V_l;
  A.tp = m->tp;
  A.rank = m->rank;
  if (m->tp > 1) setup_exchange(m);
  m->use_step = true;
}

}  // namespace

extern "C" {

int fg_llama_create(fg_ctx *ctx_h, const fg_llama_config *cfg, fg_llama **out);
int fg_llama_destroy(fg_llama *m);

}  // extern "C"

// The C entry points share the error plumbing of capi.cu through these two
// small shims (fg_ctx is defined there as a wrapper around Ctx).
struct fg_ctx {
  Ctx c;
};
namespace fg {
extern thread_local std::string g_last_error;
}
namespace {
int set_err(int st, const char *msg) {
  fg::g_last_error = msg;
  return st;
}
}  // namespace

#define FG_LAPI_BEGIN try {
#define FG_LAPI_END                                                  \
  }                                                                  \
  catch (const fg::Error &e) {                                       \
    return set_err(e.status, e.what());                              \
  }                                                                  \
  catch (const std::bad_alloc &) {                                   \
    return set_err(FG_ERR_OUT_OF_MEMORY, "host allocation failed");  \
  }                                                                  \
  catch (const std::exception &e) {                                  \
    return set_err(FG_ERR_INTERNAL_GPU, e.what());                   \
  }                                                                  \
  return FG_OK;

namespace {
std::recursive_mutex &model_mutex(fg_llama *m) {
  FG_REQUIRE(m != nullptr, FG_ERR_VALIDATION, "null model");
  return m->ctx->mu;
}
struct LGuard {
  std::lock_guard<std::recursive_mutex> lk;
  explicit LGuard(fg_llama *m) : lk(model_mutex(m)) {
    FG_REQUIRE(!m->ctx->lost, FG_ERR_DEVICE_LOST, "device lost; re-initialise the context");
    FG_CUDA(cudaSetDevice(m->ctx->device));
  }
};
}  // namespace

extern "C" {

int fg_llama_create(fg_ctx *ctx_h, const fg_llama_config *cfg, fg_llama **out) {
  FG_LAPI_BEGIN
  FG_REQUIRE(ctx_h && cfg && out, FG_ERR_VALIDATION, "fg_llama_create: null argument");
  Ctx &c = ctx_h->c;
  std::lock_guard<std::recursive_mutex> lk(c.mu);
  FG_CUDA(cudaSetDevice(c.device));
  const fg_llama_config &k = *cfg;
  FG_REQUIRE(k.qtype == FG_Q4_0 || k.qtype == FG_Q8_0 || k.qtype == FG_Q4_K, FG_ERR_DTYPE,
             "llama: qtype must be Q4_0, Q8_0 or Q4_K (a k-quant model whose Linears are Q4_K / Q6_K)");
  FG_REQUIRE(k.qtype != FG_Q4_K || c.tp_size == 1, FG_ERR_UNSUPPORTED_OP,
             "llama: k-quant models run on one GPU (no tensor parallelism)");
  FG_REQUIRE(k.qtype != FG_Q4_K || (k.hidden_size % 256 == 0 && k.intermediate_size % 256 == 0), FG_ERR_SHAPE,
             "llama: k-quant models need hidden and intermediate sizes that are multiples of 256");
  FG_REQUIRE(k.num_attention_heads > 0 && k.num_key_value_heads > 0 &&
                 k.num_attention_heads % k.num_key_value_heads == 0 && k.hidden_size % k.num_attention_heads == 0,
             FG_ERR_VALIDATION, "num_attention_heads (%d) must be divisible by num_key_value_heads (%d)",
             k.num_attention_heads, k.num_key_value_heads);
  const int tp = c.tp_size;
  const int d = k.hidden_size / k.num_attention_heads;
  FG_REQUIRE(d % 2 == 0 && d <= 256, FG_ERR_SHAPE, "head_dim %d must be even and <= 256", d);
  FG_REQUIRE(k.num_key_value_heads % tp == 0 && k.intermediate_size % tp == 0 && k.vocab_size % tp == 0, FG_ERR_SHAPE,
             "tensor parallel %d must divide KV heads (%d), intermediate (%d) and vocab (%d)", tp,
             k.num_key_value_heads, k.intermediate_size, k.vocab_size);
  FG_REQUIRE(k.hidden_size % 32 == 0 && (k.intermediate_size / tp) % 32 == 0 &&
                 (k.num_attention_heads / tp * d) % 32 == 0,
             FG_ERR_SHAPE, "shard widths must be multiples of the 32-value quant block");
  FG_REQUIRE(k.max_position_embeddings > 0 && k.max_batch > 0, FG_ERR_VALIDATION, "bad cache capacity / batch");
  std::unique_ptr<fg_llama> m(new fg_llama);
  m->ctx_handle = ctx_h;
  m->ctx = &c;
  m->cfg = k;
  m->tp = tp;
  m->rank = c.tp_rank;
  m->d = d;
  m->H = k.hidden_size;
  m->Hq_l = k.num_attention_heads / tp;
  m->Hkv_l = k.num_key_value_heads / tp;
  m->I_l = k.intermediate_size / tp;
  m->V_l = k.vocab_size / tp;
  m->cap = k.max_position_embeddings;
  m->max_batch = k.max_batch;
  m->m_max = std::max(k.max_batch, 2048);
  const int L = k.num_hidden_layers, H = k.hidden_size, qt = k.qtype;
  m->kq = qt == FG_Q4_K;
  try {
    m->embed = (__half *)m->dalloc((uint64_t)k.vocab_size * H * 2);
    m->norm = (float *)m->dalloc((uint64_t)H * 4);
    if (!m->kq) m->lm_head = make_qmat(m.get(), qt, m->V_l, H);
    m->layers.resize(L);
    const uint64_t kv_elems = (uint64_t)m->max_batch * m->Hkv_l * m->cap * d;
    for (int l = 0; l < L; ++l) {
      LayerW &w = m->layers[l];
      w.attn_norm = (float *)m->dalloc((uint64_t)H * 4);
      w.ffn_norm = (float *)m->dalloc((uint64_t)H * 4);
      if (!m->kq) {
        w.qkv = make_qmat(m.get(), qt, (int64_t)(m->Hq_l + 2 * m->Hkv_l) * d, H);
        w.o = make_qmat(m.get(), qt, H, (int64_t)m->Hq_l * d);
        w.gateup = make_qmat(m.get(), qt, 2LL * m->I_l, H);
        w.down = make_qmat(m.get(), qt, H, m->I_l);
      }
      w.k = (__half *)m->dalloc(kv_elems * 2);
      w.v = (__half *)m->dalloc(kv_elems * 2);
      // finite past the live length: the tensor-core attention reads whole 128-key blocks (masked)
      FG_CUDA(cudaMemsetAsync(w.k, 0, kv_elems * 2, c.stream));
      FG_CUDA(cudaMemsetAsync(w.v, 0, kv_elems * 2, c.stream));
    }
    std::vector<float> inv(d / 2);
    for (int p = 0; p < d / 2; ++p) inv[p] = (float)std::pow((double)k.rope_theta, -2.0 * (double)p / (double)d);
    m->inv_freq = (float *)m->dalloc((uint64_t)d / 2 * 4);
    c.h2d(m->inv_freq, inv.data(), inv.size() * 4);
    m->pos = (int *)m->dalloc((uint64_t)m->max_batch * 4);
    FG_CUDA(cudaMemsetAsync(m->pos, 0, (uint64_t)m->max_batch * 4, c.stream));
    m->ids = (int32_t *)m->dalloc((uint64_t)m->m_max * 4);
    m->keys = (unsigned long long *)m->dalloc((uint64_t)m->max_batch * 8);
    const int64_t mm = m->m_max;
    m->h = (float *)m->dalloc((uint64_t)mm * H * 4);
    m->xn = (float *)m->dalloc((uint64_t)mm * (uint64_t)std::max<int>(H, m->I_l) * 4);
    m->q = (float *)m->dalloc((uint64_t)mm * m->Hq_l * d * 4);
    m->att = (float *)m->dalloc((uint64_t)mm * m->Hq_l * d * 4);
    m->ffn = (float *)m->dalloc((uint64_t)mm * m->I_l * 4);
    m->logits = (float *)m->dalloc((uint64_t)m->max_batch * m->V_l * 4);
    if (m->kq) {
      const int64_t cols = std::max<int64_t>(std::max<int64_t>((int64_t)(m->Hq_l + 2 * m->Hkv_l) * d, 2LL * m->I_l), H);
      m->kq_tmp = (float *)m->dalloc((uint64_t)mm * cols * 4);
    }
    if (tp > 1) m->logits_all = (float *)m->dalloc((uint64_t)tp * m->max_batch * m->V_l * 4);
    // decode attention scratch, sized for the largest batch and full cache
    const LayerW empty_layer{};
    AttnArgs a = attn_args(m.get(), m->layers.empty() ? empty_layer : m->layers[0], m->max_batch, 1);
    m->decode_splits = attn_decode_splits(a, m->cap, c.num_sms);
    const uint64_t sb = attn_decode_scratch_bytes(a, m->decode_splits);
    if (sb) {
      m->attn_scratch = m->dalloc(sb);
      FG_CUDA(cudaMemsetAsync(m->attn_scratch, 0, sb, c.stream));
    }
    m->log_steps = 1 << 16;
    m->token_log = (int32_t *)m->dalloc((uint64_t)m->log_steps * m->max_batch * 4);
    m->step = (int *)m->dalloc(4);
    FG_CUDA(cudaMemsetAsync(m->step, 0, 4, c.stream));
    // fp16 activations of the tensor-core GEMM, sized for the largest prefill chunk
    c.ensure_xh(tc_xh_elems(m->m_max, std::max(std::max(H, m->I_l), m->Hq_l * d)));
    // Batch-1 decode runs as one persistent kernel per token where it applies
    // (FORGE_B200_DECODE=layered keeps the per-layer kernels, for comparison).
    const char *mode = std::getenv("FORGE_B200_DECODE");
    if (!m->kq && !(mode && std::string(mode) == "layered") &&
        decode_step_supported(d, m->Hq_l / m->Hkv_l, qt, H, m->I_l, (int64_t)m->Hq_l * d))
      setup_step(m.get());
  } catch (...) {
    c.sync();
    release_exchange(m.get());
    for (auto &p : m->allocs) c.free_async(p.first, p.second);
    throw;
  }
  *out = m.release();
  FG_LAPI_END
}

int fg_llama_destroy(fg_llama *m) {
  if (!m) return FG_OK;
  FG_LAPI_BEGIN
  {
    LGuard g(m);
    for (auto &kv : m->graphs) cudaGraphExecDestroy(kv.second);
    m->graphs.clear();
    m->ctx->sync();
    release_exchange(m);
    for (auto &p : m->allocs) m->ctx->free_async(p.first, p.second);
    m->ctx->sync();
  }
  delete m;
  FG_LAPI_END
}

int fg_llama_synthesize(fg_llama *m, uint64_t seed, float stdv) {
  FG_LAPI_BEGIN
  LGuard g(m);
  FG_REQUIRE(!m->kq, FG_ERR_UNSUPPORTED_OP,
             "llama: a k-quant model loads its Linears (fg_llama_load / fg_llama_load_gguf); no synthetic recipe");
  Ctx &c = *m->ctx;
  const auto &k = m->cfg;
  const int H = k.hidden_size, d = m->d, qt = k.qtype, r = m->rank;
  launch_synth_normal(tensor_seed(seed, kGlobal, G_EMBED), 0, (int64_t)k.vocab_size * H, 0.0f, stdv, FG_F16, m->embed,
                      c.stream);
  launch_synth_normal(tensor_seed(seed, kGlobal, G_NORM), 0, H, 1.0f, 0.1f, FG_F32, m->norm, c.stream);
  launch_synth_quant(qt, m->V_l, H, tensor_seed(seed, kGlobal, G_LM_HEAD), (int64_t)r * m->V_l, 0, H, stdv, m->lm_head,
                     1, 0, c.stream);
  const int nq = m->Hq_l * d, nkv = m->Hkv_l * d;
  for (int l = 0; l < k.num_hidden_layers; ++l) {
    LayerW &w = m->layers[l];
    launch_synth_normal(tensor_seed(seed, l, T_ATTN_NORM), 0, H, 1.0f, 0.1f, FG_F32, w.attn_norm, c.stream);
    launch_synth_normal(tensor_seed(seed, l, T_FFN_NORM), 0, H, 1.0f, 0.1f, FG_F32, w.ffn_norm, c.stream);
    launch_synth_quant(qt, nq, H, tensor_seed(seed, l, T_Q), (int64_t)r * nq, 0, H, stdv, w.qkv, 1, 0, c.stream);
    launch_synth_quant(qt, nkv, H, tensor_seed(seed, l, T_K), (int64_t)r * nkv, 0, H, stdv, w.qkv, 1, nq, c.stream);
    launch_synth_quant(qt, nkv, H, tensor_seed(seed, l, T_V), (int64_t)r * nkv, 0, H, stdv, w.qkv, 1, nq + nkv,
                       c.stream);
    launch_synth_quant(qt, H, nq, tensor_seed(seed, l, T_O), 0, (int64_t)r * nq, (int64_t)k.num_attention_heads * d,
                       stdv, w.o, 1, 0, c.stream);
    launch_synth_quant(qt, m->I_l, H, tensor_seed(seed, l, T_GATE), (int64_t)r * m->I_l, 0, H, stdv, w.gateup, 2, 0,
                       c.stream);
    launch_synth_quant(qt, m->I_l, H, tensor_seed(seed, l, T_UP), (int64_t)r * m->I_l, 0, H, stdv, w.gateup, 2, 1,
                       c.stream);
    launch_synth_quant(qt, H, m->I_l, tensor_seed(seed, l, T_DOWN), 0, (int64_t)r * m->I_l, k.intermediate_size, stdv,
                       w.down, 1, 0, c.stream);
  }
  c.sync();
  FG_LAPI_END
}

int fg_llama_load(fg_llama *m, const char *name, int32_t layer, const void *host, uint64_t bytes) {
  FG_LAPI_BEGIN
  LGuard g(m);
  Ctx &c = *m->ctx;
  const auto &k = m->cfg;
  const int H = k.hidden_size, d = m->d, qt = k.qtype, r = m->rank;
  const std::string n = name ? name : "";
  const int bb = gguf_block_bytes(qt);
  auto put_f32 = [&](float *dst, int64_t count) {
    FG_REQUIRE(bytes == (uint64_t)count * 4, FG_ERR_SHAPE, "%s: expected %lld float32 values", n.c_str(), (long long)count);
    c.h2d(dst, host, bytes);
  };
  // Row slice [row0, row0+rows) x column slice [col0, col0+cols) of a full
  // GGUF matrix [full_rows, full_cols] into rows r*rs+ro of dst.
  auto put_quant = [&](const QMat &dst, int64_t full_rows, int64_t full_cols, int64_t row0, int64_t rows, int64_t col0,
                       int64_t cols, int64_t rs, int64_t ro) {
    const uint64_t need = (uint64_t)full_rows * (full_cols / 32) * bb;
    FG_REQUIRE(bytes == need, FG_ERR_SHAPE, "%s: expected %llu GGUF bytes for [%lld, %lld], got %llu", n.c_str(),
               (unsigned long long)need, (long long)full_rows, (long long)full_cols, (unsigned long long)bytes);
    std::vector<uint8_t> shard((size_t)rows * (cols / 32) * bb);
    const uint8_t *src = (const uint8_t *)host;
    for (int64_t i = 0; i < rows; ++i)
      std::memcpy(shard.data() + (size_t)i * (cols / 32) * bb,
                  src + ((size_t)(row0 + i) * (full_cols / 32) + col0 / 32) * bb, (size_t)(cols / 32) * bb);
    void *tmp = c.alloc(shard.size());
    c.h2d(tmp, shard.data(), shard.size());
    launch_gguf_to_device((const uint8_t *)tmp, qt, rows, cols, dst, rs, ro, c.stream);
    c.free_async(tmp, shard.size());
  };
  const int nq = m->Hq_l * d, nkv = m->Hkv_l * d;
  const int Hq = k.num_attention_heads, Hkv = k.num_key_value_heads;
  if (m->kq && n != "embed" && n != "norm" && n != "attn_norm" && n != "ffn_norm") {
    // a k-quant Linear, as GGUF Q4_K or Q6_K blocks: the type follows from the byte count
    KQ *w = nullptr;
    int64_t N = 0, K = H;
    if (n == "lm_head") {
      w = &m->lm_kq, N = k.vocab_size;
    } else {
      FG_REQUIRE(layer >= 0 && layer < k.num_hidden_layers, FG_ERR_VALIDATION, "%s: layer %d out of range",
                 n.c_str(), layer);
      LayerW &L = m->layers[layer];
      if (n == "q") w = &L.kq[KQ_Q], N = nq;
      else if (n == "k") w = &L.kq[KQ_K], N = nkv;
      else if (n == "v") w = &L.kq[KQ_V], N = nkv;
      else if (n == "o") w = &L.kq[KQ_O], N = H, K = nq;
      else if (n == "gate") w = &L.kq[KQ_GATE], N = m->I_l;
      else if (n == "up") w = &L.kq[KQ_UP], N = m->I_l;
      else if (n == "down") w = &L.kq[KQ_DOWN], N = H, K = m->I_l;
      else raise(FG_ERR_VALIDATION, "unknown weight name '%s'", n.c_str());
    }
    const uint64_t sb = (uint64_t)N * (K / 256);
    const int type = bytes == sb * 144 ? FG_Q4_K : bytes == sb * 210 ? FG_Q6_K : -1;
    FG_REQUIRE(type >= 0 && K % 256 == 0, FG_ERR_SHAPE,
               "%s: a k-quant model takes Q4_K (%llu bytes) or Q6_K (%llu bytes) blocks of [%lld, %lld], got %llu",
               n.c_str(), (unsigned long long)(sb * 144), (unsigned long long)(sb * 210), (long long)N, (long long)K,
               (unsigned long long)bytes);
    if (!w->p || w->type != type) w->p = m->dalloc(bytes);
    w->type = type;
    w->N = N;
    w->K = K;
    c.h2d(w->p, host, bytes);
    c.sync();
    return FG_OK;
  }
  if (n == "embed") {
    FG_REQUIRE(bytes == (uint64_t)k.vocab_size * H * 2, FG_ERR_SHAPE, "embed: expected float16 [%d, %d]", k.vocab_size, H);
    c.h2d(m->embed, host, bytes);
  } else if (n == "norm") {
    put_f32(m->norm, H);
  } else if (n == "lm_head") {
    put_quant(m->lm_head, k.vocab_size, H, (int64_t)r * m->V_l, m->V_l, 0, H, 1, 0);
  } else {
    FG_REQUIRE(layer >= 0 && layer < k.num_hidden_layers, FG_ERR_VALIDATION, "%s: layer %d out of range", n.c_str(), layer);
    LayerW &w = m->layers[layer];
    if (n == "attn_norm") put_f32(w.attn_norm, H);
    else if (n == "ffn_norm") put_f32(w.ffn_norm, H);
    else if (n == "q") put_quant(w.qkv, (int64_t)Hq * d, H, (int64_t)r * nq, nq, 0, H, 1, 0);
    else if (n == "k") put_quant(w.qkv, (int64_t)Hkv * d, H, (int64_t)r * nkv, nkv, 0, H, 1, nq);
    else if (n == "v") put_quant(w.qkv, (int64_t)Hkv * d, H, (int64_t)r * nkv, nkv, 0, H, 1, nq + nkv);
    else if (n == "o") put_quant(w.o, H, (int64_t)Hq * d, 0, H, (int64_t)r * nq, nq, 1, 0);
    else if (n == "gate") put_quant(w.gateup, k.intermediate_size, H, (int64_t)r * m->I_l, m->I_l, 0, H, 2, 0);
    else if (n == "up") put_quant(w.gateup, k.intermediate_size, H, (int64_t)r * m->I_l, m->I_l, 0, H, 2, 1);
    else if (n == "down") put_quant(w.down, H, k.intermediate_size, 0, H, (int64_t)r * m->I_l, m->I_l, 1, 0);
    else raise(FG_ERR_VALIDATION, "unknown weight name '%s'", n.c_str());
  }
  c.sync();
  FG_LAPI_END
}

int fg_llama_reset(fg_llama *m) {
  FG_LAPI_BEGIN
  LGuard g(m);
  FG_CUDA(cudaMemsetAsync(m->pos, 0, (uint64_t)m->max_batch * 4, m->ctx->stream));
  if (m->use_step) {  // the step kernel's barrier, argmax and merge counters start over too
    const StepArgs &A = m->step_args;
    FG_CUDA(cudaMemsetAsync(A.bar, 0, kStepBarBytes, m->ctx->stream));
    FG_CUDA(cudaMemsetAsync(A.argkey, 0, 8, m->ctx->stream));
    FG_CUDA(cudaMemsetAsync(A.attn_cnt, 0, (uint64_t)A.Hkv * 8, m->ctx->stream));
  }
  m->host_pos = 0;
  FG_LAPI_END
}

int fg_llama_set_position(fg_llama *m, int32_t batch, int32_t pos) {
  FG_LAPI_BEGIN
  LGuard g(m);
  FG_REQUIRE(batch >= 1 && batch <= m->max_batch, FG_ERR_SHAPE, "batch %d outside [1, %d]", batch, m->max_batch);
  FG_REQUIRE(pos >= 0 && pos < m->cap, FG_ERR_SHAPE, "position %d outside [0, %d)", pos, m->cap);
  std::vector<int32_t> p((size_t)m->max_batch, 0);
  for (int b = 0; b < batch; ++b) p[(size_t)b] = pos;
  m->ctx->h2d(m->pos, p.data(), p.size() * 4);
  m->host_pos = pos;
  FG_LAPI_END
}

}  // extern "C"

namespace {
// Positions [0, len) of one layer's K (or V) cache for sequences [0, B): element (b, h, p, c) of this rank's
// heads takes generator index ((b * Hkv_all + h0 + h) * len + p) * d + c, so every tensor-parallel rank
// writes its slice of the same global cache.
__global__ void k_synth_kv(uint64_t seed, int B, int Hkv_l, int Hkv_all, int h0, int len, int d, int cap,
                           float stdv, __half *cache) {
  const int64_t n = (int64_t)B * Hkv_l * len * d;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % d);
    const int64_t r = i / d;
    const int p = (int)(r % len);
    const int64_t bh = r / len;
    const int h = (int)(bh % Hkv_l), b = (int)(bh / Hkv_l);
    const uint64_t gi = ((uint64_t)((int64_t)b * Hkv_all + h0 + h) * len + p) * d + c;
    cache[(((int64_t)b * Hkv_l + h) * cap + p) * d + c] = __float2half_rn(__fadd_rn(__fmul_rn(normal01(seed, gi), stdv), 0.0f));
  }
}
}  // namespace

extern "C" {

int fg_llama_synthesize_kv(fg_llama *m, uint64_t seed, int32_t batch, int32_t len, float stdv) {
  FG_LAPI_BEGIN
  LGuard g(m);
  Ctx &c = *m->ctx;
  FG_REQUIRE(batch >= 1 && batch <= m->max_batch, FG_ERR_SHAPE, "batch %d outside [1, %d]", batch, m->max_batch);
  FG_REQUIRE(len >= 0 && len < m->cap, FG_ERR_SHAPE, "length %d outside [0, %d)", len, m->cap);
  const int64_t n = (int64_t)batch * m->Hkv_l * len * m->d;
  if (n > 0) {
    const int grid = (int)std::min<int64_t>(ceil_div(n, 256), (int64_t)c.num_sms * 16);
    for (int l = 0; l < (int)m->layers.size(); ++l) {
      const LayerW &w = m->layers[l];
      k_synth_kv<<<grid, 256, 0, c.stream>>>(tensor_seed(seed, l, 9), batch, m->Hkv_l, m->cfg.num_key_value_heads,
                                             m->rank * m->Hkv_l, len, m->d, m->cap, stdv, w.k);
      FG_LAUNCH_CHECK();
      k_synth_kv<<<grid, 256, 0, c.stream>>>(tensor_seed(seed, l, 10), batch, m->Hkv_l, m->cfg.num_key_value_heads,
                                             m->rank * m->Hkv_l, len, m->d, m->cap, stdv, w.v);
      FG_LAUNCH_CHECK();
    }
  }
  std::vector<int32_t> p((size_t)m->max_batch, 0);
  for (int b = 0; b < batch; ++b) p[(size_t)b] = len;
  c.h2d(m->pos, p.data(), p.size() * 4);
  m->host_pos = len;
  c.sync();
  FG_LAPI_END
}

int fg_llama_decode_path(fg_llama *m, int32_t batch, int32_t *kind) {
  FG_LAPI_BEGIN
  FG_REQUIRE(m && kind, FG_ERR_VALIDATION, "fg_llama_decode_path: null argument");
  FG_REQUIRE(batch >= 1 && batch <= m->max_batch, FG_ERR_SHAPE, "batch %d outside [1, %d]", batch, m->max_batch);
  *kind = (batch == 1 && m->use_step) ? 1 : 0;
  FG_LAPI_END
}

int fg_llama_position(fg_llama *m, int32_t *pos) {
  FG_LAPI_BEGIN
  *pos = m->host_pos;
  FG_LAPI_END
}

int fg_llama_forward(fg_llama *m, const int32_t *ids, int32_t batch, int32_t len, float *logits, int32_t *next_ids) {
  FG_LAPI_BEGIN
  LGuard g(m);
  Ctx &c = *m->ctx;
  FG_REQUIRE(batch >= 1 && batch <= m->max_batch, FG_ERR_SHAPE, "batch %d outside [1, %d]", batch, m->max_batch);
  FG_REQUIRE(len >= 1, FG_ERR_SHAPE, "forward needs at least one token");
  FG_REQUIRE(m->host_pos + len <= m->cap, FG_ERR_SHAPE, "KV cache capacity %d exceeded (%d + %d)", m->cap, m->host_pos, len);
  // chunk the sequence so that batch * chunk <= m_max
  const int chunk = std::max(1, m->m_max / batch);
  std::vector<int32_t> buf;
  for (int t0 = 0; t0 < len; t0 += chunk) {
    const int T = std::min(chunk, len - t0);
    buf.resize((size_t)batch * T);
    for (int b = 0; b < batch; ++b) std::memcpy(&buf[(size_t)b * T], ids + (size_t)b * len + t0, (size_t)T * 4);
    c.h2d(m->ids, buf.data(), buf.size() * 4);
    forward_tokens(m, batch, T, false);
    m->host_pos += T;
  }
  m->last_batch = batch;
  if (logits) read_logits(m, batch, logits);
  if (next_ids) c.d2h(next_ids, m->ids, (uint64_t)batch * 4);
  c.sync();
  FG_LAPI_END
}

static cudaGraphExec_t decode_graph(fg_llama *m, int B) {
  auto it = m->graphs.find(B);
  if (it != m->graphs.end()) return it->second;
  Ctx &c = *m->ctx;
  cudaGraph_t graph = nullptr;
  FG_CUDA(cudaStreamBeginCapture(c.stream, cudaStreamCaptureModeThreadLocal));
  try {
    if (B == 1 && m->use_step)
      launch_decode_step(m->step_args, c.num_sms, c.stream);
    else
      forward_tokens(m, B, 1, true);
  } catch (...) {
    cudaStreamEndCapture(c.stream, &graph);
    if (graph) cudaGraphDestroy(graph);
    throw;
  }
  FG_CUDA(cudaStreamEndCapture(c.stream, &graph));
  cudaGraphExec_t exec = nullptr;
  FG_CUDA(cudaGraphInstantiate(&exec, graph, 0));
  FG_CUDA(cudaGraphDestroy(graph));
  m->graphs[B] = exec;
  return exec;
}

int fg_llama_decode(fg_llama *m, const int32_t *ids, int32_t batch, int32_t *next_ids, float *logits) {
  FG_LAPI_BEGIN
  LGuard g(m);
  Ctx &c = *m->ctx;
  FG_REQUIRE(batch >= 1 && batch <= m->max_batch, FG_ERR_SHAPE, "batch %d outside [1, %d]", batch, m->max_batch);
  FG_REQUIRE(m->host_pos + 1 <= m->cap, FG_ERR_SHAPE, "KV cache capacity %d exceeded", m->cap);
  if (ids) c.h2d(m->ids, ids, (uint64_t)batch * 4);
  if (m->kq) {  // launched directly: the k-quant path may take pool scratch, which a captured graph cannot
    forward_tokens(m, batch, 1, true);
  } else {
    cudaGraphExec_t exec = decode_graph(m, batch);
    FG_CUDA(cudaGraphLaunch(exec, c.stream));
  }
  m->host_pos += 1;
  m->last_batch = batch;
  if (logits) read_logits(m, batch, logits);
  if (next_ids) {
    c.d2h_checked(next_ids, m->ids, (uint64_t)batch * 4);  // the tokens and the error word in one round trip
  } else if (logits) {
    c.check_device_error();
  }
  FG_LAPI_END
}

int fg_llama_generate_device(fg_llama *m, int32_t batch, int32_t steps) {
  FG_LAPI_BEGIN
  LGuard g(m);
  Ctx &c = *m->ctx;
  FG_REQUIRE(batch >= 1 && batch <= m->max_batch, FG_ERR_SHAPE, "batch %d outside [1, %d]", batch, m->max_batch);
  FG_REQUIRE(steps >= 0 && steps <= m->log_steps, FG_ERR_SHAPE, "steps %d outside [0, %d]", steps, m->log_steps);
  FG_REQUIRE(m->host_pos + steps <= m->cap, FG_ERR_SHAPE, "KV cache capacity %d exceeded", m->cap);
  FG_CUDA(cudaMemsetAsync(m->step, 0, 4, c.stream));
  if (m->kq) {
    for (int s = 0; s < steps; ++s) forward_tokens(m, batch, 1, true);
  } else {
    cudaGraphExec_t exec = decode_graph(m, batch);
    for (int s = 0; s < steps; ++s) FG_CUDA(cudaGraphLaunch(exec, c.stream));
  }
  m->host_pos += steps;
  m->last_batch = batch;
  FG_LAPI_END
}

int fg_llama_get_config(fg_llama *m, fg_llama_config *cfg) {
  FG_LAPI_BEGIN
  FG_REQUIRE(m && cfg, FG_ERR_VALIDATION, "fg_llama_get_config: null argument");
  *cfg = m->cfg;
  FG_LAPI_END
}

int fg_llama_tokens(fg_llama *m, int32_t *host, int64_t count) {
  FG_LAPI_BEGIN
  LGuard g(m);
  FG_REQUIRE(count >= 0 && count <= (int64_t)m->log_steps * m->max_batch, FG_ERR_SHAPE, "token count out of range");
  m->ctx->d2h(host, m->token_log, (uint64_t)count * 4);
  m->ctx->check_device_error();
  FG_LAPI_END
}

}  // extern "C"
