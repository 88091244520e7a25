// Context, tensor registry, stream-ordered allocator with quota, pinned
// staging, and the extern "C" entry points of include/forge_b200.h.
//
// Replaces the reference's WebGPU backend: device singleton (packages/forge/
// src/webgpu/device.ts:77-201), buffer pool and staging ring (buffers.ts:
// 24-242), quota manager (quota.ts:65-313) and tensor registry
// (packages/forge/src/tensor/tensorRegistry.ts:24-255).
#include "nccl_dyn.cuh"

#include <cmath>
#include <cstring>
#include <map>
#include <memory>

#include "runtime.cuh"

namespace fg {

thread_local std::string g_last_error;

uint64_t dtype_bytes(int dtype, int64_t numel, const int64_t *shape, int ndim) {
  switch (dtype) {
    case FG_F32:
    case FG_I32:
    case FG_U32:
      return 4ull * (uint64_t)numel;
    case FG_F16:
      return 2ull * (uint64_t)numel;
    case FG_U8:
      return (uint64_t)numel;
    case FG_Q4_0:
    case FG_Q8_0:
      FG_REQUIRE(ndim == 2 && shape[1] % 32 == 0, FG_ERR_SHAPE, "quantized tensors are [rows, cols] with cols %% 32 == 0");
      return qmat_bytes(dtype, shape[0], shape[1]);
    case FG_Q4_K:
    case FG_Q6_K:
      FG_REQUIRE(ndim == 2 && shape[1] % 256 == 0, FG_ERR_SHAPE, "k-quant tensors are [rows, cols] with cols %% 256 == 0");
      return (uint64_t)shape[0] * (uint64_t)(shape[1] / 256) * (dtype == FG_Q4_K ? 144ull : 210ull);
    default:
      raise(FG_ERR_DTYPE, "unknown dtype %d", dtype);
  }
}

void *Ctx::alloc(uint64_t bytes) {
  const uint64_t req = std::max<uint64_t>(align_up(bytes, 256), 256);
  if (active + req > limit)
    raise(FG_ERR_QUOTA_EXCEEDED, "VRAM quota exceeded: requested %llu bytes, active %llu, limit %llu",
          (unsigned long long)req, (unsigned long long)active, (unsigned long long)limit);
  void *p = nullptr;
  cudaError_t e = cudaMallocFromPoolAsync(&p, req, pool, stream);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    raise(FG_ERR_OUT_OF_MEMORY, "device allocation of %llu bytes failed", (unsigned long long)req);
  }
  FG_CUDA(e);
  active += req;
  peak = std::max(peak, active);
  return p;
}

void Ctx::free_async(void *p, uint64_t bytes) {
  if (!p) return;
  const uint64_t req = std::max<uint64_t>(align_up(bytes, 256), 256);
  FG_CUDA(cudaFreeAsync(p, stream));
  active -= std::min(active, req);
  pending += req;
}

fg_handle Ctx::add(const Tensor &t) {
  const fg_handle h = (epoch << 40) | (next_id++ & ((1ull << 40) - 1));
  tensors[h] = t;
  return h;
}

Tensor &Ctx::peek(fg_handle h) {
  if (h != 0 && (h >> 40) != epoch) raise(FG_ERR_STALE_HANDLE, "Stale tensor handle from a previous device: tensor_%llx", (unsigned long long)h);
  auto it = tensors.find(h);
  if (it == tensors.end()) raise(FG_ERR_DISPOSED, "Tensor not found: tensor_%llx", (unsigned long long)h);
  return it->second;
}

Tensor &Ctx::get(fg_handle h) {
  Tensor &t = peek(h);
  if (t.lazy) materialize(h, t);
  return t;
}

fg_handle Ctx::make(const int64_t *shape, int ndim, int dtype, Tensor **out) {
  FG_REQUIRE(ndim >= 0 && ndim <= FG_MAX_DIMS, FG_ERR_SHAPE, "rank %d outside [0, %d]", ndim, FG_MAX_DIMS);
  Tensor t;
  t.dtype = dtype;
  t.ndim = ndim;
  for (int i = 0; i < ndim; ++i) {
    FG_REQUIRE(shape[i] >= 0, FG_ERR_SHAPE, "negative dimension %lld", (long long)shape[i]);
    t.shape[i] = shape[i];
  }
  t.bytes = dtype_bytes(dtype, t.numel(), t.shape, ndim);
  t.ptr = alloc(t.bytes);
  const fg_handle h = add(t);
  if (out) *out = &tensors[h];
  return h;
}

void Ctx::dispose(fg_handle h) {
  if (h == 0 || (h >> 40) != epoch) return;
  auto it = tensors.find(h);
  if (it == tensors.end()) return;  // double dispose is a no-op (tensorRegistry.ts:137-139)
  // lazy tensors that read h take their values now
  std::vector<fg_handle> users;
  for (auto r = lazy_users.equal_range(h); r.first != r.second; ++r.first) users.push_back(r.first->second);
  for (fg_handle u : users) get(u);
  it = tensors.find(h);
  if (it->second.lazy) {  // an unread lazy tensor: drop its link to the source
    for (auto r = lazy_users.equal_range(it->second.lazy->src); r.first != r.second; ++r.first)
      if (r.first->second == h) {
        lazy_users.erase(r.first);
        break;
      }
  }
  free_async(it->second.ptr, it->second.bytes);
  tensors.erase(it);
}

void Ctx::h2d(void *dst, const void *src, uint64_t bytes) {
  uint64_t off = 0;
  int i = 0;
  while (off < bytes) {
    const uint64_t n = std::min(staging_bytes, bytes - off);
    FG_CUDA(cudaEventSynchronize(staging_ev[i]));  // previous DMA out of this half is done
    std::memcpy(staging[i], (const char *)src + off, n);
    FG_CUDA(cudaMemcpyAsync((char *)dst + off, staging[i], n, cudaMemcpyHostToDevice, stream));
    FG_CUDA(cudaEventRecord(staging_ev[i], stream));
    off += n;
    i ^= 1;
  }
}

void Ctx::d2h(void *dst, const void *src, uint64_t bytes) {
  uint64_t off = 0;
  while (off < bytes) {
    const uint64_t n = std::min(staging_bytes, bytes - off);
    FG_CUDA(cudaMemcpyAsync(staging[0], (const char *)src + off, n, cudaMemcpyDeviceToHost, stream));
    FG_CUDA(cudaStreamSynchronize(stream));
    std::memcpy((char *)dst + off, staging[0], n);
    off += n;
  }
  pending = 0;
}

void Ctx::sync() {
  FG_CUDA(cudaStreamSynchronize(stream));
  pending = 0;
  check_device_error();
}

void Ctx::ensure_xh(uint64_t elems) {
  if (elems <= gemv.xh_elems) return;
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  FG_CUDA(cudaStreamIsCapturing(stream, &st));
  FG_REQUIRE(st == cudaStreamCaptureStatusNone, FG_ERR_VALIDATION,
             "GEMM activation scratch must grow outside stream capture (run the shape once before capturing)");
  if (gemv.xh) free_async(gemv.xh, gemv.xh_elems * 2);
  gemv.xh = nullptr;
  gemv.xh_elems = 0;
  const uint64_t n = align_up(elems, 1u << 16);
  gemv.xh = (__half *)alloc(n * 2);
  gemv.xh_elems = n;
}

void Ctx::check_device_error() {
  if (!gemv.err) return;
  int e = 0;
  FG_CUDA(cudaMemcpy(&e, gemv.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e != 0) {
    int zero = 0;
    FG_CUDA(cudaMemcpy(gemv.err, &zero, sizeof(int), cudaMemcpyHostToDevice));
    raise(FG_ERR_INTERNAL_GPU, "a kernel wait timed out on the device (code %d); results of the step are invalid", e);
  }
}

void Ctx::d2h_checked(void *dst, const void *src, uint64_t bytes) {
  const uint64_t eoff = align_up(bytes, 16);
  if (!gemv.err || eoff + sizeof(int) > staging_bytes) {
    d2h(dst, src, bytes);
    check_device_error();
    return;
  }
  FG_CUDA(cudaMemcpyAsync(staging[0], src, bytes, cudaMemcpyDeviceToHost, stream));
  FG_CUDA(cudaMemcpyAsync((char *)staging[0] + eoff, gemv.err, sizeof(int), cudaMemcpyDeviceToHost, stream));
  FG_CUDA(cudaStreamSynchronize(stream));
  std::memcpy(dst, staging[0], bytes);
  pending = 0;
  int e = 0;
  std::memcpy(&e, (const char *)staging[0] + eoff, sizeof(int));
  if (e != 0) {
    int zero = 0;
    FG_CUDA(cudaMemcpy(gemv.err, &zero, sizeof(int), cudaMemcpyHostToDevice));
    raise(FG_ERR_INTERNAL_GPU, "a kernel wait timed out on the device (code %d); results of the step are invalid", e);
  }
}

// inv_freq tables for standalone RoPE calls, cached per (base, d).
struct RopeCache {
  std::map<std::pair<float, int64_t>, float *> tables;
};
static std::map<Ctx *, RopeCache> g_rope;

const float *rope_table(Ctx *c, float base, int64_t d) {
  auto &rc = g_rope[c];
  auto key = std::make_pair(base, d);
  auto it = rc.tables.find(key);
  if (it != rc.tables.end()) return it->second;
  std::vector<float> t(d / 2);
  for (int64_t p = 0; p < d / 2; ++p) t[p] = (float)std::pow((double)base, -2.0 * (double)p / (double)d);
  float *dp = (float *)c->alloc(t.size() * 4);
  c->h2d(dp, t.data(), t.size() * 4);
  rc.tables[key] = dp;
  return dp;
}

}  // namespace fg

using namespace fg;

struct fg_ctx {
  Ctx c;
};

namespace {

int set_error(int status, const char *msg) {
  g_last_error = msg;
  return status;
}

#define FG_API_BEGIN try {
#define FG_API_END                                                       \
  }                                                                      \
  catch (const fg::Error &e) {                                           \
    return set_error(e.status, e.what());                                \
  }                                                                      \
  catch (const std::bad_alloc &) {                                       \
    return set_error(FG_ERR_OUT_OF_MEMORY, "host allocation failed");    \
  }                                                                      \
  catch (const std::exception &e) {                                      \
    return set_error(FG_ERR_INTERNAL_GPU, e.what());                     \
  }                                                                      \
  return FG_OK;

std::recursive_mutex &ctx_mutex(fg_ctx *ctx) {
  FG_REQUIRE(ctx != nullptr, FG_ERR_VALIDATION, "null context");
  return ctx->c.mu;
}

struct Guard {  // serialise calls on a context and select its device
  std::lock_guard<std::recursive_mutex> lk;
  explicit Guard(fg_ctx *ctx) : lk(ctx_mutex(ctx)) {
    FG_REQUIRE(!ctx->c.lost, FG_ERR_DEVICE_LOST, "device lost; re-initialise the context");
    FG_CUDA(cudaSetDevice(ctx->c.device));
  }
};

Ctx &C(fg_ctx *ctx) {
  FG_REQUIRE(ctx != nullptr, FG_ERR_VALIDATION, "null context");
  return ctx->c;
}

void check_f32(const Tensor &t, const char *what) {
  FG_REQUIRE(t.dtype == FG_F32, FG_ERR_DTYPE, "%s requires float32 tensors", what);
}

bool is_kquant(int dt) { return dt == FG_Q4_K || dt == FG_Q6_K; }  // 256-value super-blocks, GGUF order
bool is_quant(int dt) { return dt == FG_Q4_0 || dt == FG_Q8_0 || is_kquant(dt); }
uint64_t kquant_block_bytes(int dt) { return dt == FG_Q4_K ? 144 : 210; }

}  // namespace

extern "C" {

const char *fg_version(void) { return "forge_b200 0.1.0 (sm_100a)"; }

const char *fg_last_error(void) { return g_last_error.c_str(); }

const char *fg_status_name(int status) {
  switch (status) {
    case FG_OK: return "OK";
    case FG_ERR_SHAPE: return "AMEVAForgeShapeError";
    case FG_ERR_DTYPE: return "AMEVAForgeDTypeError";
    case FG_ERR_DEVICE: return "AMEVAForgeDeviceError";
    case FG_ERR_DISPOSED: return "AMEVAForgeDisposedError";
    case FG_ERR_QUOTA_EXCEEDED: return "AMEVAForgeQuotaExceededError";
    case FG_ERR_UNAVAILABLE: return "AMEVAForgeWebGPUUnavailableError";
    case FG_ERR_SECURITY: return "AMEVAForgeSecurityError";
    case FG_ERR_UNSUPPORTED_OP: return "AMEVAForgeUnsupportedOpError";
    case FG_ERR_VALIDATION: return "AMEVAForgeValidationError";
    case FG_ERR_OUT_OF_MEMORY: return "AMEVAForgeOutOfMemoryError";
    case FG_ERR_INTERNAL_GPU: return "AMEVAForgeInternalGPUError";
    case FG_ERR_DEVICE_LOST: return "AMEVAForgeDeviceLostError";
    case FG_ERR_STALE_HANDLE: return "AMEVAForgeStaleHandleError";
    default: return "AMEVAForgeError";
  }
}

int fg_device_count(int32_t *out) {
  FG_API_BEGIN
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  *out = n;
  FG_API_END
}

int fg_nccl_unique_id(uint8_t out[128]) {
  FG_API_BEGIN
  ncclUniqueId id;
  ncclResult_t r = nccl().GetUniqueId(&id);
  FG_REQUIRE(r == ncclSuccess, FG_ERR_DEVICE, "ncclGetUniqueId: %s", nccl().GetErrorString(r));
  static_assert(sizeof(id) == 128, "NCCL unique id size");
  std::memcpy(out, &id, 128);
  FG_API_END
}

int fg_init(const fg_init_opts *opts, fg_ctx **out) {
  FG_API_BEGIN
  FG_REQUIRE(opts && out, FG_ERR_VALIDATION, "fg_init: null argument");
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    raise(FG_ERR_UNAVAILABLE, "no CUDA device is available");
  }
  FG_REQUIRE(opts->device >= 0 && opts->device < n, FG_ERR_DEVICE, "device %d out of range (%d devices)", opts->device, n);
  FG_REQUIRE(opts->tp_size >= 1 && opts->tp_rank >= 0 && opts->tp_rank < opts->tp_size, FG_ERR_VALIDATION,
             "bad tensor-parallel rank %d / size %d", opts->tp_rank, opts->tp_size);
  cudaDeviceProp prop;
  FG_CUDA(cudaGetDeviceProperties(&prop, opts->device));
  FG_REQUIRE(prop.major == 10, FG_ERR_UNAVAILABLE, "forge_b200 needs an sm_100 (B200) device, found sm_%d%d", prop.major,
             prop.minor);
  std::unique_ptr<fg_ctx> ctx(new fg_ctx);
  Ctx &c = ctx->c;
  c.device = opts->device;
  c.tp_rank = opts->tp_rank;
  c.tp_size = opts->tp_size;
  c.num_sms = prop.multiProcessorCount;
  FG_CUDA(cudaSetDevice(c.device));
  FG_CUDA(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
  FG_CUDA(cudaDeviceGetDefaultMemPool(&c.pool, c.device));
  uint64_t thresh = UINT64_MAX;
  FG_CUDA(cudaMemPoolSetAttribute(c.pool, cudaMemPoolAttrReleaseThreshold, &thresh));
  size_t free_b = 0, total_b = 0;
  FG_CUDA(cudaMemGetInfo(&free_b, &total_b));
  c.limit = opts->vram_limit_bytes ? opts->vram_limit_bytes : (uint64_t)(0.92 * (double)free_b);
  c.staging_bytes = 32ull << 20;
  for (int i = 0; i < 2; ++i) {
    FG_CUDA(cudaHostAlloc(&c.staging[i], c.staging_bytes, cudaHostAllocDefault));
    FG_CUDA(cudaEventCreateWithFlags(&c.staging_ev[i], cudaEventDisableTiming));
    FG_CUDA(cudaEventRecord(c.staging_ev[i], c.stream));
  }
  {  // GEMV workspace: 4 Mi partial floats, 64 Ki tickets, the error word
    c.gemv.part_floats = 4ull << 20;
    c.gemv.n_tickets = 1 << 16;
    const uint64_t bytes = c.gemv.part_floats * 4 + (uint64_t)c.gemv.n_tickets * 4 + 256;
    char *p = (char *)c.alloc(bytes);
    FG_CUDA(cudaMemsetAsync(p, 0, bytes, c.stream));
    c.gemv.part = (float *)p;
    c.gemv.tickets = (int *)(p + c.gemv.part_floats * 4);
    c.gemv.err = (int *)(p + c.gemv.part_floats * 4 + (uint64_t)c.gemv.n_tickets * 4);
    FG_CUDA(cudaStreamSynchronize(c.stream));
  }
  if (c.tp_size > 1) {
    ncclUniqueId id;
    std::memcpy(&id, opts->nccl_id, 128);
    ncclComm_t comm = nullptr;
    ncclResult_t r = nccl().CommInitRank(&comm, c.tp_size, id, c.tp_rank);
    FG_REQUIRE(r == ncclSuccess, FG_ERR_DEVICE, "ncclCommInitRank(rank %d of %d): %s", c.tp_rank, c.tp_size,
               nccl().GetErrorString(r));
    c.nccl = (ncclComm *)comm;
  }
  *out = ctx.release();
  FG_API_END
}

int fg_shutdown(fg_ctx *ctx) {
  if (!ctx) return FG_OK;
  FG_API_BEGIN
  {
    std::lock_guard<std::recursive_mutex> lk(ctx->c.mu);
    Ctx &c = ctx->c;
    cudaSetDevice(c.device);
    cudaStreamSynchronize(c.stream);
    for (auto &kv : c.tensors)
      if (kv.second.ptr) cudaFreeAsync(kv.second.ptr, c.stream);
    c.lazy_users.clear();
    if (c.gemv.part) cudaFreeAsync(c.gemv.part, c.stream);
    if (c.gemv.xh) cudaFreeAsync(c.gemv.xh, c.stream);
    c.tensors.clear();
    auto it = g_rope.find(&c);
    if (it != g_rope.end()) {
      for (auto &t : it->second.tables) cudaFreeAsync(t.second, c.stream);
      g_rope.erase(it);
    }
    cudaStreamSynchronize(c.stream);
    if (c.nccl) nccl().CommDestroy((ncclComm_t)c.nccl);
    for (int i = 0; i < 2; ++i) {
      if (c.staging_ev[i]) cudaEventDestroy(c.staging_ev[i]);
      if (c.staging[i]) cudaFreeHost(c.staging[i]);
    }
    cudaStreamDestroy(c.stream);
  }
  delete ctx;
  FG_API_END
}

int fg_synchronize(fg_ctx *ctx) {
  FG_API_BEGIN
  Guard g(ctx);
  C(ctx).sync();
  FG_API_END
}

int fg_get_stream(fg_ctx *ctx, void **stream) {
  FG_API_BEGIN
  *stream = (void *)C(ctx).stream;
  FG_API_END
}

int fg_quota_snapshot(fg_ctx *ctx, fg_quota *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  out->limit_bytes = c.limit;
  out->active_bytes = c.active;
  out->pending_bytes = c.pending;
  out->peak_bytes = c.peak;
  out->live_tensors = c.tensors.size();
  FG_API_END
}

int fg_set_allow_non_finite(fg_ctx *ctx, int32_t allow) {
  FG_API_BEGIN
  Guard g(ctx);
  C(ctx).allow_non_finite = allow != 0;
  FG_API_END
}

int fg_upload(fg_ctx *ctx, const void *host, uint64_t bytes, const int64_t *shape, int32_t ndim, int32_t dtype,
              fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  FG_REQUIRE(out && (host || bytes == 0), FG_ERR_VALIDATION, "fg_upload: null argument");
  FG_REQUIRE(!is_quant(dtype), FG_ERR_DTYPE, "quantized weights go through fg_upload_quant");
  Tensor probe;
  probe.ndim = ndim;
  FG_REQUIRE(ndim >= 0 && ndim <= FG_MAX_DIMS, FG_ERR_SHAPE, "rank %d outside [0, %d]", ndim, FG_MAX_DIMS);
  for (int i = 0; i < ndim; ++i) probe.shape[i] = shape[i];
  const uint64_t need = dtype_bytes(dtype, probe.numel(), probe.shape, ndim);
  FG_REQUIRE(bytes == need, FG_ERR_SHAPE, "upload of %llu bytes does not match shape (%llu bytes)",
             (unsigned long long)bytes, (unsigned long long)need);
  if (dtype == FG_F32 && !c.allow_non_finite) {  // graphExecutor.ts:667-681
    const float *f = (const float *)host;
    for (int64_t i = 0, n = probe.numel(); i < n; ++i)
      if (!std::isfinite(f[i])) raise(FG_ERR_VALIDATION, "upload contains a non-finite value at element %lld", (long long)i);
  }
  Tensor *t = nullptr;
  const fg_handle h = c.make(shape, ndim, dtype, &t);
  c.h2d(t->ptr, host, bytes);
  *out = h;
  FG_API_END
}

int fg_upload_quant(fg_ctx *ctx, int32_t qtype, const void *gguf_blocks, uint64_t bytes, int64_t rows, int64_t cols,
                    fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  FG_REQUIRE(is_quant(qtype), FG_ERR_DTYPE, "fg_upload_quant: qtype must be Q4_0, Q8_0, Q4_K or Q6_K");
  if (is_kquant(qtype)) {  // GGUF order on the device: a plain copy
    FG_REQUIRE(rows >= 0 && cols >= 0 && cols % 256 == 0, FG_ERR_SHAPE,
               "k-quant matrix [%lld, %lld]: cols %% 256 != 0", (long long)rows, (long long)cols);
    const uint64_t need = (uint64_t)rows * (uint64_t)(cols / 256) * kquant_block_bytes(qtype);
    FG_REQUIRE(bytes == need, FG_ERR_SHAPE, "GGUF payload of %llu bytes, expected %llu", (unsigned long long)bytes,
               (unsigned long long)need);
    const int64_t shape[2] = {rows, cols};
    Tensor *t = nullptr;
    const fg_handle h = c.make(shape, 2, qtype, &t);
    if (need) c.h2d(t->ptr, gguf_blocks, need);
    *out = h;
    return FG_OK;
  }
  FG_REQUIRE(rows >= 0 && cols >= 0 && cols % 32 == 0, FG_ERR_SHAPE, "quantized matrix [%lld, %lld]: cols %% 32 != 0",
             (long long)rows, (long long)cols);
  const uint64_t need = (uint64_t)rows * (uint64_t)(cols / 32) * (uint64_t)gguf_block_bytes(qtype);
  FG_REQUIRE(bytes == need, FG_ERR_SHAPE, "GGUF payload of %llu bytes, expected %llu", (unsigned long long)bytes,
             (unsigned long long)need);
  const int64_t shape[2] = {rows, cols};
  Tensor *t = nullptr;
  const fg_handle h = c.make(shape, 2, qtype, &t);
  FG_CUDA(cudaMemsetAsync(t->ptr, 0, t->bytes, c.stream));  // defined scale padding
  if (need) {
    void *tmp = c.alloc(need);
    c.h2d(tmp, gguf_blocks, need);
    launch_gguf_to_device((const uint8_t *)tmp, qtype, rows, cols, t->qmat(), 1, 0, c.stream);
    c.free_async(tmp, need);
  }
  *out = h;
  FG_API_END
}

int fg_empty(fg_ctx *ctx, const int64_t *shape, int32_t ndim, int32_t dtype, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  *out = C(ctx).make(shape, ndim, dtype);
  FG_API_END
}

int fg_read(fg_ctx *ctx, fg_handle h, void *host, uint64_t bytes) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &t = c.get(h);
  FG_REQUIRE(bytes == t.bytes, FG_ERR_SHAPE, "read of %llu bytes from a %llu-byte tensor", (unsigned long long)bytes,
             (unsigned long long)t.bytes);
  c.d2h(host, t.ptr, bytes);
  FG_API_END
}

int fg_read_quant_gguf(fg_ctx *ctx, fg_handle h, void *host, uint64_t bytes) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &t = c.get(h);
  FG_REQUIRE(is_quant(t.dtype), FG_ERR_DTYPE, "fg_read_quant_gguf: tensor is not quantized");
  if (is_kquant(t.dtype)) {
    FG_REQUIRE(bytes == t.bytes, FG_ERR_SHAPE, "GGUF read of %llu bytes, expected %llu", (unsigned long long)bytes,
               (unsigned long long)t.bytes);
    if (bytes) c.d2h(host, t.ptr, bytes);
    return FG_OK;
  }
  const uint64_t need = (uint64_t)t.shape[0] * (uint64_t)(t.shape[1] / 32) * (uint64_t)gguf_block_bytes(t.dtype);
  FG_REQUIRE(bytes == need, FG_ERR_SHAPE, "GGUF read of %llu bytes, expected %llu", (unsigned long long)bytes,
             (unsigned long long)need);
  if (need) {
    void *tmp = c.alloc(need);
    launch_device_to_gguf(t.qmat(), (uint8_t *)tmp, c.stream);
    c.d2h(host, tmp, need);
    c.free_async(tmp, need);
  }
  FG_API_END
}

int fg_info(fg_ctx *ctx, fg_handle h, fg_tensor_info *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Tensor &t = C(ctx).get(h);
  out->dtype = t.dtype;
  out->ndim = t.ndim;
  for (int i = 0; i < FG_MAX_DIMS; ++i) out->shape[i] = i < t.ndim ? t.shape[i] : 0;
  out->bytes = t.bytes;
  out->device_ptr = (uint64_t)(uintptr_t)t.ptr;
  FG_API_END
}

int fg_dispose(fg_ctx *ctx, fg_handle h) {
  FG_API_BEGIN
  Guard g(ctx);
  C(ctx).dispose(h);
  FG_API_END
}

int fg_dispose_batch(fg_ctx *ctx, const fg_handle *hs, int32_t n) {
  FG_API_BEGIN
  Guard g(ctx);
  for (int32_t i = 0; i < n; ++i) C(ctx).dispose(hs[i]);
  FG_API_END
}

// ------------------------------------------------------------------ ops
int fg_unpack_quant(fg_ctx *ctx, fg_handle packed, fg_handle scales, fg_handle zeros, int32_t bits, int64_t group_size,
                    int64_t num_elements, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  FG_REQUIRE(bits == 4 || bits == 8, FG_ERR_VALIDATION, "unpack_quant: bits must be 4 or 8, got %d", bits);
  FG_REQUIRE(group_size > 0 && num_elements >= 0, FG_ERR_VALIDATION, "unpack_quant: bad group size / element count");
  Tensor &p = c.get(packed), &s = c.get(scales), &z = c.get(zeros);
  FG_REQUIRE(p.dtype == FG_U32 || p.dtype == FG_F32, FG_ERR_DTYPE, "unpack_quant: packed words must be U32 (or F32 bit patterns)");
  check_f32(s, "unpack_quant scales");
  check_f32(z, "unpack_quant zeros");
  const int64_t words = ceil_div(num_elements, bits == 4 ? 8 : 4);
  const int64_t groups = ceil_div(num_elements, group_size);
  FG_REQUIRE(p.numel() >= words && s.numel() >= groups && z.numel() >= groups, FG_ERR_SHAPE,
             "unpack_quant: %lld elements need %lld words and %lld groups", (long long)num_elements, (long long)words,
             (long long)groups);
  const int64_t shp[1] = {num_elements};
  Tensor *o = nullptr;
  const fg_handle h = c.make(shp, 1, FG_F32, &o);
  launch_unpack_quant((const uint32_t *)p.ptr, (const float *)s.ptr, (const float *)z.ptr, bits, group_size,
                      num_elements, (float *)o->ptr, c.stream);
  *out = h;
  FG_API_END
}

int fg_dequant(fg_ctx *ctx, fg_handle w, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &t = c.get(w);
  FG_REQUIRE(is_quant(t.dtype), FG_ERR_DTYPE, "dequant: tensor is not Q4_0/Q8_0/Q4_K/Q6_K");
  if (is_kquant(t.dtype)) {
    const int64_t shp[2] = {t.shape[0], t.shape[1]};
    const void *src = t.ptr;
    const int dt = t.dtype;  // `t` may move when the registry grows
    Tensor *o = nullptr;
    const fg_handle h = c.make(shp, 2, FG_F32, &o);
    if (dt == FG_Q4_K)
      launch_dequant_q4k(src, shp[0] * shp[1] / 256, (float *)o->ptr, c.stream);
    else
      launch_dequant_q6k(src, shp[0] * shp[1] / 256, (float *)o->ptr, c.stream);
    *out = h;
    return FG_OK;
  }
  const QMat q = t.qmat();
  const int64_t shp[2] = {q.N, q.K};
  Tensor *o = nullptr;
  const fg_handle h = c.make(shp, 2, FG_F32, &o);
  launch_dequant(q, (float *)o->ptr, c.stream);
  *out = h;
  FG_API_END
}

namespace {
// Validates x [..., K] against W [N, K]; returns M (rows of x).
int64_t qmatmul_rows(const Tensor &xt, const Tensor &wt) {
  check_f32(xt, "qmatmul activations");
  FG_REQUIRE(is_quant(wt.dtype), FG_ERR_DTYPE, "qmatmul: weight must be Q4_0/Q8_0/Q4_K/Q6_K");
  const int64_t K = wt.shape[1];
  FG_REQUIRE(xt.ndim >= 1 && xt.shape[xt.ndim - 1] == K, FG_ERR_SHAPE, "qmatmul: x[..., %lld] vs W[%lld, %lld]",
             (long long)(xt.ndim ? xt.shape[xt.ndim - 1] : 0), (long long)wt.shape[0], (long long)K);
  const int64_t M = K ? xt.numel() / K : 0;
  FG_REQUIRE(M <= INT32_MAX, FG_ERR_SHAPE, "qmatmul: too many rows");
  return M;
}

// Q4_K / Q6_K: GEMV for M <= 8, else the matrix dequantised (bit-exact) into a temporary and the fp32
// matmul (the tensor-core path for all but small products).
void qmatmul_kquant(Ctx &c, const Tensor &xt, const Tensor &wt, int64_t M, float *y) {
  const int64_t N = wt.shape[0], K = wt.shape[1];
  if (M <= 8) {
    if (wt.dtype == FG_Q4_K)
      launch_qmatmul_q4k(wt.ptr, N, K, (const float *)xt.ptr, M, y, nullptr, c.gemv.err, c.stream);
    else
      launch_qmatmul_q6k(wt.ptr, N, K, (const float *)xt.ptr, M, y, nullptr, c.stream);
    return;
  }
  if (N * K == 0) return;
  float *w32 = (float *)c.alloc(4ull * (uint64_t)(N * K));
  try {
    if (wt.dtype == FG_Q4_K)
      launch_dequant_q4k(wt.ptr, N * K / 256, w32, c.stream);
    else
      launch_dequant_q6k(wt.ptr, N * K / 256, w32, c.stream);
    launch_matmul(c, (const float *)xt.ptr, w32, y, M, K, N, /*b_trans=*/true);
  } catch (...) {
    c.free_async(w32, 4ull * (uint64_t)(N * K));
    throw;
  }
  c.free_async(w32, 4ull * (uint64_t)(N * K));
}

void qmatmul_launch(Ctx &c, const Tensor &xt, const QMat &q, int64_t M, float *y) {
  Epilogue ep;
  ep.mode = EPI_PLAIN;
  ep.y = y;
  ep.ldy = q.N;
  if (M == 0 || q.N == 0) return;
  if (gemv_supported(q, (int)M))
    launch_qgemv_ld(q, (const float *)xt.ptr, (int)M, q.K, nullptr, 0.0f, false, ep, c.gemv, c.num_sms, c.stream);
  else {
    if (qgemm_tc_supported(q, (int)M)) c.ensure_xh(tc_xh_elems(M, q.K));
    launch_qgemm(q, (const float *)xt.ptr, (int)M, q.K, ep, c.gemv, c.num_sms, c.stream);
  }
}
}  // namespace

int fg_qmatmul(fg_ctx *ctx, fg_handle x, fg_handle w, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &xt = c.get(x);
  Tensor &wt = c.get(w);
  const int64_t M = qmatmul_rows(xt, wt);
  int64_t shp[FG_MAX_DIMS];
  for (int i = 0; i < xt.ndim; ++i) shp[i] = xt.shape[i];
  shp[xt.ndim - 1] = wt.shape[0];
  Tensor *o = nullptr;
  const fg_handle h = c.make(shp, xt.ndim, FG_F32, &o);
  if (is_kquant(c.get(w).dtype))
    qmatmul_kquant(c, c.get(x), c.get(w), M, (float *)o->ptr);
  else
    qmatmul_launch(c, c.get(x), c.get(w).qmat(), M, (float *)o->ptr);
  *out = h;
  FG_API_END
}

int fg_qmatmul_into(fg_ctx *ctx, fg_handle x, fg_handle w, fg_handle out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &xt = c.get(x);
  Tensor &wt = c.get(w);
  Tensor &ot = c.get(out);
  const int64_t M = qmatmul_rows(xt, wt);
  FG_REQUIRE(ot.dtype == FG_F32 && ot.numel() == M * wt.shape[0], FG_ERR_SHAPE,
             "qmatmul_into: output must be F32 [.., %lld]", (long long)wt.shape[0]);
  if (is_kquant(wt.dtype))
    qmatmul_kquant(c, xt, wt, M, (float *)ot.ptr);
  else
    qmatmul_launch(c, xt, wt.qmat(), M, (float *)ot.ptr);
  FG_API_END
}

int fg_matmul(fg_ctx *ctx, fg_handle a, fg_handle b, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &at = c.get(a), &bt = c.get(b);
  check_f32(at, "matmul");
  check_f32(bt, "matmul");
  FG_REQUIRE(at.ndim == 2 && bt.ndim == 2 && at.shape[1] == bt.shape[0], FG_ERR_SHAPE,
             "matmul: [%lld, %lld] x [%lld, %lld]", (long long)at.shape[0], (long long)at.shape[1],
             (long long)bt.shape[0], (long long)bt.shape[1]);
  const int64_t shp[2] = {at.shape[0], bt.shape[1]};
  Tensor *o = nullptr;
  const fg_handle h = c.make(shp, 2, FG_F32, &o);
  launch_matmul(c, (const float *)at.ptr, (const float *)bt.ptr, (float *)o->ptr, at.shape[0], at.shape[1],
                bt.shape[1], false);
  *out = h;
  FG_API_END
}

int fg_flash_attention(fg_ctx *ctx, fg_handle q, fg_handle k, fg_handle v, float scale, int32_t has_scale,
                       int32_t causal, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &qt = c.get(q), &kt = c.get(k), &vt = c.get(v);
  // gpuCore.flashAttention validation order and messages (gpuCore.ts:960-980)
  FG_REQUIRE(qt.ndim == 4 && kt.ndim == 4 && vt.ndim == 4, FG_ERR_SHAPE,
             "FlashAttention requires 4D tensors [Batch, Heads, SeqLen, HeadDim]");
  FG_REQUIRE((qt.dtype == FG_F32 || qt.dtype == FG_F16) && kt.dtype == qt.dtype && vt.dtype == qt.dtype, FG_ERR_DTYPE,
             "FlashAttention requires float32 (or float16) tensors of one dtype");
  const int64_t B = qt.shape[0], H = qt.shape[1], Nq = qt.shape[2], d = qt.shape[3];
  const int64_t Hkv = kt.shape[1], Nk = kt.shape[2];
  FG_REQUIRE(B == kt.shape[0] && B == vt.shape[0], FG_ERR_SHAPE, "Batch mismatch: %lld vs %lld, %lld", (long long)B,
             (long long)kt.shape[0], (long long)vt.shape[0]);
  FG_REQUIRE(Hkv == vt.shape[1], FG_ERR_SHAPE, "KV heads mismatch: %lld vs %lld", (long long)Hkv, (long long)vt.shape[1]);
  FG_REQUIRE(Hkv > 0 && H % Hkv == 0, FG_ERR_SHAPE, "Query heads %lld must be divisible by KV heads %lld (GQA requirement)",
             (long long)H, (long long)Hkv);
  FG_REQUIRE(Nk == vt.shape[2], FG_ERR_SHAPE, "Key/Value SeqLen mismatch: %lld vs %lld", (long long)Nk,
             (long long)vt.shape[2]);
  FG_REQUIRE(d == kt.shape[3] && d == vt.shape[3], FG_ERR_SHAPE, "HeadDim mismatch: %lld vs %lld, %lld", (long long)d,
             (long long)kt.shape[3], (long long)vt.shape[3]);
  FG_REQUIRE(d <= 256, FG_ERR_SHAPE, "HeadDim %lld exceeds max supported dimension 256", (long long)d);
  const int64_t shp[4] = {B, H, Nq, d};
  Tensor *o = nullptr;
  const fg_handle h = c.make(shp, 4, FG_F32, &o);
  AttnArgs a;
  a.q = qt.ptr;
  a.k = kt.ptr;
  a.v = vt.ptr;
  a.o = (float *)o->ptr;
  a.q_f16 = a.kv_f16 = qt.dtype == FG_F16;
  a.B = (int)B;
  a.H = (int)H;
  a.Hkv = (int)Hkv;
  a.Nq = (int)Nq;
  a.d = (int)d;
  a.q_sb = H * Nq * d;
  a.q_sh = Nq * d;
  a.q_si = d;
  a.o_sb = a.q_sb;
  a.o_sh = a.q_sh;
  a.o_si = a.q_si;
  a.kv_sb = Hkv * Nk * d;
  a.kv_sh = Nk * d;
  a.n_kv = (int)Nk;
  a.scale = has_scale ? scale : (float)(1.0 / std::sqrt((double)d));
  a.causal = causal ? 1 : 0;
  a.err = c.gemv.err;
  launch_attention(c, a, c.stream);
  *out = h;
  FG_API_END
}

int fg_rmsnorm(fg_ctx *ctx, fg_handle x, fg_handle gamma, float eps, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &xt = c.get(x);
  check_f32(xt, "rmsNorm");
  FG_REQUIRE(xt.ndim >= 1, FG_ERR_SHAPE, "rmsNorm needs at least one dimension");
  const int64_t dim = xt.shape[xt.ndim - 1];
  const float *gp = nullptr;
  if (gamma) {
    Tensor &gt = c.get(gamma);
    check_f32(gt, "rmsNorm gamma");
    FG_REQUIRE(gt.numel() == dim, FG_ERR_SHAPE, "rmsNorm gamma has %lld elements, dim is %lld", (long long)gt.numel(),
               (long long)dim);
    gp = (const float *)gt.ptr;
  }
  Tensor *o = nullptr;
  const fg_handle h = c.make(xt.shape, xt.ndim, FG_F32, &o);
  if (dim > 0) launch_rmsnorm((const float *)xt.ptr, dim, gp, eps, xt.numel() / dim, dim, (float *)o->ptr, c.stream);
  *out = h;
  FG_API_END
}

int fg_rope(fg_ctx *ctx, fg_handle x, float base, int64_t offset, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &xt = c.get(x);
  check_f32(xt, "rope");
  FG_REQUIRE(xt.ndim == 4, FG_ERR_SHAPE, "rope requires a 4D tensor [B, H, N, d]");
  const int64_t d = xt.shape[3];
  FG_REQUIRE(d % 2 == 0, FG_ERR_SHAPE, "rope head dim %lld must be even", (long long)d);
  Tensor *o = nullptr;
  const fg_handle h = c.make(xt.shape, 4, FG_F32, &o);
  if (xt.numel()) {
    const float *tab = rope_table(&c, base, d);
    launch_rope((const float *)xt.ptr, xt.shape[0] * xt.shape[1], xt.shape[2], d, tab, offset, (float *)o->ptr,
                c.stream);
  }
  *out = h;
  FG_API_END
}

int fg_swiglu(fg_ctx *ctx, fg_handle gate, fg_handle up, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &gt = c.get(gate), &ut = c.get(up);
  check_f32(gt, "swiglu");
  check_f32(ut, "swiglu");
  FG_REQUIRE(gt.numel() == ut.numel(), FG_ERR_SHAPE, "swiglu: gate and up sizes differ");
  Tensor *o = nullptr;
  const fg_handle h = c.make(gt.shape, gt.ndim, FG_F32, &o);
  launch_swiglu((const float *)gt.ptr, (const float *)ut.ptr, gt.numel(), (float *)o->ptr, c.stream);
  *out = h;
  FG_API_END
}

int fg_embedding(fg_ctx *ctx, fg_handle table, fg_handle ids, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &tt = c.get(table), &it = c.get(ids);
  FG_REQUIRE(tt.ndim == 2 && (tt.dtype == FG_F32 || tt.dtype == FG_F16), FG_ERR_SHAPE,
             "embedding table must be a 2D float32/float16 tensor");
  FG_REQUIRE(it.dtype == FG_I32 || it.dtype == FG_F32, FG_ERR_DTYPE, "embedding ids must be int32 or float32");
  FG_REQUIRE(it.ndim < FG_MAX_DIMS, FG_ERR_SHAPE, "embedding ids rank too large");
  int64_t shp[FG_MAX_DIMS];
  for (int i = 0; i < it.ndim; ++i) shp[i] = it.shape[i];
  shp[it.ndim] = tt.shape[1];
  Tensor *o = nullptr;
  const fg_handle h = c.make(shp, it.ndim + 1, FG_F32, &o);
  launch_embedding(tt.ptr, tt.dtype == FG_F16, tt.shape[0], tt.shape[1], it.ptr, it.dtype == FG_F32, it.numel(),
                   (float *)o->ptr, c.stream);
  *out = h;
  FG_API_END
}

int fg_add(fg_ctx *ctx, fg_handle a, fg_handle b, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &at = c.get(a), &bt = c.get(b);
  check_f32(at, "add");
  check_f32(bt, "add");
  FG_REQUIRE(at.numel() == bt.numel(), FG_ERR_SHAPE, "add: sizes differ (%lld vs %lld)", (long long)at.numel(),
             (long long)bt.numel());
  Tensor *o = nullptr;
  const fg_handle h = c.make(at.shape, at.ndim, FG_F32, &o);
  launch_add((const float *)at.ptr, (const float *)bt.ptr, at.numel(), (float *)o->ptr, c.stream);
  *out = h;
  FG_API_END
}

int fg_argmax(fg_ctx *ctx, fg_handle logits, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &lt = c.get(logits);
  check_f32(lt, "argmax");
  FG_REQUIRE(lt.ndim >= 1 && lt.shape[lt.ndim - 1] > 0, FG_ERR_VALIDATION, "Logits array cannot be empty");
  const int64_t n = lt.shape[lt.ndim - 1];
  const int64_t rows = lt.numel() / n;
  const int64_t shp[1] = {rows};
  Tensor *o = nullptr;
  const fg_handle h = c.make(shp, 1, FG_I32, &o);
  launch_argmax((const float *)lt.ptr, rows, n, n, (int32_t *)o->ptr, c.stream);
  *out = h;
  FG_API_END
}

int fg_sample(fg_ctx *ctx, fg_handle logits, double temperature, int32_t top_k, double top_p, int32_t has_seed,
              uint32_t seed, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &lt = c.get(logits);
  check_f32(lt, "sample");
  FG_REQUIRE(lt.ndim >= 1 && lt.shape[lt.ndim - 1] > 0, FG_ERR_VALIDATION, "Logits array cannot be empty");
  const int64_t n = lt.shape[lt.ndim - 1];
  const int64_t rows = lt.numel() / n;
  const int64_t shp[1] = {rows};
  Tensor *o = nullptr;
  const fg_handle h = c.make(shp, 1, FG_I32, &o);
  const uint64_t sb = sample_scratch_bytes(rows, n);
  void *scratch = sb ? c.alloc(sb) : nullptr;
  launch_sample((const float *)lt.ptr, rows, n, n, temperature, top_k, top_p, has_seed != 0, seed, scratch,
                (int32_t *)o->ptr, c.stream);
  if (scratch) c.free_async(scratch, sb);
  *out = h;
  FG_API_END
}

int fg_cast(fg_ctx *ctx, fg_handle x, int32_t dtype, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  Tensor &xt = c.get(x);
  FG_REQUIRE((xt.dtype == FG_F32 || xt.dtype == FG_F16) && (dtype == FG_F32 || dtype == FG_F16), FG_ERR_DTYPE,
             "cast: only float32 <-> float16");
  Tensor *o = nullptr;
  const fg_handle h = c.make(xt.shape, xt.ndim, dtype, &o);
  launch_cast(xt.ptr, xt.dtype, o->ptr, dtype, xt.numel(), c.stream);
  *out = h;
  FG_API_END
}

int fg_synth_normal(fg_ctx *ctx, const int64_t *shape, int32_t ndim, int32_t dtype, uint64_t seed, uint64_t offset,
                    float mean, float stdv, fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  FG_REQUIRE(dtype == FG_F32 || dtype == FG_F16, FG_ERR_DTYPE, "synth_normal: dtype must be float32 or float16");
  Tensor *o = nullptr;
  const fg_handle h = c.make(shape, ndim, dtype, &o);
  launch_synth_normal(seed, offset, o->numel(), mean, stdv, dtype, o->ptr, c.stream);
  *out = h;
  FG_API_END
}

int fg_synth_quant(fg_ctx *ctx, int32_t qtype, int64_t rows, int64_t cols, uint64_t seed, int64_t row0, float stdv,
                   fg_handle *out) {
  FG_API_BEGIN
  Guard g(ctx);
  Ctx &c = C(ctx);
  FG_REQUIRE(qtype == FG_Q4_0 || qtype == FG_Q8_0, FG_ERR_DTYPE, "synth_quant: qtype must be Q4_0 or Q8_0");
  const int64_t shp[2] = {rows, cols};
  Tensor *o = nullptr;
  const fg_handle h = c.make(shp, 2, qtype, &o);
  FG_CUDA(cudaMemsetAsync(o->ptr, 0, o->bytes, c.stream));
  launch_synth_quant(qtype, rows, cols, seed, row0, 0, cols, stdv, o->qmat(), 1, 0, c.stream);
  *out = h;
  FG_API_END
}

}  // extern "C"
