// Node-API binding of libforge_b200 for the reference's TypeScript host.
//
// It exposes the surface that packages/forge/src/bridge/pyodideBridge.ts:31-58
// publishes as globalThis.amevaForge (init, read, dispose, getTensorInfo,
// mapBufferAsync, readMappedInto, executeGraph, warmupKernels, disposeBatch,
// getQuotaSnapshot, snapshotHandles, flushGC) and the gpuCore op object
// (packages/forge/src/tensor/gpuCore.ts:1448-1467) over the C ABI of
// include/forge_b200.h.  gpuCore.ts in this directory wraps it so the host
// keeps the reference's names, argument order and Promise-returning calls.
//
// Conventions (include/forge_b200.h):
//  * handles are rendered as "tensor_<16 hex digits>" strings (types.ts:19);
//  * a failing call throws a JS Error whose `name` is the reference's error
//    class (fg_status_name), because forge-py maps errors by class name
//    (forge-py bridge.py:206-226);
//  * calls that wait for the device (read, mapBufferAsync, executeGraph,
//    flushGC) run on the libuv pool through napi_create_async_work and settle
//    a Promise, so the event loop never blocks on the GPU;
//  * host buffers are borrowed for the duration of a call: the async calls
//    copy their inputs before they leave the JS thread.
#include <node_api.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "forge_b200.h"

namespace {

fg_ctx *g_ctx = nullptr;
std::mutex g_mu;                                        // live handles and staged reads
std::set<fg_handle> g_live;                             // snapshotHandles()
std::map<fg_handle, std::vector<unsigned char>> g_staged;  // mapBufferAsync -> readMappedInto

#define NAPI_OK(call)                                         \
  do {                                                        \
    if ((call) != napi_ok) return throw_msg(env, "AMEVAForgeInternalGPUError", "Node-API call failed: " #call); \
  } while (0)

napi_value throw_msg(napi_env env, const char *name, const char *message) {
  napi_value msg, nm, err;
  napi_create_string_utf8(env, message, NAPI_AUTO_LENGTH, &msg);
  napi_create_error(env, nullptr, msg, &err);
  napi_create_string_utf8(env, name, NAPI_AUTO_LENGTH, &nm);
  napi_set_named_property(env, err, "name", nm);
  napi_throw(env, err);
  return nullptr;
}

napi_value make_error(napi_env env, int st, const std::string &message) {
  napi_value msg, nm, err;
  napi_create_string_utf8(env, message.c_str(), NAPI_AUTO_LENGTH, &msg);
  napi_create_error(env, nullptr, msg, &err);
  napi_create_string_utf8(env, fg_status_name(st), NAPI_AUTO_LENGTH, &nm);
  napi_set_named_property(env, err, "name", nm);
  return err;
}

napi_value throw_status(napi_env env, int st) {
  napi_throw(env, make_error(env, st, fg_last_error()));
  return nullptr;
}

napi_value handle_str(napi_env env, fg_handle h) {
  char buf[32];
  snprintf(buf, sizeof buf, "tensor_%016llx", (unsigned long long)h);
  napi_value v;
  napi_create_string_utf8(env, buf, NAPI_AUTO_LENGTH, &v);
  return v;
}

// "tensor_<hex>" -> handle; false for anything else (a non-string, another prefix, no digits).
bool parse_handle(napi_env env, napi_value v, fg_handle *h) {
  char buf[40];
  size_t n = 0;
  if (napi_get_value_string_utf8(env, v, buf, sizeof buf, &n) != napi_ok || n < 8 || n > 23) return false;
  if (std::strncmp(buf, "tensor_", 7) != 0) return false;
  char *end = nullptr;
  const unsigned long long x = std::strtoull(buf + 7, &end, 16);
  if (!end || *end != '\0' || x == 0) return false;
  *h = (fg_handle)x;
  return true;
}

napi_value undefined(napi_env env) {
  napi_value u;
  napi_get_undefined(env, &u);
  return u;
}

bool get_args(napi_env env, napi_callback_info info, size_t want, napi_value *a, size_t *argc) {
  *argc = want;
  if (napi_get_cb_info(env, info, argc, a, nullptr, nullptr) != napi_ok) return false;
  for (size_t i = *argc; i < want; ++i) a[i] = undefined(env);
  return true;
}

bool is_type(napi_env env, napi_value v, napi_valuetype t) {
  napi_valuetype got;
  return napi_typeof(env, v, &got) == napi_ok && got == t;
}

double num_or(napi_env env, napi_value v, double dflt) {
  double d = dflt;
  if (is_type(env, v, napi_number)) napi_get_value_double(env, v, &d);
  return d;
}

bool bool_or(napi_env env, napi_value v, bool dflt) {
  bool b = dflt;
  if (is_type(env, v, napi_boolean)) napi_get_value_bool(env, v, &b);
  return b;
}

napi_value ret_handle(napi_env env, int st, fg_handle h) {
  if (st) return throw_status(env, st);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    g_live.insert(h);
  }
  return handle_str(env, h);
}

bool need_ctx(napi_env env) {
  if (g_ctx) return true;
  throw_msg(env, "AMEVAForgeWebGPUUnavailableError", "forge_b200: init() has not been called");
  return false;
}

// Reads a handle argument or throws AMEVAForgeStaleHandleError.
bool arg_handle(napi_env env, napi_value v, fg_handle *h) {
  if (parse_handle(env, v, h)) return true;
  throw_msg(env, "AMEVAForgeStaleHandleError", "expected a tensor handle string \"tensor_<hex>\"");
  return false;
}

const char *dtype_name(int32_t dt) {
  switch (dt) {
    case FG_F32: return "float32";
    case FG_F16: return "float16";
    case FG_I32: return "int32";
    case FG_U8: return "uint8";
    case FG_U32: return "uint32";
    case FG_Q4_0: return "q4_0";
    case FG_Q8_0: return "q8_0";
    case FG_Q4_K: return "q4_k";
    case FG_Q6_K: return "q6_k";
  }
  return "unknown";
}

// ---------------------------------------------------------------------------
// Async work: the device-waiting calls
// ---------------------------------------------------------------------------
struct Job {
  napi_async_work work = nullptr;
  napi_deferred deferred = nullptr;
  int status = 0;
  std::string error;
  virtual ~Job() = default;
  virtual void run() = 0;                           // libuv worker thread: C ABI only
  virtual napi_value result(napi_env env) = 0;      // JS thread
};

void job_execute(napi_env, void *data) {
  Job *j = static_cast<Job *>(data);
  j->run();
  if (j->status) j->error = fg_last_error();  // thread-local: read on the thread that failed
}

void job_complete(napi_env env, napi_status, void *data) {
  Job *j = static_cast<Job *>(data);
  if (j->status)
    napi_reject_deferred(env, j->deferred, make_error(env, j->status, j->error));
  else
    napi_resolve_deferred(env, j->deferred, j->result(env));
  napi_delete_async_work(env, j->work);
  delete j;
}

napi_value queue(napi_env env, Job *j, const char *name) {
  napi_value promise, res;
  napi_create_promise(env, &j->deferred, &promise);
  napi_create_string_utf8(env, name, NAPI_AUTO_LENGTH, &res);
  napi_create_async_work(env, nullptr, res, job_execute, job_complete, j, &j->work);
  napi_queue_async_work(env, j->work);
  return promise;
}

struct ReadJob : Job {
  fg_handle h = 0;
  fg_tensor_info info{};
  std::vector<unsigned char> bytes;
  bool stage = false;  // mapBufferAsync: keep the bytes for readMappedInto
  void run() override {
    if ((status = fg_info(g_ctx, h, &info))) return;
    bytes.resize(info.bytes);
    status = fg_read(g_ctx, h, bytes.data(), info.bytes);
  }
  napi_value result(napi_env env) override {
    if (stage) {
      std::lock_guard<std::mutex> lk(g_mu);
      g_staged[h] = std::move(bytes);
      return undefined(env);
    }
    // read() resolves to a Float32Array (gpuCore.ts:357); other dtypes come back in their own typed array
    void *data = nullptr;
    napi_value ab, arr;
    napi_create_arraybuffer(env, bytes.size(), &data, &ab);
    if (!bytes.empty()) std::memcpy(data, bytes.data(), bytes.size());
    napi_typedarray_type t = napi_uint8_array;
    size_t es = 1;
    switch (info.dtype) {
      case FG_F32: t = napi_float32_array; es = 4; break;
      case FG_F16: t = napi_uint16_array; es = 2; break;
      case FG_I32: t = napi_int32_array; es = 4; break;
      case FG_U32: t = napi_uint32_array; es = 4; break;
      default: break;
    }
    napi_create_typedarray(env, t, bytes.size() / es, ab, 0, &arr);
    return arr;
  }
};

struct GraphJob : Job {
  std::string json;
  std::vector<std::vector<unsigned char>> inputs;  // copied: the JS arrays may change after the call returns
  std::vector<int64_t> ids;
  std::vector<fg_handle> hs;
  int32_t n = 0;
  void run() override {
    std::vector<const void *> ptrs(inputs.size());
    std::vector<uint64_t> sizes(inputs.size());
    for (size_t i = 0; i < inputs.size(); ++i) {
      ptrs[i] = inputs[i].data();
      sizes[i] = inputs[i].size();
    }
    // one output slot per node: every node carries an "op" key, so their count bounds the node count
    size_t cap = 1;
    for (size_t at = json.find("\"op\""); at != std::string::npos; at = json.find("\"op\"", at + 4)) ++cap;
    ids.resize(cap);
    hs.resize(cap);
    status = fg_execute_graph(g_ctx, json.c_str(), ptrs.data(), sizes.data(), (int32_t)inputs.size(), ids.data(),
                              hs.data(), (int32_t)cap, &n);
    if (!status) status = fg_synchronize(g_ctx);
  }
  napi_value result(napi_env env) override {
    // {[id: string]: handle} keyed by the decimal node id, as graphExecutor.ts returns it
    napi_value out;
    napi_create_object(env, &out);
    std::lock_guard<std::mutex> lk(g_mu);
    for (int32_t i = 0; i < n; ++i) {
      g_live.insert(hs[i]);
      napi_set_named_property(env, out, std::to_string(ids[i]).c_str(), handle_str(env, hs[i]));
    }
    return out;
  }
};

struct SyncJob : Job {
  void run() override { status = fg_synchronize(g_ctx); }
  napi_value result(napi_env env) override {
    napi_value o, t;
    napi_create_object(env, &o);
    napi_get_boolean(env, true, &t);
    napi_set_named_property(env, o, "ok", t);
    return o;
  }
};

// ---------------------------------------------------------------------------
// Bridge surface (pyodideBridge.ts:31-58)
// ---------------------------------------------------------------------------

// init({device?, vramLimitBytes?, tpRank?, tpSize?, ncclId?: Uint8Array}) -> Promise<void>
napi_value Init(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[1];
  if (!get_args(env, info, 1, a, &argc)) return nullptr;
  fg_init_opts o{};
  o.tp_size = 1;
  if (is_type(env, a[0], napi_object)) {
    napi_value v;
    if (napi_get_named_property(env, a[0], "device", &v) == napi_ok) o.device = (int32_t)num_or(env, v, 0);
    if (napi_get_named_property(env, a[0], "vramLimitBytes", &v) == napi_ok)
      o.vram_limit_bytes = (uint64_t)num_or(env, v, 0);
    if (napi_get_named_property(env, a[0], "tpRank", &v) == napi_ok) o.tp_rank = (int32_t)num_or(env, v, 0);
    if (napi_get_named_property(env, a[0], "tpSize", &v) == napi_ok) o.tp_size = (int32_t)num_or(env, v, 1);
    bool has = false;
    if (napi_has_named_property(env, a[0], "ncclId", &has) == napi_ok && has &&
        napi_get_named_property(env, a[0], "ncclId", &v) == napi_ok) {
      napi_typedarray_type t;
      size_t len = 0;
      void *data = nullptr;
      napi_value ab;
      size_t off;
      if (napi_get_typedarray_info(env, v, &t, &len, &data, &ab, &off) == napi_ok && t == napi_uint8_array &&
          len == sizeof o.nccl_id)
        std::memcpy(o.nccl_id, data, sizeof o.nccl_id);
    }
  }
  napi_deferred d;
  napi_value promise;
  NAPI_OK(napi_create_promise(env, &d, &promise));
  if (g_ctx) {  // init is idempotent, as initWebGPU is once a device exists
    napi_resolve_deferred(env, d, undefined(env));
    return promise;
  }
  const int st = fg_init(&o, &g_ctx);
  if (st)
    napi_reject_deferred(env, d, make_error(env, st, fg_last_error()));
  else
    napi_resolve_deferred(env, d, undefined(env));
  return promise;
}

// read(handle) -> Promise<Float32Array>
napi_value Read(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[1];
  if (!get_args(env, info, 1, a, &argc) || !need_ctx(env)) return nullptr;
  auto *j = new ReadJob;
  if (!arg_handle(env, a[0], &j->h)) {
    delete j;
    return nullptr;
  }
  return queue(env, j, "forge_b200.read");
}

// mapBufferAsync(handle) -> Promise<void>: the bytes are staged on the host for readMappedInto
napi_value MapBufferAsync(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[1];
  if (!get_args(env, info, 1, a, &argc) || !need_ctx(env)) return nullptr;
  auto *j = new ReadJob;
  j->stage = true;
  if (!arg_handle(env, a[0], &j->h)) {
    delete j;
    return nullptr;
  }
  return queue(env, j, "forge_b200.mapBufferAsync");
}

// readMappedInto(handle, outArray): copies the staged bytes into a typed array (no device wait)
napi_value ReadMappedInto(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[2];
  if (!get_args(env, info, 2, a, &argc)) return nullptr;
  fg_handle h;
  if (!arg_handle(env, a[0], &h)) return nullptr;
  std::vector<unsigned char> bytes;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_staged.find(h);
    if (it == g_staged.end())
      return throw_msg(env, "AMEVAForgeValidationError", "No staged buffer for this handle. Call mapBufferAsync first.");
    bytes = std::move(it->second);
    g_staged.erase(it);
  }
  napi_typedarray_type t;
  size_t len = 0;
  void *data = nullptr;
  napi_value ab;
  size_t off;
  NAPI_OK(napi_get_typedarray_info(env, a[1], &t, &len, &data, &ab, &off));
  size_t es = 1;
  switch (t) {
    case napi_int16_array: case napi_uint16_array: es = 2; break;
    case napi_int32_array: case napi_uint32_array: case napi_float32_array: es = 4; break;
    case napi_float64_array: case napi_bigint64_array: case napi_biguint64_array: es = 8; break;
    default: break;
  }
  std::memcpy(data, bytes.data(), std::min(bytes.size(), len * es));
  return undefined(env);
}

// dispose(handle): deferred until the stream has passed every use; a second dispose is a no-op
napi_value Dispose(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[1];
  if (!get_args(env, info, 1, a, &argc) || !need_ctx(env)) return nullptr;
  fg_handle h;
  if (!arg_handle(env, a[0], &h)) return nullptr;
  if (int st = fg_dispose(g_ctx, h)) return throw_status(env, st);
  std::lock_guard<std::mutex> lk(g_mu);
  g_live.erase(h);
  g_staged.erase(h);
  return undefined(env);
}

// disposeBatch(handles[])
napi_value DisposeBatch(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[1];
  if (!get_args(env, info, 1, a, &argc) || !need_ctx(env)) return nullptr;
  uint32_t n = 0;
  NAPI_OK(napi_get_array_length(env, a[0], &n));
  std::vector<fg_handle> hs;
  for (uint32_t i = 0; i < n; ++i) {
    napi_value e;
    fg_handle h;
    NAPI_OK(napi_get_element(env, a[0], i, &e));
    if (parse_handle(env, e, &h)) hs.push_back(h);
  }
  if (int st = fg_dispose_batch(g_ctx, hs.data(), (int32_t)hs.size())) return throw_status(env, st);
  std::lock_guard<std::mutex> lk(g_mu);
  for (fg_handle h : hs) {
    g_live.erase(h);
    g_staged.erase(h);
  }
  return undefined(env);
}

// getTensorInfo(handle) -> {handle, shape, dtype, byteLength, disposed}
napi_value GetTensorInfo(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[1];
  if (!get_args(env, info, 1, a, &argc) || !need_ctx(env)) return nullptr;
  fg_handle h;
  if (!arg_handle(env, a[0], &h)) return nullptr;
  fg_tensor_info ti;
  if (int st = fg_info(g_ctx, h, &ti)) return throw_status(env, st);
  napi_value o, shape, v;
  napi_create_object(env, &o);
  napi_set_named_property(env, o, "handle", handle_str(env, h));
  napi_create_array_with_length(env, (size_t)ti.ndim, &shape);
  for (int i = 0; i < ti.ndim; ++i) {
    napi_create_double(env, (double)ti.shape[i], &v);
    napi_set_element(env, shape, (uint32_t)i, v);
  }
  napi_set_named_property(env, o, "shape", shape);
  napi_create_string_utf8(env, dtype_name(ti.dtype), NAPI_AUTO_LENGTH, &v);
  napi_set_named_property(env, o, "dtype", v);
  napi_create_double(env, (double)ti.bytes, &v);
  napi_set_named_property(env, o, "byteLength", v);
  napi_get_boolean(env, false, &v);
  napi_set_named_property(env, o, "disposed", v);
  return o;
}

// getQuotaSnapshot() (quota.ts:315-336)
napi_value GetQuotaSnapshot(napi_env env, napi_callback_info) {
  if (!need_ctx(env)) return nullptr;
  fg_quota q;
  if (int st = fg_quota_snapshot(g_ctx, &q)) return throw_status(env, st);
  napi_value o, v;
  napi_create_object(env, &o);
  const std::pair<const char *, uint64_t> f[] = {{"limitBytes", q.limit_bytes}, {"activeBytes", q.active_bytes},
                                                 {"pendingBytes", q.pending_bytes}, {"peakBytes", q.peak_bytes},
                                                 {"liveTensors", q.live_tensors}};
  for (const auto &kv : f) {
    napi_create_double(env, (double)kv.second, &v);
    napi_set_named_property(env, o, kv.first, v);
  }
  return o;
}

napi_value SnapshotHandles(napi_env env, napi_callback_info) {
  napi_value arr;
  std::lock_guard<std::mutex> lk(g_mu);
  napi_create_array_with_length(env, g_live.size(), &arr);
  uint32_t i = 0;
  for (fg_handle h : g_live) napi_set_element(env, arr, i++, handle_str(env, h));
  return arr;
}

// flushGC(options?) -> Promise<{ok}>: waits for the stream (deferred disposals complete with it)
napi_value FlushGC(napi_env env, napi_callback_info) {
  if (!need_ctx(env)) return nullptr;
  return queue(env, new SyncJob, "forge_b200.flushGC");
}

// warmupKernels() -> Promise<void>: every kernel is compiled ahead of time for sm_100a
napi_value WarmupKernels(napi_env env, napi_callback_info) {
  napi_deferred d;
  napi_value promise;
  NAPI_OK(napi_create_promise(env, &d, &promise));
  napi_resolve_deferred(env, d, undefined(env));
  return promise;
}

// executeGraph(instructionsJson, inputs: Float32Array[]) -> Promise<{[id]: handle}> (graphExecutor.ts:489)
napi_value ExecuteGraph(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[2];
  if (!get_args(env, info, 2, a, &argc) || !need_ctx(env)) return nullptr;
  auto *j = new GraphJob;
  size_t jn = 0;
  if (napi_get_value_string_utf8(env, a[0], nullptr, 0, &jn) != napi_ok) {
    delete j;
    return throw_msg(env, "AMEVAForgeValidationError", "executeGraph: instructions must be a JSON string");
  }
  j->json.assign(jn + 1, '\0');
  napi_get_value_string_utf8(env, a[0], &j->json[0], jn + 1, &jn);
  j->json.resize(jn);
  bool is_arr = false;
  if (napi_is_array(env, a[1], &is_arr) == napi_ok && is_arr) {
    uint32_t n = 0;
    napi_get_array_length(env, a[1], &n);
    j->inputs.resize(n);
    for (uint32_t i = 0; i < n; ++i) {
      napi_value e, ab;
      napi_typedarray_type t;
      size_t len = 0, off = 0;
      void *data = nullptr;
      napi_get_element(env, a[1], i, &e);
      if (napi_get_typedarray_info(env, e, &t, &len, &data, &ab, &off) != napi_ok || t != napi_float32_array) {
        delete j;
        return throw_msg(env, "AMEVAForgeDTypeError", "executeGraph: every input must be a Float32Array");
      }
      const unsigned char *p = static_cast<const unsigned char *>(data);
      j->inputs[i].assign(p, p + len * 4);
    }
  }
  return queue(env, j, "forge_b200.executeGraph");
}

// uploadFloat32Array(data, shape) -> handle (gpuCore.ts:660)
napi_value UploadFloat32Array(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[2];
  if (!get_args(env, info, 2, a, &argc) || !need_ctx(env)) return nullptr;
  napi_typedarray_type t;
  size_t len = 0, off = 0;
  void *data = nullptr;
  napi_value ab;
  if (napi_get_typedarray_info(env, a[0], &t, &len, &data, &ab, &off) != napi_ok || t != napi_float32_array)
    return throw_msg(env, "AMEVAForgeDTypeError", "uploadFloat32Array: data must be a Float32Array");
  uint32_t nd = 0;
  NAPI_OK(napi_get_array_length(env, a[1], &nd));
  if (nd > FG_MAX_DIMS) return throw_msg(env, "AMEVAForgeShapeError", "uploadFloat32Array: rank above 8");
  int64_t shape[FG_MAX_DIMS];
  for (uint32_t i = 0; i < nd; ++i) {
    napi_value e;
    napi_get_element(env, a[1], i, &e);
    shape[i] = (int64_t)num_or(env, e, -1);
  }
  fg_handle h = 0;
  return ret_handle(env, fg_upload(g_ctx, data, len * 4, shape, (int32_t)nd, FG_F32, &h), h);
}

// uploadQuant(type, blocks: Uint8Array, rows, cols) -> handle (GGUF blocks; repacked on the device)
napi_value UploadQuant(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[4];
  if (!get_args(env, info, 4, a, &argc) || !need_ctx(env)) return nullptr;
  char ty[8] = {0};
  size_t n = 0;
  napi_get_value_string_utf8(env, a[0], ty, sizeof ty, &n);
  const int32_t qt = !std::strcmp(ty, "Q4_0") ? FG_Q4_0 : !std::strcmp(ty, "Q8_0") ? FG_Q8_0
                     : !std::strcmp(ty, "Q4_K") ? FG_Q4_K : !std::strcmp(ty, "Q6_K") ? FG_Q6_K : -1;
  if (qt < 0) return throw_msg(env, "AMEVAForgeDTypeError", "uploadQuant: type must be Q4_0, Q8_0, Q4_K or Q6_K");
  napi_typedarray_type t;
  size_t len = 0, off = 0;
  void *data = nullptr;
  napi_value ab;
  if (napi_get_typedarray_info(env, a[1], &t, &len, &data, &ab, &off) != napi_ok || t != napi_uint8_array)
    return throw_msg(env, "AMEVAForgeDTypeError", "uploadQuant: blocks must be a Uint8Array");
  fg_handle h = 0;
  return ret_handle(env,
                    fg_upload_quant(g_ctx, qt, data, len, (int64_t)num_or(env, a[2], 0), (int64_t)num_or(env, a[3], 0),
                                    &h),
                    h);
}

// ---------------------------------------------------------------------------
// gpuCore ops (gpuCore.ts:1448-1467); each enqueues and returns the output handle
// ---------------------------------------------------------------------------
napi_value Matmul(napi_env env, napi_callback_info info) {  // matmul(a, b) and matmulTiled(a, b)
  size_t argc;
  napi_value a[2];
  fg_handle x, y, out = 0;
  if (!get_args(env, info, 2, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &x) || !arg_handle(env, a[1], &y))
    return nullptr;
  return ret_handle(env, fg_matmul(g_ctx, x, y, &out), out);
}

napi_value QMatmul(napi_env env, napi_callback_info info) {  // x @ W^T with W quantized (nn.Linear over GGUF)
  size_t argc;
  napi_value a[2];
  fg_handle x, w, out = 0;
  if (!get_args(env, info, 2, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &x) || !arg_handle(env, a[1], &w))
    return nullptr;
  return ret_handle(env, fg_qmatmul(g_ctx, x, w, &out), out);
}

// flashAttention(q, k, v, scale?, isCausal = false)
napi_value FlashAttention(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[5];
  fg_handle q, k, v, out = 0;
  if (!get_args(env, info, 5, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &q) ||
      !arg_handle(env, a[1], &k) || !arg_handle(env, a[2], &v))
    return nullptr;
  const bool has_scale = is_type(env, a[3], napi_number);
  const double scale = num_or(env, a[3], 0.0);
  return ret_handle(env, fg_flash_attention(g_ctx, q, k, v, (float)scale, has_scale, bool_or(env, a[4], false), &out),
                    out);
}

// rmsNorm(x, gamma?, eps = 1e-5)
napi_value RmsNorm(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[3];
  fg_handle x, g = 0, out = 0;
  if (!get_args(env, info, 3, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &x)) return nullptr;
  if (is_type(env, a[1], napi_string) && !arg_handle(env, a[1], &g)) return nullptr;
  return ret_handle(env, fg_rmsnorm(g_ctx, x, g, (float)num_or(env, a[2], 1e-5), &out), out);
}

// rope(x, base = 1e4, offset = 0)
napi_value Rope(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[3];
  fg_handle x, out = 0;
  if (!get_args(env, info, 3, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &x)) return nullptr;
  return ret_handle(env, fg_rope(g_ctx, x, (float)num_or(env, a[1], 1e4), (int64_t)num_or(env, a[2], 0), &out), out);
}

napi_value Swiglu(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[2];
  fg_handle g, u, out = 0;
  if (!get_args(env, info, 2, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &g) || !arg_handle(env, a[1], &u))
    return nullptr;
  return ret_handle(env, fg_swiglu(g_ctx, g, u, &out), out);
}

napi_value Add(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[2];
  fg_handle x, y, out = 0;
  if (!get_args(env, info, 2, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &x) || !arg_handle(env, a[1], &y))
    return nullptr;
  return ret_handle(env, fg_add(g_ctx, x, y, &out), out);
}

// embedding(w, idx)
napi_value Embedding(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[2];
  fg_handle w, idx, out = 0;
  if (!get_args(env, info, 2, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &w) ||
      !arg_handle(env, a[1], &idx))
    return nullptr;
  return ret_handle(env, fg_embedding(g_ctx, w, idx, &out), out);
}

// unpackQuant(packed, scales, zeros, bits = 4, groupSize = 128, numElements) (gpuCore.ts:1123-1130)
napi_value UnpackQuant(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[6];
  fg_handle p, s, z, out = 0;
  if (!get_args(env, info, 6, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &p) ||
      !arg_handle(env, a[1], &s) || !arg_handle(env, a[2], &z))
    return nullptr;
  return ret_handle(env,
                    fg_unpack_quant(g_ctx, p, s, z, (int32_t)num_or(env, a[3], 4), (int64_t)num_or(env, a[4], 128),
                                    (int64_t)num_or(env, a[5], -1), &out),
                    out);
}

// sample(logits, temperature = 1, topK = 0, topP = 1, seed?) -> handle of the chosen id (sampling.ts:35-128)
napi_value Sample(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[5];
  fg_handle lg, out = 0;
  if (!get_args(env, info, 5, a, &argc) || !need_ctx(env) || !arg_handle(env, a[0], &lg)) return nullptr;
  const bool has_seed = is_type(env, a[4], napi_number);
  return ret_handle(env,
                    fg_sample(g_ctx, lg, num_or(env, a[1], 1.0), (int32_t)num_or(env, a[2], 0), num_or(env, a[3], 1.0),
                              has_seed, (uint32_t)num_or(env, a[4], 0), &out),
                    out);
}

// configureRuntime({allowNonFinite?, maxInstructions?, maxShapeDim?, maxElements?}) (graphExecutor.ts:118-127)
napi_value ConfigureRuntime(napi_env env, napi_callback_info info) {
  size_t argc;
  napi_value a[1];
  if (!get_args(env, info, 1, a, &argc) || !need_ctx(env)) return nullptr;
  if (!is_type(env, a[0], napi_object)) return undefined(env);
  napi_value v;
  bool has = false;
  if (napi_has_named_property(env, a[0], "allowNonFinite", &has) == napi_ok && has) {
    napi_get_named_property(env, a[0], "allowNonFinite", &v);
    if (int st = fg_set_allow_non_finite(g_ctx, bool_or(env, v, false))) return throw_status(env, st);
  }
  // keys left out keep their current value (graphExecutor.ts:118-127 merges the options the same way)
  static int64_t lim[3] = {10000, 8, 1ll << 28};
  int64_t next[3] = {lim[0], lim[1], lim[2]};
  const char *keys[3] = {"maxInstructions", "maxShapeDim", "maxElements"};
  bool any = false;
  for (int i = 0; i < 3; ++i)
    if (napi_has_named_property(env, a[0], keys[i], &has) == napi_ok && has &&
        napi_get_named_property(env, a[0], keys[i], &v) == napi_ok) {
      next[i] = (int64_t)num_or(env, v, (double)lim[i]);
      any = true;
    }
  if (any) {
    if (int st = fg_configure_graph(g_ctx, next[0], (int32_t)next[1], next[2])) return throw_status(env, st);
    for (int i = 0; i < 3; ++i) lim[i] = next[i];
  }
  return undefined(env);
}

napi_value Shutdown(napi_env env, napi_callback_info) {
  if (g_ctx) {
    fg_shutdown(g_ctx);
    g_ctx = nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_live.clear();
  g_staged.clear();
  return undefined(env);
}

}  // namespace

NAPI_MODULE_INIT() {
  const napi_property_descriptor p[] = {
      {"init", nullptr, Init, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"read", nullptr, Read, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"dispose", nullptr, Dispose, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"disposeBatch", nullptr, DisposeBatch, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"getTensorInfo", nullptr, GetTensorInfo, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"mapBufferAsync", nullptr, MapBufferAsync, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"readMappedInto", nullptr, ReadMappedInto, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"executeGraph", nullptr, ExecuteGraph, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"warmupKernels", nullptr, WarmupKernels, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"getQuotaSnapshot", nullptr, GetQuotaSnapshot, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"snapshotHandles", nullptr, SnapshotHandles, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"flushGC", nullptr, FlushGC, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"configureRuntime", nullptr, ConfigureRuntime, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"uploadFloat32Array", nullptr, UploadFloat32Array, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"uploadQuant", nullptr, UploadQuant, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"matmul", nullptr, Matmul, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"qmatmul", nullptr, QMatmul, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"flashAttention", nullptr, FlashAttention, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"rmsNorm", nullptr, RmsNorm, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"rope", nullptr, Rope, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"swiglu", nullptr, Swiglu, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"add", nullptr, Add, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"embedding", nullptr, Embedding, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"unpackQuant", nullptr, UnpackQuant, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"sample", nullptr, Sample, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"shutdown", nullptr, Shutdown, nullptr, nullptr, nullptr, napi_default, nullptr},
  };
  napi_define_properties(env, exports, sizeof p / sizeof *p, p);
  return exports;
}
