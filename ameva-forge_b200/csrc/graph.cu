// Graph front-end: executeGraph of the reference (packages/forge/src/tensor/
// graphExecutor.ts:487-1979) over this library's kernels.
//
// The JSON instruction list that forge-py's GraphBuilder emits
// (packages/forge-py/src/forge/graph.py:26-203) is parsed, validated with the
// reference's rules (validateInstruction, graphExecutor.ts:310-478: op
// allow-list, per-op input/param counts, shape rank / element limits, finite
// params, forbidden JSON keys, in-place optimizer ops last), then executed in
// order on the context stream.  Every node gets a tensor handle, returned as
// id -> handle; a failure disposes every tensor the call created (the
// reference's GraphTransaction rollback, graphExecutor.ts:1847-1871).
//
// Four rewrites keep the model path off the reference's materialised copies,
// all as lazy tensors whose values are computed only if something reads them:
//  * transpose(W) feeding matmul as its right operand -> x W^T read straight
//    from W (nn.Linear, forge-py nn.py:248-259); a Q4_0 / Q8_0 W runs the fused
//    dequant GEMV / tensor-core GEMM;
//  * slice(k, head h) and dim-1 cat of such slices (the GQA head repetition of
//    llama.py:116-127) -> a head map over k; flash_attention over a repeated
//    map reads k with native GQA instead of the repeated copy;
//  * cat(past, new) along the position dim of [B, H, S, d] (the KV append of
//    llama.py:111-113) -> a key/value store with spare positions: the append
//    to the newest tensor of a store writes only the new rows in place, and
//    flash_attention reads the store with its position stride.  The reference
//    copies the whole cache every step.
// Ops outside the Llama path's set (listed in exec_node) are rejected with
// FG_ERR_UNSUPPORTED_OP.
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "json.cuh"
#include "runtime.cuh"

struct fg_ctx {
  fg::Ctx c;
};

namespace fg {
extern thread_local std::string g_last_error;
const float *rope_table(Ctx *c, float base, int64_t d);

namespace {

constexpr int kR = 8;  // max rank (graphExecutor.ts:109 maxShapeDim)

// ------------------------------------------------------------------ kernels
struct GatherP {  // out[idx] = in[base + sum_i coord_i * s_i], coords of idx over dims (row-major)
  int rank;
  int64_t dim[kR], s[kR];
  int64_t base;
};

__global__ void k_gather(const float *__restrict__ in, float *__restrict__ out, int64_t n, GatherP p) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = idx, off = p.base;
    for (int i = p.rank - 1; i >= 0; --i) {
      const int64_t c = t % p.dim[i];
      t /= p.dim[i];
      off += c * p.s[i];
    }
    out[idx] = in[off];
  }
}

// slice.wgsl.ts:77-92: coordinates from the caller's output strides, then start + coord * step.
struct SliceP {
  int rank;
  int64_t start[kR], step[kR], istr[kR], ostr[kR];
};

__global__ void k_slice(const float *__restrict__ in, float *__restrict__ out, int64_t n, SliceP p) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = idx, off = 0;
    for (int i = 0; i < p.rank; ++i) {
      const int64_t os = p.ostr[i] > 1 ? p.ostr[i] : 1;
      const int64_t c = t / os;
      t %= os;
      off += (p.start[i] + c * p.step[i]) * p.istr[i];
    }
    out[idx] = in[off];
  }
}

// cat.wgsl.ts: out = [a | b] along one dimension; chunk = (a_dim + b_dim) * stride.
__global__ void k_cat(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ out, int64_t n,
                      int64_t a_dim, int64_t b_dim, int64_t stride) {
  const int64_t chunk = (a_dim + b_dim) * stride;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bi = idx / chunk, rem = idx % chunk, di = rem / stride, si = rem % stride;
    out[idx] = di < a_dim ? a[(bi * a_dim + di) * stride + si] : b[(bi * b_dim + di - a_dim) * stride + si];
  }
}

// [B][M][N] -> [B][N][M] through 32 x 33 shared tiles (transpose.wgsl.ts semantics).
__global__ void k_transpose(const float *__restrict__ in, float *__restrict__ out, int64_t M, int64_t N) {
  __shared__ float tile[32][33];
  const int64_t b = blockIdx.z, n0 = (int64_t)blockIdx.x * 32, m0 = (int64_t)blockIdx.y * 32;
  const float *ib = in + b * M * N;
  float *ob = out + b * M * N;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int64_t m = m0 + r, nn = n0 + threadIdx.x;
    if (m < M && nn < N) tile[r][threadIdx.x] = ib[m * N + nn];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int64_t nn = n0 + r, m = m0 + threadIdx.x;
    if (m < M && nn < N) ob[nn * M + m] = tile[threadIdx.x][r];
  }
}

// add/sub/mul/div with the reference's 8-D broadcast (add.wgsl.ts, broadcastParams.ts).
struct BcastP {
  int64_t d[kR], sa[kR], sb[kR];
};
enum BinOp { B_ADD, B_SUB, B_MUL, B_DIV };
template <int OP>
__global__ void k_binary(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ out, int64_t n,
                         BcastP p) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = idx, ia = 0, ib = 0;
    for (int k = kR - 1; k >= 1; --k) {
      const int64_t c = t % p.d[k];
      t /= p.d[k];
      ia += c * p.sa[k];
      ib += c * p.sb[k];
    }
    ia += t * p.sa[0];
    ib += t * p.sb[0];
    const float x = a[ia], y = b[ib];
    out[idx] = OP == B_ADD ? x + y : OP == B_SUB ? x - y : OP == B_MUL ? x * y : x / y;
  }
}

enum UnOp { U_RELU, U_NEG, U_EXP, U_LOG, U_SIGMOID, U_TANH };
template <int OP>
__global__ void k_unary(const float *__restrict__ a, float *__restrict__ out, int64_t n) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const float x = a[idx];
    out[idx] = OP == U_RELU ? fmaxf(x, 0.0f)
               : OP == U_NEG ? -x
               : OP == U_EXP ? expf(x)
               : OP == U_LOG ? logf(x)
               : OP == U_SIGMOID ? 1.0f / (1.0f + expf(-x))
                                 : tanhf(x);
  }
}

unsigned grid_for(int64_t n, int num_sms) {
  const int64_t blocks = (n + 255) / 256;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)num_sms * 16));
}

// ------------------------------------------------------------------ instructions
const char *const kAllowedOps[] = {  // graphExecutor.ts:89-95 (ALLOWED_OPS)
    "upload", "load", "matmul", "matmul_tiled", "batched_matmul", "relu", "add", "mul", "transpose", "relu_backward",
    "sub", "neg", "div", "exp", "log", "sigmoid", "tanh", "sigmoid_backward", "tanh_backward", "fill", "sum", "max",
    "sum_axis", "max_axis", "max_axis_backward", "axpy", "cat", "where", "pad", "gather", "scatter", "maxpool2d",
    "avgpool2d", "im2col", "col2im", "dropout", "permute", "matmul_bias_relu", "reshape", "slice", "slice_backward",
    "reduce_axes", "flash_attention", "rope", "rmsnorm", "swiglu", "unpack_quant", "embedding", "embedding_backward",
    "adam_step", "sgd_momentum_step", "sparse_cross_entropy", "sparse_cross_entropy_backward"};

struct Schema {  // graphExecutor.ts:361-404 (OP_SCHEMA)
  const char *op;
  int min_in;
  bool exact_in;
  int min_params;
  bool exact_params;
};
const Schema kSchemas[] = {
    {"upload", 0, true, 0, true}, {"load", 0, true, 0, true}, {"fill", 0, true, 2, true}, {"sum", 1, true, 0, true},
    {"max", 1, true, 0, true}, {"relu", 1, true, 0, true}, {"exp", 1, true, 0, true}, {"log", 1, true, 0, true},
    {"sigmoid", 1, true, 0, true}, {"tanh", 1, true, 0, true}, {"neg", 1, true, 0, true},
    {"relu_backward", 2, true, 0, false}, {"sigmoid_backward", 2, true, 0, true}, {"tanh_backward", 2, true, 0, true},
    {"pad", 1, true, 9, false}, {"sum_axis", 1, true, 2, false}, {"max_axis", 1, true, 2, false},
    {"max_axis_backward", 2, true, 2, false}, {"dropout", 1, true, 2, true}, {"maxpool2d", 1, true, 10, false},
    {"avgpool2d", 1, true, 10, false}, {"im2col", 1, true, 10, true}, {"col2im", 1, true, 10, true},
    {"transpose", 1, true, 2, false}, {"permute", 1, true, 1, false}, {"reshape", 1, true, 0, false},
    {"add", 2, true, 0, false}, {"sub", 2, true, 0, false}, {"mul", 2, true, 0, false}, {"div", 2, true, 0, false},
    {"axpy", 2, true, 2, false}, {"gather", 2, true, 7, false}, {"scatter", 2, false, 7, false},
    {"matmul", 2, true, 3, true}, {"matmul_bias_relu", 3, true, 3, true}, {"batched_matmul", 2, true, 4, false},
    {"where", 3, true, 0, false}, {"embedding", 2, true, 0, false}, {"embedding_backward", 2, true, 0, false},
    {"adam_step", 4, true, 6, false}, {"sgd_momentum_step", 3, true, 2, false},
    {"sparse_cross_entropy", 2, true, 0, false}, {"sparse_cross_entropy_backward", 3, true, 0, false},
    {"cat", 2, true, 3, true}};

struct Node {
  std::string op;
  int64_t id = 0;
  std::vector<int64_t> shape;
  int64_t numel = 1;
  std::vector<int64_t> in;
  std::vector<double> params;
  bool has_params = false;
  std::string handle;
  bool has_handle = false;
};

constexpr double kMaxSafe = 9007199254740991.0;  // Number.MAX_SAFE_INTEGER

bool safe_int(const json::Value &v) {
  return v.kind == json::Value::NUM && std::floor(v.num) == v.num && std::fabs(v.num) <= kMaxSafe;
}

Node validate(const json::Value &v, int idx, const GraphLimits &lim) {
  FG_REQUIRE(v.kind == json::Value::OBJ, FG_ERR_SECURITY, "Instruction[%d]: must be an object", idx);
  Node n;
  const json::Value *op = v.find("op");
  FG_REQUIRE(op && op->kind == json::Value::STR, FG_ERR_SECURITY, "Instruction[%d]: op must be a string", idx);
  n.op = op->str;
  bool allowed = false;
  for (const char *a : kAllowedOps) allowed = allowed || n.op == a;
  FG_REQUIRE(allowed, FG_ERR_UNSUPPORTED_OP, "Instruction[%d]: unknown op \"%s\"", idx, n.op.c_str());
  const json::Value *id = v.find("id");
  FG_REQUIRE(id && safe_int(*id) && id->num >= 1, FG_ERR_SECURITY, "Instruction[%d]: id must be a positive safe integer",
             idx);
  n.id = (int64_t)id->num;
  const json::Value *shape = v.find("shape");
  FG_REQUIRE(shape && shape->kind == json::Value::ARR, FG_ERR_SHAPE, "Instruction[%d]: shape must be an array", idx);
  FG_REQUIRE((int)shape->arr.size() <= lim.max_shape_dim, FG_ERR_SHAPE, "Instruction[%d]: shape rank must be 0–%d, got %d",
             idx, lim.max_shape_dim, (int)shape->arr.size());
  double elements = 1;
  for (const auto &d : shape->arr) {
    FG_REQUIRE(safe_int(d) && d.num >= 0, FG_ERR_SHAPE, "Instruction[%d]: shape dim must be a non-negative safe integer",
               idx);
    FG_REQUIRE(!(d.num > kMaxSafe / elements), FG_ERR_SHAPE, "Instruction[%d]: shape product integer overflow", idx);
    elements *= d.num;
    n.shape.push_back((int64_t)d.num);
  }
  FG_REQUIRE(elements <= (double)lim.max_elements, FG_ERR_SHAPE, "Instruction[%d]: tensor too large (%.0f elements > %lld)",
             idx, elements, (long long)lim.max_elements);
  n.numel = (int64_t)elements;
  const json::Value *in = v.find("in");
  FG_REQUIRE(!in || in->kind == json::Value::ARR, FG_ERR_SECURITY, "Instruction[%d]: 'in' field must be an array", idx);
  const json::Value *params = v.find("params");
  FG_REQUIRE(!params || params->kind == json::Value::ARR, FG_ERR_SECURITY,
             "Instruction[%d]: 'params' field must be an array", idx);
  const int n_in = in ? (int)in->arr.size() : 0, n_par = params ? (int)params->arr.size() : 0;
  for (const Schema &s : kSchemas) {
    if (n.op != s.op) continue;
    if (s.exact_in)
      FG_REQUIRE(n_in == s.min_in, FG_ERR_SECURITY, "Instruction[%d] op=\"%s\": expected exact %d inputs, got %d", idx,
                 s.op, s.min_in, n_in);
    else
      FG_REQUIRE(n_in >= s.min_in, FG_ERR_SECURITY, "Instruction[%d] op=\"%s\": expected min %d inputs, got %d", idx,
                 s.op, s.min_in, n_in);
    if (s.exact_params)
      FG_REQUIRE(n_par == s.min_params, FG_ERR_SECURITY, "Instruction[%d] op=\"%s\": expected exact %d params, got %d",
                 idx, s.op, s.min_params, n_par);
    else
      FG_REQUIRE(n_par >= s.min_params, FG_ERR_SECURITY, "Instruction[%d] op=\"%s\": expected min %d params, got %d",
                 idx, s.op, s.min_params, n_par);
  }
  if (params) {
    n.has_params = true;
    for (const auto &p : params->arr) {
      FG_REQUIRE(p.kind == json::Value::NUM && std::isfinite(p.num), FG_ERR_SECURITY,
                 "Instruction[%d]: param must be a finite number", idx);
      n.params.push_back(p.num);
    }
  }
  if (in)
    for (const auto &x : in->arr) {
      FG_REQUIRE(safe_int(x) && x.num >= 1, FG_ERR_SECURITY, "Instruction[%d]: 'in' ids must be positive integers", idx);
      n.in.push_back((int64_t)x.num);
    }
  if (n.op == "flash_attention") {
    if (n.shape.size() >= 4)
      FG_REQUIRE(n.shape[3] <= 256, FG_ERR_SECURITY,
                 "Instruction[%d] flash_attention: head_dim (d=%lld) exceeds maximum supported shared memory tile (256)",
                 idx, (long long)n.shape[3]);
    if (!n.params.empty())
      FG_REQUIRE(n.params[0] >= 1, FG_ERR_SECURITY, "Instruction[%d] flash_attention: H_kv must be >= 1, got %g", idx,
                 n.params[0]);
  }
  if (const json::Value *h = v.find("handle")) {
    n.has_handle = h->kind == json::Value::STR;
    if (n.has_handle) n.handle = h->str;
  }
  return n;
}

// "tensor_<hex>" (this library's handle names) or a decimal handle.
bool parse_handle(const std::string &s, fg_handle &h) {
  const char *p = s.c_str();
  int base = 10;
  if (s.rfind("tensor_", 0) == 0) {
    p += 7;
    base = 16;
  }
  if (!*p) return false;
  char *end = nullptr;
  h = std::strtoull(p, &end, base);
  return end && *end == 0 && h != 0;
}

// ------------------------------------------------------------------ executor
struct Exec {
  Ctx &c;
  fg_ctx *ctx;
  const std::vector<Node> &nodes;
  std::unordered_map<int64_t, size_t> index;                   // id -> instruction index
  std::vector<std::vector<std::pair<size_t, int>>> consumers;  // instruction -> (consumer, input slot)
  std::unordered_map<int64_t, fg_handle> id2h;
  std::vector<fg_handle> created;

  Exec(Ctx &cc, fg_ctx *x, const std::vector<Node> &n) : c(cc), ctx(x), nodes(n), consumers(n.size()) {}

  fg_handle in_h(const Node &n, int k) const {
    auto it = id2h.find(n.in[k]);
    FG_REQUIRE(it != id2h.end(), FG_ERR_SECURITY, "%s input tensor not found for id %lld", n.op.c_str(),
               (long long)n.in[k]);
    return it->second;
  }
  Tensor &in_t(const Node &n, int k) { return c.get(in_h(n, k)); }
  Tensor &in_f32(const Node &n, int k) {
    Tensor &t = in_t(n, k);
    FG_REQUIRE(t.dtype == FG_F32, FG_ERR_DTYPE, "%s input %d must be float32", n.op.c_str(), k);
    return t;
  }
  double param(const Node &n, size_t i, double dflt) const { return i < n.params.size() ? n.params[i] : dflt; }

  fg_handle new_tensor(const Node &n, Tensor **out) {
    const fg_handle h = c.make(n.shape.data(), (int)n.shape.size(), FG_F32, out);
    created.push_back(h);
    return h;
  }
  fg_handle new_lazy(const Node &n, LazyView lv) {
    Tensor t;
    t.dtype = FG_F32;
    t.ndim = (int)n.shape.size();
    for (int i = 0; i < t.ndim; ++i) t.shape[i] = n.shape[i];
    t.bytes = 4ull * (uint64_t)n.numel;
    const uint64_t src = lv.src;
    t.lazy = std::make_shared<LazyView>(std::move(lv));
    const fg_handle h = c.add(t);
    if (src) c.lazy_users.emplace(src, h);
    created.push_back(h);
    return h;
  }
  // adopt a tensor made by a C entry point: the node's shape (same element count)
  fg_handle adopt(int st, fg_handle h, const Node &n) {
    if (st != FG_OK) raise(st, "%s", g_last_error.c_str());
    created.push_back(h);
    Tensor &t = c.peek(h);
    FG_REQUIRE(t.numel() == n.numel, FG_ERR_SHAPE, "%s: result has %lld elements, instruction shape %lld",
               n.op.c_str(), (long long)t.numel(), (long long)n.numel);
    t.ndim = (int)n.shape.size();
    for (int i = 0; i < t.ndim; ++i) t.shape[i] = n.shape[i];
    return h;
  }

  // every consumer of instruction i is one of `ops` (with flash_attention only as k or v)
  bool consumers_only(size_t i, std::initializer_list<const char *> ops) const {
    for (const auto &u : consumers[i]) {
      const std::string &op = nodes[u.first].op;
      bool ok = false;
      for (const char *o : ops) ok = ok || op == o;
      if (op == "flash_attention") ok = ok && u.second >= 1;
      if (op == "matmul") ok = ok && u.second == 1;
      if (!ok) return false;
    }
    return true;
  }

  void run(const void *const *inputs, const uint64_t *input_bytes, int n_inputs);
  fg_handle exec_node(size_t i, const void *const *inputs, const uint64_t *input_bytes, int n_inputs, int &input_idx);
};

void Exec::run(const void *const *inputs, const uint64_t *input_bytes, int n_inputs) {
  for (size_t i = 0; i < nodes.size(); ++i) {
    FG_REQUIRE(index.emplace(nodes[i].id, i).second, FG_ERR_SECURITY, "Instruction[%d]: duplicate id %lld", (int)i,
               (long long)nodes[i].id);
    for (int k = 0; k < (int)nodes[i].in.size(); ++k) {
      auto it = index.find(nodes[i].in[k]);
      FG_REQUIRE(it != index.end(), FG_ERR_SECURITY, "%s input tensor not found for id %lld", nodes[i].op.c_str(),
                 (long long)nodes[i].in[k]);
      consumers[it->second].push_back({i, k});
    }
  }
  int input_idx = 0;
  for (size_t i = 0; i < nodes.size(); ++i) id2h[nodes[i].id] = exec_node(i, inputs, input_bytes, n_inputs, input_idx);
}

fg_handle Exec::exec_node(size_t i, const void *const *inputs, const uint64_t *input_bytes, int n_inputs,
                          int &input_idx) {
  const Node &n = nodes[i];
  const std::string &op = n.op;
  const cudaStream_t s = c.stream;
  Tensor *o = nullptr;

  if (op == "load") {  // graphExecutor.ts:630-650
    fg_handle h = 0;
    FG_REQUIRE(n.has_handle, FG_ERR_SECURITY, "load instruction missing handle");
    FG_REQUIRE(parse_handle(n.handle, h), FG_ERR_DISPOSED, "Tensor not found: %s", n.handle.c_str());
    Tensor &t = c.peek(h);
    bool same = t.ndim == (int)n.shape.size();
    for (int k = 0; same && k < t.ndim; ++k) same = t.shape[k] == n.shape[k];
    FG_REQUIRE(same, FG_ERR_SHAPE, "load instruction shape mismatch for handle %s", n.handle.c_str());
    return h;
  }
  if (op == "upload") {  // graphExecutor.ts:652-720
    const int k = input_idx++;
    FG_REQUIRE(k < n_inputs && inputs && inputs[k], FG_ERR_SECURITY, "upload input[%d] is not a Float32Array", k);
    FG_REQUIRE(input_bytes[k] > 0, FG_ERR_SECURITY, "upload input[%d] buffer is detached (WASM heap growth)", k);
    FG_REQUIRE(input_bytes[k] == 4ull * (uint64_t)n.numel, FG_ERR_SHAPE,
               "upload input[%d] has %llu bytes, instruction shape needs %llu", k,
               (unsigned long long)input_bytes[k], 4ull * (unsigned long long)n.numel);
    const float *f = (const float *)inputs[k];
    if (!c.allow_non_finite)
      for (int64_t e = 0; e < n.numel; ++e)
        FG_REQUIRE(std::isfinite(f[e]), FG_ERR_VALIDATION,
                   "Invalid tensor data: upload input[%d] contains NaN or Infinity at index %lld. Configure runtime "
                   "allowNonFinite=true to bypass if intended.",
                   k, (long long)e);
    const fg_handle h = new_tensor(n, &o);
    c.h2d(o->ptr, f, input_bytes[k]);
    return h;
  }
  if (op == "reshape") {  // graphExecutor.ts:722-757: a copy of the same element count
    Tensor &a = in_t(n, 0);
    FG_REQUIRE(a.dtype == FG_F32, FG_ERR_DTYPE, "reshape of a non-float32 tensor");
    FG_REQUIRE(a.numel() == n.numel, FG_ERR_SHAPE,
               "reshape size mismatch: input has %lld elements, output has %lld elements", (long long)a.numel(),
               (long long)n.numel);
    const void *src = a.ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) FG_CUDA(cudaMemcpyAsync(o->ptr, src, 4ull * n.numel, cudaMemcpyDeviceToDevice, s));
    return h;
  }
  if (op == "transpose") {  // transpose.wgsl.ts; params [M, N, (B)]
    const int64_t M = (int64_t)n.params[0], N = (int64_t)n.params[1], B = (int64_t)param(n, 2, 1);
    FG_REQUIRE(M >= 0 && N >= 0 && B >= 1 && B * M * N == n.numel, FG_ERR_SHAPE,
               "transpose params [%lld, %lld, %lld] do not match the output's %lld elements", (long long)M,
               (long long)N, (long long)B, (long long)n.numel);
    const fg_handle src = in_h(n, 0);
    Tensor &a = c.peek(src);
    const bool quant = a.dtype == FG_Q4_0 || a.dtype == FG_Q8_0 || a.dtype == FG_Q4_K || a.dtype == FG_Q6_K;
    if (B == 1 && !a.lazy && (quant || (a.dtype == FG_F32 && consumers_only(i, {"matmul"})))) {
      FG_REQUIRE(quant ? (a.shape[0] == M && a.shape[1] == N) : a.numel() == M * N, FG_ERR_SHAPE,
                 "transpose input does not hold [%lld, %lld]", (long long)M, (long long)N);
      LazyView lv;
      lv.kind = LazyView::T2D;
      lv.src = src;
      return new_lazy(n, lv);
    }
    Tensor &ai = in_f32(n, 0);
    FG_REQUIRE(ai.numel() == n.numel, FG_ERR_SHAPE, "transpose input has %lld elements, expected %lld",
               (long long)ai.numel(), (long long)n.numel);
    FG_REQUIRE(B <= 65535 && ceil_div(M, 32) <= 65535, FG_ERR_SHAPE, "transpose extent too large");
    const float *ip = (const float *)ai.ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) {
      k_transpose<<<dim3((unsigned)ceil_div(N, 32), (unsigned)ceil_div(M, 32), (unsigned)B), dim3(32, 8), 0, s>>>(
          ip, (float *)o->ptr, M, N);
      FG_LAUNCH_CHECK();
    }
    return h;
  }
  if (op == "matmul" || op == "matmul_tiled") {  // params [M, N, K]; A [M, K], B [K, N]
    const int64_t M = (int64_t)n.params[0], N = (int64_t)n.params[1], K = (int64_t)n.params[2];
    FG_REQUIRE(M >= 0 && N >= 0 && K >= 0 && M * N == n.numel, FG_ERR_SHAPE,
               "%s params [%lld, %lld, %lld] do not match the output's %lld elements", op.c_str(), (long long)M,
               (long long)N, (long long)K, (long long)n.numel);
    const fg_handle ha = in_h(n, 0), hb = in_h(n, 1);
    Tensor &a = c.get(ha);
    FG_REQUIRE(a.dtype == FG_F32 && a.numel() == M * K, FG_ERR_SHAPE, "%s: A must be float32 [%lld, %lld]",
               op.c_str(), (long long)M, (long long)K);
    Tensor &bp = c.peek(hb);
    if (bp.lazy && bp.lazy->kind == LazyView::T2D) {  // x W^T straight from W [N, K]
      const fg_handle hw = bp.lazy->src;
      Tensor &w = c.get(hw);
      FG_REQUIRE(w.shape[0] == N && w.numel() == N * K, FG_ERR_SHAPE, "%s: transposed B must come from [%lld, %lld]",
                 op.c_str(), (long long)N, (long long)K);
      if (w.dtype == FG_Q4_0 || w.dtype == FG_Q8_0 || w.dtype == FG_Q4_K || w.dtype == FG_Q6_K) {
        // x is [M, K]: give the activation tensor that shape for the quantized GEMV / GEMM
        FG_REQUIRE(a.ndim == 2 || M * K == 0 || a.shape[a.ndim - 1] == K, FG_ERR_SHAPE, "%s: A rows", op.c_str());
        fg_handle h = 0;
        const int st = fg_qmatmul(ctx, ha, hw, &h);
        return adopt(st, h, n);
      }
      FG_REQUIRE(w.dtype == FG_F32, FG_ERR_DTYPE, "%s: B must be float32", op.c_str());
      const float *ap = (const float *)c.get(ha).ptr, *wp = (const float *)w.ptr;
      const fg_handle h = new_tensor(n, &o);
      launch_matmul(c, ap, wp, (float *)o->ptr, M, K, N, /*b_trans=*/true);
      return h;
    }
    Tensor &b = c.get(hb);
    FG_REQUIRE(b.dtype == FG_F32 && b.numel() == K * N, FG_ERR_SHAPE, "%s: B must be float32 [%lld, %lld]",
               op.c_str(), (long long)K, (long long)N);
    const float *ap = (const float *)c.get(ha).ptr, *bq = (const float *)b.ptr;
    const fg_handle h = new_tensor(n, &o);
    launch_matmul(c, ap, bq, (float *)o->ptr, M, K, N, false);
    return h;
  }
  if (op == "permute") {  // permute.wgsl.ts; params = dims
    Tensor &a = in_f32(n, 0);
    const int r = (int)n.params.size();
    FG_REQUIRE(r == a.ndim && r == (int)n.shape.size(), FG_ERR_SHAPE, "permute: %d dims for a rank-%d tensor", r, a.ndim);
    GatherP p{};
    p.rank = r;
    int64_t istr[kR];
    int64_t st = 1;
    for (int k = r - 1; k >= 0; --k) {
      istr[k] = st;
      st *= a.shape[k];
    }
    bool seen[kR] = {};
    for (int k = 0; k < r; ++k) {
      const int d = (int)n.params[k];
      FG_REQUIRE(d >= 0 && d < r && !seen[d] && n.params[k] == (double)d, FG_ERR_SHAPE, "permute: dims are not a permutation");
      seen[d] = true;
      FG_REQUIRE(n.shape[k] == a.shape[d], FG_ERR_SHAPE, "permute: output dim %d is %lld, input dim %d is %lld", k,
                 (long long)n.shape[k], d, (long long)a.shape[d]);
      p.dim[k] = n.shape[k];
      p.s[k] = istr[d];
    }
    const float *ip = (const float *)a.ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) {
      k_gather<<<grid_for(n.numel, c.num_sms), 256, 0, s>>>(ip, (float *)o->ptr, n.numel, p);
      FG_LAUNCH_CHECK();
    }
    return h;
  }
  if (op == "slice") {  // slice.wgsl.ts; params [rank, start x8, step x8, in_stride x8, out_stride x8]
    FG_REQUIRE(n.params.size() >= 33, FG_ERR_SECURITY, "slice instruction needs 33 params");
    SliceP p{};
    p.rank = (int)n.params[0];
    FG_REQUIRE(p.rank >= 0 && p.rank <= kR, FG_ERR_SHAPE, "slice rank %d", p.rank);
    for (int k = 0; k < kR; ++k) {
      p.start[k] = (int64_t)n.params[1 + k];
      p.step[k] = (int64_t)n.params[9 + k];
      p.istr[k] = (int64_t)n.params[17 + k];
      p.ostr[k] = (int64_t)n.params[25 + k];
    }
    const fg_handle src = in_h(n, 0);
    Tensor &a0 = c.peek(src);
    // head selection k[:, h:h+1, :, :] of a 4-D tensor feeding the GQA repetition: a lazy head map
    if ((a0.lazy ? a0.lazy->kind == LazyView::KVCAP : a0.dtype == FG_F32) && a0.ndim == 4 && p.rank == 4 &&
        n.shape.size() == 4 &&
        n.shape[0] == a0.shape[0] && n.shape[1] == 1 && n.shape[2] == a0.shape[2] && n.shape[3] == a0.shape[3] &&
        p.start[0] == 0 && p.start[2] == 0 && p.start[3] == 0 && p.start[1] >= 0 && p.start[1] < a0.shape[1] &&
        p.step[0] == 1 && p.step[2] == 1 && p.step[3] == 1 && p.istr[3] == 1 && p.istr[2] == a0.shape[3] &&
        p.istr[1] == a0.shape[2] * a0.shape[3] && p.istr[0] == a0.shape[1] * a0.shape[2] * a0.shape[3] &&
        p.ostr[3] == 1 && p.ostr[2] == n.shape[3] && p.ostr[1] == n.shape[2] * n.shape[3] &&
        p.ostr[0] == n.shape[2] * n.shape[3] && consumers_only(i, {"cat", "flash_attention"})) {
      LazyView lv;
      lv.kind = LazyView::HEADS;
      lv.src = src;
      lv.heads.push_back((int32_t)p.start[1]);
      return new_lazy(n, lv);
    }
    Tensor &a = in_f32(n, 0);
    // every index the kernel can form lies inside the input
    int64_t lo = 0, hi = 0, rem = n.numel;
    for (int k = 0; k < p.rank; ++k) {
      const int64_t os = std::max<int64_t>(p.ostr[k], 1);
      const int64_t cmax = rem > 0 ? (std::min(rem, n.numel) - 1) / os : 0;
      rem = os;
      const int64_t a0v = p.start[k] * p.istr[k], a1v = (p.start[k] + cmax * p.step[k]) * p.istr[k];
      lo += std::min(a0v, a1v);
      hi += std::max(a0v, a1v);
    }
    FG_REQUIRE(n.numel == 0 || (lo >= 0 && hi < a.numel()), FG_ERR_SHAPE,
               "slice reads outside its input (indices %lld..%lld of %lld)", (long long)lo, (long long)hi,
               (long long)a.numel());
    const float *ip = (const float *)a.ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) {
      k_slice<<<grid_for(n.numel, c.num_sms), 256, 0, s>>>(ip, (float *)o->ptr, n.numel, p);
      FG_LAUNCH_CHECK();
    }
    return h;
  }
  if (op == "cat") {  // cat.wgsl.ts; params [a_dim, b_dim, stride]
    const int64_t ad = (int64_t)n.params[0], bd = (int64_t)n.params[1], st = std::max<int64_t>((int64_t)n.params[2], 1);
    FG_REQUIRE(ad >= 0 && bd >= 0, FG_ERR_SHAPE, "cat dims must be non-negative");
    const int64_t chunk = (ad + bd) * st;
    FG_REQUIRE(chunk > 0 ? n.numel % chunk == 0 : n.numel == 0, FG_ERR_SHAPE, "cat: %lld elements are not whole chunks of %lld",
               (long long)n.numel, (long long)chunk);
    const int64_t batch = chunk > 0 ? n.numel / chunk : 0;
    const fg_handle ha = in_h(n, 0), hb = in_h(n, 1);
    Tensor &pa = c.peek(ha), &pb = c.peek(hb);
    // dim-1 cat of two head maps over one source: the concatenated map
    if (pa.lazy && pb.lazy && pa.lazy->kind == LazyView::HEADS && pb.lazy->kind == LazyView::HEADS &&
        pa.lazy->src == pb.lazy->src && n.shape.size() == 4 && st == n.shape[2] * n.shape[3] &&
        ad == pa.shape[1] && bd == pb.shape[1] && n.shape[1] == ad + bd && n.shape[0] == pa.shape[0] &&
        consumers_only(i, {"cat", "flash_attention"})) {
      LazyView lv;
      lv.kind = LazyView::HEADS;
      lv.src = pa.lazy->src;
      lv.heads = pa.lazy->heads;
      lv.heads.insert(lv.heads.end(), pb.lazy->heads.begin(), pb.lazy->heads.end());
      return new_lazy(n, lv);
    }
    // dim-2 cat of [B, H, S, d] tensors (the KV append of llama.py:111-113): into a key/value store,
    // in place when `a` is the store's newest tensor and the store has room
    if (n.shape.size() == 4 && pa.ndim == 4 && pb.ndim == 4 && !pb.lazy && pb.dtype == FG_F32 && st == n.shape[3] &&
        ad == pa.shape[2] && bd == pb.shape[2] && n.shape[2] == ad + bd && pa.shape[0] == n.shape[0] &&
        pb.shape[0] == n.shape[0] && pa.shape[1] == n.shape[1] && pb.shape[1] == n.shape[1] &&
        pa.shape[3] == n.shape[3] && pb.shape[3] == n.shape[3] && (pa.dtype == FG_F32 || pa.lazy) &&
        (!pa.lazy || pa.lazy->kind == LazyView::KVCAP) && consumers_only(i, {"cat", "slice", "flash_attention"})) {
      const int64_t B = n.shape[0], H = n.shape[1], d = n.shape[3], len = ad + bd;
      std::shared_ptr<KVStore> store;
      if (pa.lazy && pa.lazy->store->tip == ad && pa.lazy->store->cap >= len) {
        store = pa.lazy->store;
      } else {  // a new store with room to grow; copy a's positions in
        store = std::make_shared<KVStore>();
        store->B = B;
        store->H = H;
        store->d = d;
        store->cap = std::max<int64_t>(align_up((uint64_t)(2 * len), 64), 64);
        store->bytes = 4ull * (uint64_t)(B * H * store->cap * d);
        store->ptr = (float *)c.alloc(store->bytes);
        store->ctx = &c;
        if (ad && B * H) {
          const KVStore *sa = pa.lazy ? pa.lazy->store.get() : nullptr;
          const void *src = sa ? (const void *)sa->ptr : c.get(ha).ptr;
          const int64_t spitch = sa ? sa->cap * d : ad * d;
          FG_CUDA(cudaMemcpy2DAsync(store->ptr, (size_t)(store->cap * d * 4), src, (size_t)(spitch * 4),
                                    (size_t)(ad * d * 4), (size_t)(B * H), cudaMemcpyDeviceToDevice, s));
        }
      }
      if (bd && B * H)
        FG_CUDA(cudaMemcpy2DAsync(store->ptr + ad * d, (size_t)(store->cap * d * 4), c.peek(hb).ptr, (size_t)(bd * d * 4),
                                  (size_t)(bd * d * 4), (size_t)(B * H), cudaMemcpyDeviceToDevice, s));
      store->tip = len;
      LazyView lv;
      lv.kind = LazyView::KVCAP;
      lv.store = store;
      lv.len = len;
      return new_lazy(n, lv);
    }
    Tensor &a = in_f32(n, 0);
    Tensor &b = in_f32(n, 1);
    FG_REQUIRE(a.numel() == batch * ad * st && b.numel() == batch * bd * st, FG_ERR_SHAPE,
               "cat: inputs hold %lld and %lld elements, params need %lld and %lld", (long long)a.numel(),
               (long long)b.numel(), (long long)(batch * ad * st), (long long)(batch * bd * st));
    const float *ap = (const float *)a.ptr, *bq = (const float *)c.get(hb).ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) {
      k_cat<<<grid_for(n.numel, c.num_sms), 256, 0, s>>>(ap, bq, (float *)o->ptr, n.numel, ad, bd, st);
      FG_LAUNCH_CHECK();
    }
    return h;
  }
  if (op == "add" || op == "sub" || op == "mul" || op == "div") {  // graphExecutor.ts:1522-1540
    const fg_handle ha = in_h(n, 0), hb = in_h(n, 1);
    Tensor &a = c.get(ha);
    Tensor &b = c.get(hb);
    FG_REQUIRE(a.dtype == FG_F32 && b.dtype == FG_F32, FG_ERR_DTYPE, "%s requires float32 tensors", op.c_str());
    auto pad8 = [](const int64_t *sh, int r, int64_t *d) {
      for (int k = 0; k < kR; ++k) d[k] = 1;
      for (int k = 0; k < r; ++k) d[kR - r + k] = sh[k];
    };
    BcastP p{};
    int64_t da[kR], db[kR];
    pad8(n.shape.data(), (int)n.shape.size(), p.d);
    pad8(a.shape, a.ndim, da);
    pad8(b.shape, b.ndim, db);
    int64_t sa = 1, sb = 1;
    for (int k = kR - 1; k >= 0; --k) {
      FG_REQUIRE((da[k] == 1 || da[k] == p.d[k]) && (db[k] == 1 || db[k] == p.d[k]), FG_ERR_SHAPE,
                 "%s: input shapes do not broadcast to the output shape", op.c_str());
      p.sa[k] = da[k] == 1 ? 0 : sa;
      p.sb[k] = db[k] == 1 ? 0 : sb;
      sa *= da[k];
      sb *= db[k];
    }
    const float *ap = (const float *)a.ptr, *bq = (const float *)b.ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) {
      const unsigned g = grid_for(n.numel, c.num_sms);
      float *op_ = (float *)o->ptr;
      if (op == "add") k_binary<B_ADD><<<g, 256, 0, s>>>(ap, bq, op_, n.numel, p);
      else if (op == "sub") k_binary<B_SUB><<<g, 256, 0, s>>>(ap, bq, op_, n.numel, p);
      else if (op == "mul") k_binary<B_MUL><<<g, 256, 0, s>>>(ap, bq, op_, n.numel, p);
      else k_binary<B_DIV><<<g, 256, 0, s>>>(ap, bq, op_, n.numel, p);
      FG_LAUNCH_CHECK();
    }
    return h;
  }
  if (op == "relu" || op == "neg" || op == "exp" || op == "log" || op == "sigmoid" || op == "tanh") {
    Tensor &a = in_f32(n, 0);
    FG_REQUIRE(a.numel() >= n.numel, FG_ERR_SHAPE, "%s: input smaller than the output", op.c_str());
    const float *ap = (const float *)a.ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) {
      const unsigned g = grid_for(n.numel, c.num_sms);
      float *op_ = (float *)o->ptr;
      if (op == "relu") k_unary<U_RELU><<<g, 256, 0, s>>>(ap, op_, n.numel);
      else if (op == "neg") k_unary<U_NEG><<<g, 256, 0, s>>>(ap, op_, n.numel);
      else if (op == "exp") k_unary<U_EXP><<<g, 256, 0, s>>>(ap, op_, n.numel);
      else if (op == "log") k_unary<U_LOG><<<g, 256, 0, s>>>(ap, op_, n.numel);
      else if (op == "sigmoid") k_unary<U_SIGMOID><<<g, 256, 0, s>>>(ap, op_, n.numel);
      else k_unary<U_TANH><<<g, 256, 0, s>>>(ap, op_, n.numel);
      FG_LAUNCH_CHECK();
    }
    return h;
  }
  if (op == "rope") {  // graphExecutor.ts:1257-1279; params [base, offset]
    FG_REQUIRE(n.shape.size() == 4, FG_ERR_SHAPE, "rope requires a 4D shape [B, H, N, d]");
    const int64_t d = n.shape[3];
    FG_REQUIRE(d % 2 == 0, FG_ERR_SHAPE, "rope head dim %lld must be even", (long long)d);
    Tensor &a = in_f32(n, 0);
    FG_REQUIRE(a.numel() >= n.numel, FG_ERR_SHAPE, "rope: input smaller than the output");
    const float base = (float)param(n, 0, 10000.0);
    // the offset goes through a Uint32Array (ToUint32: truncate, modulo 2^32)
    const int64_t off = (int64_t)(uint32_t)(int64_t)std::trunc(param(n, 1, 0.0));
    const float *ap = (const float *)a.ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel)
      launch_rope(ap, n.shape[0] * n.shape[1], n.shape[2], d, rope_table(&c, base, d), off, (float *)o->ptr, s);
    return h;
  }
  if (op == "rmsnorm") {  // graphExecutor.ts:1280-1303; params [eps]; in (x[, gamma])
    FG_REQUIRE(!n.shape.empty(), FG_ERR_SHAPE, "rmsnorm needs at least one dimension");
    const int64_t dim = n.shape.back(), tokens = dim ? n.numel / dim : 0;
    Tensor &x = in_f32(n, 0);
    FG_REQUIRE(x.numel() >= n.numel, FG_ERR_SHAPE, "rmsnorm: input smaller than the output");
    const float *gp = nullptr;
    if (n.in.size() >= 2) {
      Tensor &g = in_f32(n, 1);
      FG_REQUIRE(g.numel() >= dim, FG_ERR_SHAPE, "rmsnorm gamma has %lld elements, dim is %lld", (long long)g.numel(),
                 (long long)dim);
      gp = (const float *)g.ptr;
    }
    const float *xp = (const float *)in_t(n, 0).ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) launch_rmsnorm(xp, dim, gp, (float)param(n, 0, 1e-5), tokens, dim, (float *)o->ptr, s);
    return h;
  }
  if (op == "swiglu") {  // graphExecutor.ts:1304-1312
    Tensor &g = in_f32(n, 0);
    Tensor &u = in_f32(n, 1);
    FG_REQUIRE(g.numel() >= n.numel && u.numel() >= n.numel, FG_ERR_SHAPE, "swiglu: inputs smaller than the output");
    const float *gp = (const float *)g.ptr, *up = (const float *)in_t(n, 1).ptr;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) launch_swiglu(gp, up, n.numel, (float *)o->ptr, s);
    return h;
  }
  if (op == "unpack_quant") {  // graphExecutor.ts:1313-1323; params [bits, group_size]
    const int bits = (int)param(n, 0, 4);
    const int64_t gs = (int64_t)param(n, 1, 128);
    fg_handle h = 0;
    const int st = fg_unpack_quant(ctx, in_h(n, 0), in_h(n, 1), in_h(n, 2), bits, gs, n.numel, &h);
    return adopt(st, h, n);
  }
  if (op == "embedding") {  // graphExecutor.ts:1324-1338; params [tokens, dim, vocab, 0]
    FG_REQUIRE(!n.shape.empty(), FG_ERR_SHAPE, "embedding needs at least one dimension");
    const int64_t dim = n.shape.back(), tokens = dim ? n.numel / dim : 0;
    const double vocab = param(n, 2, 0);
    FG_REQUIRE(vocab > 0, FG_ERR_VALIDATION,
               "Instruction[%lld] op=\"embedding\": requires valid positive vocab_size parameter (params[2]), got %g",
               (long long)n.id, vocab);
    Tensor &w = in_t(n, 0);
    Tensor &ids = in_t(n, 1);
    FG_REQUIRE(w.dtype == FG_F32 || w.dtype == FG_F16, FG_ERR_DTYPE, "embedding weight must be float32 or float16");
    FG_REQUIRE(ids.dtype == FG_F32 || ids.dtype == FG_I32, FG_ERR_DTYPE, "embedding index must be float32 or int32");
    FG_REQUIRE(w.numel() >= (int64_t)vocab * dim && ids.numel() >= tokens, FG_ERR_SHAPE,
               "embedding: weight holds %lld elements for vocab %g x dim %lld, index %lld for %lld tokens",
               (long long)w.numel(), vocab, (long long)dim, (long long)ids.numel(), (long long)tokens);
    const void *wp = w.ptr, *ip = in_t(n, 1).ptr;
    const int wf16 = w.dtype == FG_F16, if32 = ids.dtype == FG_F32;
    const fg_handle h = new_tensor(n, &o);
    if (n.numel) launch_embedding(wp, wf16, (int64_t)vocab, dim, ip, if32, tokens, (float *)o->ptr, s);
    return h;
  }
  if (op == "flash_attention") {  // graphExecutor.ts:1220-1256; params [H_kv, scale, causal, N_kv]
    FG_REQUIRE(n.shape.size() == 4, FG_ERR_SHAPE, "flash_attention requires a 4D shape [B, H, N_q, d]");
    const int64_t B = n.shape[0], H = n.shape[1], Nq = n.shape[2], d = n.shape[3];
    int64_t Hkv = (int64_t)param(n, 0, (double)H);
    const float scale = (float)param(n, 1, 1.0 / std::sqrt((double)d));
    const int causal = param(n, 2, 0) == 1.0 ? 1 : 0;
    fg_handle hk = in_h(n, 1), hv = in_h(n, 2);
    Tensor &pk = c.peek(hk), &pv = c.peek(hv);
    int64_t Nkv = n.params.size() > 3 ? (int64_t)n.params[3] : (pk.ndim >= 2 ? pk.shape[pk.ndim - 2] : Nq);
    // K/V as repeated head maps of one [B, Hs, S, d] tensor each: attend the sources with native GQA
    if (pk.lazy && pv.lazy && pk.lazy->kind == LazyView::HEADS && pv.lazy->kind == LazyView::HEADS &&
        pk.lazy->heads == pv.lazy->heads && (int64_t)pk.lazy->heads.size() == Hkv) {
      Tensor &sk = c.peek(pk.lazy->src), &sv = c.peek(pv.lazy->src);
      const int64_t Hs = sk.shape[1];
      bool repeat = sk.ndim == 4 && sv.ndim == 4 && Hs > 0 && Hkv % Hs == 0 && sv.shape[1] == Hs;
      for (int64_t j = 0; repeat && j < Hkv; ++j) repeat = pk.lazy->heads[j] == (int32_t)(j / (Hkv / Hs));
      if (repeat) {
        hk = pk.lazy->src;
        hv = pv.lazy->src;
        Hkv = Hs;
      }
    }
    FG_REQUIRE(Hkv >= 1 && H % Hkv == 0, FG_ERR_SHAPE, "Query heads %lld must be divisible by KV heads %lld (GQA requirement)",
               (long long)H, (long long)Hkv);
    // K / V inside a key/value store: read in place with the store's position stride
    const KVStore *ks = nullptr, *vs = nullptr;
    {
      Tensor &tk = c.peek(hk), &tv = c.peek(hv);
      if (tk.lazy && tv.lazy && tk.lazy->kind == LazyView::KVCAP && tv.lazy->kind == LazyView::KVCAP &&
          tk.lazy->len == Nkv && tv.lazy->len == Nkv && tk.lazy->store->H == Hkv && tv.lazy->store->H == Hkv &&
          tk.lazy->store->B == B && tv.lazy->store->B == B && tk.lazy->store->d == d && tv.lazy->store->d == d) {
        ks = tk.lazy->store.get();
        vs = tv.lazy->store.get();
      }
    }
    Tensor &q = in_t(n, 0);
    AttnArgs a;
    if (ks) {
      FG_REQUIRE(q.dtype == FG_F32 && q.numel() == n.numel, FG_ERR_SHAPE, "flash_attention: Q must be float32 %lld elements",
                 (long long)n.numel);
      a.q = q.ptr;
      a.k = ks->ptr;
      a.v = vs->ptr;
      a.kv_sb = Hkv * ks->cap * d;
      a.kv_sh = ks->cap * d;
      FG_REQUIRE(vs->cap == ks->cap, FG_ERR_SHAPE, "flash_attention: K and V stores differ");
    } else {
      Tensor &k = c.get(hk);
      Tensor &v = c.get(hv);
      Tensor &q2 = in_t(n, 0);
      FG_REQUIRE((q2.dtype == FG_F32 || q2.dtype == FG_F16) && k.dtype == q2.dtype && v.dtype == q2.dtype, FG_ERR_DTYPE,
                 "FlashAttention requires float32 (or float16) tensors of one dtype");
      FG_REQUIRE(q2.numel() == n.numel && k.numel() == B * Hkv * Nkv * d && v.numel() == k.numel(), FG_ERR_SHAPE,
                 "flash_attention: Q holds %lld elements (expected %lld), K/V %lld/%lld (expected %lld)",
                 (long long)q2.numel(), (long long)n.numel, (long long)k.numel(), (long long)v.numel(),
                 (long long)(B * Hkv * Nkv * d));
      a.q = q2.ptr;
      a.k = k.ptr;
      a.v = v.ptr;
      a.q_f16 = a.kv_f16 = q2.dtype == FG_F16;
      a.kv_sb = Hkv * Nkv * d;
      a.kv_sh = Nkv * d;
    }
    const fg_handle h = new_tensor(n, &o);
    a.o = (float *)o->ptr;
    a.B = (int)B;
    a.H = (int)H;
    a.Hkv = (int)Hkv;
    a.Nq = (int)Nq;
    a.d = (int)d;
    a.q_sb = a.o_sb = H * Nq * d;
    a.q_sh = a.o_sh = Nq * d;
    a.q_si = a.o_si = d;
    a.n_kv = (int)Nkv;
    a.scale = scale;
    a.causal = causal;
    a.err = c.gemv.err;
    if (n.numel) launch_attention(c, a, s);
    return h;
  }
  if (op == "axpy" || op == "adam_step" || op == "sgd_momentum_step")
    raise(FG_ERR_UNSUPPORTED_OP, "op \"%s\" (optimizer commit phase) is outside this backend's inference path",
          op.c_str());
  raise(FG_ERR_UNSUPPORTED_OP, "op \"%s\" is outside this backend's Llama path (upload, load, reshape, transpose, "
                               "permute, slice, cat, matmul, add/sub/mul/div, relu/neg/exp/log/sigmoid/tanh, rope, "
                               "rmsnorm, swiglu, unpack_quant, embedding, flash_attention)",
        op.c_str());
}

}  // namespace

KVStore::~KVStore() {
  if (!ptr || !ctx) return;
  try {
    ctx->free_async(ptr, bytes);
  } catch (...) {  // a destructor must not throw; the context reports the CUDA error on its next call
  }
}

// Materialise a lazy tensor of the graph front-end (first read, or its source is being disposed).
void Ctx::materialize(fg_handle h, Tensor &t) {
  std::shared_ptr<LazyView> lv = t.lazy;
  if (lv->kind == LazyView::KVCAP) {  // positions [0, len) of every (b, h) into a dense tensor
    const KVStore &st = *lv->store;
    void *dst = alloc(t.bytes);
    if (lv->len && st.B * st.H)
      FG_CUDA(cudaMemcpy2DAsync(dst, (size_t)(lv->len * st.d * 4), st.ptr, (size_t)(st.cap * st.d * 4),
                                (size_t)(lv->len * st.d * 4), (size_t)(st.B * st.H), cudaMemcpyDeviceToDevice, stream));
    t.ptr = dst;
    t.lazy.reset();
    return;
  }
  Tensor &src = get(lv->src);
  void *dst = alloc(t.bytes);
  const int64_t n = t.numel();
  if (lv->kind == LazyView::T2D) {  // src [M, N] -> [N, M]
    const int64_t M = src.shape[0], N = src.ndim == 2 ? src.shape[1] : (M ? src.numel() / M : 0);
    const float *sp = (const float *)src.ptr;
    float *tmp = nullptr;
    if (src.dtype == FG_Q4_0 || src.dtype == FG_Q8_0 || src.dtype == FG_Q4_K || src.dtype == FG_Q6_K) {
      tmp = (float *)alloc(4ull * (uint64_t)src.numel());  // dequantise, then transpose
      if (src.dtype == FG_Q4_K)
        launch_dequant_q4k(src.ptr, src.numel() / 256, tmp, stream);
      else if (src.dtype == FG_Q6_K)
        launch_dequant_q6k(src.ptr, src.numel() / 256, tmp, stream);
      else
        launch_dequant(src.qmat(), tmp, stream);
      sp = tmp;
    }
    if (n) {
      k_transpose<<<dim3((unsigned)ceil_div(N, 32), (unsigned)ceil_div(M, 32), 1), dim3(32, 8), 0, stream>>>(
          sp, (float *)dst, M, N);
      FG_LAUNCH_CHECK();
    }
    if (tmp) free_async(tmp, 4ull * (uint64_t)src.numel());
  } else {  // HEADS: [B, Hs, S, d] -> [B, len(heads), S, d]
    const int64_t B = src.shape[0], Hs = src.shape[1], row = src.shape[2] * src.shape[3];
    const int64_t Hn = (int64_t)lv->heads.size();
    for (int64_t j = 0; j < Hn && row && B; ++j)
      FG_CUDA(cudaMemcpy2DAsync((float *)dst + j * row, (size_t)(Hn * row * 4), (const float *)src.ptr + lv->heads[j] * row,
                                (size_t)(Hs * row * 4), (size_t)(row * 4), (size_t)B, cudaMemcpyDeviceToDevice, stream));
  }
  for (auto r = lazy_users.equal_range(lv->src); r.first != r.second; ++r.first)
    if (r.first->second == h) {
      lazy_users.erase(r.first);
      break;
    }
  t.ptr = dst;
  t.lazy.reset();
}

}  // namespace fg

using namespace fg;

extern "C" int fg_execute_graph(fg_ctx *ctx, const char *instructions_json, const void *const *inputs,
                                const uint64_t *input_bytes, int32_t n_inputs, int64_t *out_ids,
                                fg_handle *out_handles, int32_t out_cap, int32_t *n_out) {
  try {
    FG_REQUIRE(ctx != nullptr, FG_ERR_VALIDATION, "null context");
    std::lock_guard<std::recursive_mutex> lk(ctx->c.mu);
    Ctx &c = ctx->c;
    FG_REQUIRE(!c.lost, FG_ERR_DEVICE_LOST, "Cannot execute graph: device was lost during a previous transaction");
    FG_CUDA(cudaSetDevice(c.device));
    FG_REQUIRE(instructions_json != nullptr, FG_ERR_SECURITY, "executeGraph: invalid JSON in instructionsJson");
    FG_REQUIRE(n_inputs >= 0 && (n_inputs == 0 || input_bytes), FG_ERR_VALIDATION, "executeGraph: bad input list");
    // 1. parse (graphExecutor.ts:523-545), rejecting keys that could pollute a JS prototype
    json::Value root;
    try {
      json::Parser ps(instructions_json);
      root = ps.parse([](const std::string &k) {
        if (k == "__proto__" || k == "constructor" || k == "prototype")
          raise(FG_ERR_SECURITY, "Forbidden property name in JSON: %s", k.c_str());
      });
    } catch (const json::ParseError &) {
      raise(FG_ERR_SECURITY, "executeGraph: invalid JSON in instructionsJson");
    }
    FG_REQUIRE(root.kind == json::Value::ARR, FG_ERR_SECURITY, "executeGraph: instructionsJson must be a JSON array");
    FG_REQUIRE((int64_t)root.arr.size() <= c.graph.max_instructions, FG_ERR_SECURITY,
               "executeGraph: too many instructions (%lld > %lld)", (long long)root.arr.size(),
               (long long)c.graph.max_instructions);
    // 2. validate (graphExecutor.ts:547-567)
    std::vector<Node> nodes;
    nodes.reserve(root.arr.size());
    for (size_t i = 0; i < root.arr.size(); ++i) nodes.push_back(validate(root.arr[i], (int)i, c.graph));
    bool in_place = false;
    std::string in_place_op;
    for (const Node &n : nodes) {
      if (n.op == "axpy" || n.op == "adam_step" || n.op == "sgd_momentum_step") {
        in_place = true;
        in_place_op = n.op;
      } else if (in_place) {
        raise(FG_ERR_SECURITY,
              "Invalid graph execution: In-place '%s' is an optimizer commit phase operation and cannot be followed "
              "by downstream op '%s' in the same transaction.",
              in_place_op.c_str(), n.op.c_str());
      }
    }
    if (out_ids && out_cap < (int32_t)nodes.size()) {  // nothing has run: report the size needed
      if (n_out) *n_out = (int32_t)nodes.size();
      raise(FG_ERR_VALIDATION, "executeGraph: output arrays hold %d entries, the graph has %d nodes", out_cap,
            (int)nodes.size());
    }
    // 3. execute; any failure disposes what this call created
    Exec ex(c, ctx, nodes);
    try {
      ex.run(inputs, input_bytes, n_inputs);
    } catch (...) {
      for (auto it = ex.created.rbegin(); it != ex.created.rend(); ++it) c.dispose(*it);
      throw;
    }
    if (n_out) *n_out = (int32_t)nodes.size();
    if (out_ids && out_handles)
      for (size_t i = 0; i < nodes.size(); ++i) {
        out_ids[i] = nodes[i].id;
        out_handles[i] = ex.id2h[nodes[i].id];
      }
    return FG_OK;
  } catch (const fg::Error &e) {
    g_last_error = e.what();
    return e.status;
  } catch (const std::bad_alloc &) {
    g_last_error = "host allocation failed";
    return FG_ERR_OUT_OF_MEMORY;
  } catch (const std::exception &e) {
    g_last_error = e.what();
    return FG_ERR_INTERNAL_GPU;
  }
}

// configureRuntime (graphExecutor.ts:98-127): instruction count, rank and element limits of graphs.
extern "C" int fg_configure_graph(fg_ctx *ctx, int64_t max_instructions, int32_t max_shape_dim, int64_t max_elements) {
  try {
    FG_REQUIRE(ctx != nullptr, FG_ERR_VALIDATION, "null context");
    std::lock_guard<std::recursive_mutex> lk(ctx->c.mu);
    FG_REQUIRE(max_instructions > 0 && max_shape_dim >= 0 && max_shape_dim <= FG_MAX_DIMS && max_elements > 0,
               FG_ERR_VALIDATION, "configure_graph: limits out of range (rank limit at most %d)", FG_MAX_DIMS);
    ctx->c.graph.max_instructions = max_instructions;
    ctx->c.graph.max_shape_dim = max_shape_dim;
    ctx->c.graph.max_elements = max_elements;
    return FG_OK;
  } catch (const fg::Error &e) {
    g_last_error = e.what();
    return e.status;
  }
}
