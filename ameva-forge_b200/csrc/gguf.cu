// GGUF file reader and the Llama weight loader (host code).
//
// The reference has no GGUF parser (its loader is a planned component); this
// reads the published GGUF container, versions 2 and 3:
//   header   : magic "GGUF", u32 version, u64 tensor_count, u64 kv_count
//   metadata : kv_count x (string key, u32 type, value); strings are u64 length
//              + bytes; arrays are u32 element type + u64 count + elements
//   tensors  : tensor_count x (string name, u32 n_dims, u64 ne[n_dims] (ne[0]
//              innermost), u32 ggml type, u64 offset into the data section)
//   data     : starts at the next multiple of general.alignment (default 32)
// The file is memory-mapped; every length and offset is checked against the
// file size, so a malformed file is a FG_ERR_VALIDATION, never a bad read.
//
// fg_llama_load_gguf feeds the llama.cpp tensor names (token_embd, output_norm,
// output, blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,ffn_norm,ffn_gate,
// ffn_up,ffn_down}) through fg_llama_load, so tensor parallelism keeps each
// rank's shard exactly as for any other weight source.  Q and K rows are used
// as stored: GGUF Llama files already hold them in the interleaved-pair RoPE
// order the model applies.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "runtime.cuh"

extern "C" int fg_llama_load(fg_llama *m, const char *name, int32_t layer, const void *host, uint64_t bytes);
extern "C" int fg_llama_get_config(fg_llama *m, fg_llama_config *cfg);

namespace fg {
extern thread_local std::string g_last_error;
}

namespace {

// ggml tensor types read here
constexpr uint32_t kGgmlF32 = 0, kGgmlF16 = 1, kGgmlQ4_0 = 2, kGgmlQ8_0 = 8, kGgmlQ4_K = 12, kGgmlQ6_K = 14;
// metadata value types
enum : uint32_t {
  GV_U8 = 0, GV_I8 = 1, GV_U16 = 2, GV_I16 = 3, GV_U32 = 4, GV_I32 = 5, GV_F32 = 6, GV_BOOL = 7,
  GV_STR = 8, GV_ARR = 9, GV_U64 = 10, GV_I64 = 11, GV_F64 = 12
};

struct Meta {
  uint32_t type = 0;
  double num = 0;        // numeric scalar (any integer or float type, bool)
  std::string str;       // GV_STR
  uint32_t arr_type = 0; // GV_ARR
  uint64_t arr_len = 0;
};

struct Tensor {
  std::string name;
  uint32_t type = 0, ndim = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  uint64_t offset = 0, bytes = 0;
  const unsigned char *data = nullptr;
};

// Bytes of ne elements of a ggml type (row-major, blocks along ne[0]).
uint64_t type_bytes(uint32_t t, int64_t ne0, int64_t rows) {
  switch (t) {
    case kGgmlF32: return (uint64_t)ne0 * rows * 4;
    case kGgmlF16: return (uint64_t)ne0 * rows * 2;
    case kGgmlQ4_0: return ne0 % 32 ? 0 : (uint64_t)(ne0 / 32) * 18 * rows;
    case kGgmlQ8_0: return ne0 % 32 ? 0 : (uint64_t)(ne0 / 32) * 34 * rows;
    case kGgmlQ4_K: return ne0 % 256 ? 0 : (uint64_t)(ne0 / 256) * 144 * rows;
    case kGgmlQ6_K: return ne0 % 256 ? 0 : (uint64_t)(ne0 / 256) * 210 * rows;
    default: return 0;
  }
}

struct Reader {
  const unsigned char *p, *end;
  const char *what = "GGUF";
  template <class T>
  T get() {
    FG_REQUIRE((uint64_t)(end - p) >= sizeof(T), FG_ERR_VALIDATION, "GGUF: truncated %s", what);
    T v;
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    FG_REQUIRE(n <= (uint64_t)(end - p) && n < (1u << 30), FG_ERR_VALIDATION, "GGUF: bad string length in %s", what);
    std::string s((const char *)p, (size_t)n);
    p += n;
    return s;
  }
  void skip(uint64_t n) {
    FG_REQUIRE(n <= (uint64_t)(end - p), FG_ERR_VALIDATION, "GGUF: truncated %s", what);
    p += n;
  }
};

uint64_t scalar_size(uint32_t t) {
  switch (t) {
    case GV_U8: case GV_I8: case GV_BOOL: return 1;
    case GV_U16: case GV_I16: return 2;
    case GV_U32: case GV_I32: case GV_F32: return 4;
    case GV_U64: case GV_I64: case GV_F64: return 8;
    default: return 0;
  }
}

double read_scalar(Reader &r, uint32_t t) {
  switch (t) {
    case GV_U8: return r.get<uint8_t>();
    case GV_I8: return r.get<int8_t>();
    case GV_BOOL: return r.get<uint8_t>() ? 1 : 0;
    case GV_U16: return r.get<uint16_t>();
    case GV_I16: return r.get<int16_t>();
    case GV_U32: return r.get<uint32_t>();
    case GV_I32: return r.get<int32_t>();
    case GV_F32: return r.get<float>();
    case GV_U64: return (double)r.get<uint64_t>();
    case GV_I64: return (double)r.get<int64_t>();
    case GV_F64: return r.get<double>();
    default: fg::raise(FG_ERR_VALIDATION, "GGUF: unknown metadata type %u", t);
  }
}

}  // namespace

struct fg_gguf {
  int fd = -1;
  void *map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t alignment = 32;
  std::unordered_map<std::string, Meta> meta;
  std::vector<Tensor> tensors;
  std::unordered_map<std::string, size_t> index;

  ~fg_gguf() {
    if (map && map != MAP_FAILED) munmap(map, size);
    if (fd >= 0) close(fd);
  }
  const Meta *find(const std::string &k) const {
    auto it = meta.find(k);
    return it == meta.end() ? nullptr : &it->second;
  }
  double num(const std::string &k, double dflt, bool required) const {
    const Meta *m = find(k);
    if (!m || m->type == GV_STR || m->type == GV_ARR) {
      FG_REQUIRE(!required, FG_ERR_VALIDATION, "GGUF: missing numeric metadata %s", k.c_str());
      return dflt;
    }
    return m->num;
  }
  const Tensor *tensor(const std::string &name) const {
    auto it = index.find(name);
    return it == index.end() ? nullptr : &tensors[it->second];
  }

  void parse() {
    Reader r{(const unsigned char *)map, (const unsigned char *)map + size};
    r.what = "header";
    FG_REQUIRE(size >= 24 && std::memcmp(map, "GGUF", 4) == 0, FG_ERR_VALIDATION, "GGUF: bad magic");
    r.skip(4);
    version = r.get<uint32_t>();
    FG_REQUIRE(version == 2 || version == 3, FG_ERR_VALIDATION, "GGUF: version %u not supported (2, 3)", version);
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    FG_REQUIRE(n_tensors < (1u << 24) && n_kv < (1u << 24), FG_ERR_VALIDATION, "GGUF: implausible counts");
    r.what = "metadata";
    for (uint64_t i = 0; i < n_kv; ++i) {
      std::string key = r.str();
      Meta m;
      m.type = r.get<uint32_t>();
      if (m.type == GV_STR) {
        m.str = r.str();
      } else if (m.type == GV_ARR) {
        m.arr_type = r.get<uint32_t>();
        m.arr_len = r.get<uint64_t>();
        if (m.arr_type == GV_STR) {
          for (uint64_t j = 0; j < m.arr_len; ++j) r.skip(r.get<uint64_t>());
        } else {
          const uint64_t es = scalar_size(m.arr_type);
          FG_REQUIRE(es && m.arr_len <= (uint64_t)(r.end - r.p) / es, FG_ERR_VALIDATION, "GGUF: bad array %s",
                     key.c_str());
          r.skip(es * m.arr_len);
        }
      } else {
        m.num = read_scalar(r, m.type);
      }
      meta[key] = std::move(m);
    }
    alignment = (uint64_t)num("general.alignment", 32, false);
    FG_REQUIRE(alignment >= 1 && alignment <= 65536 && (alignment & (alignment - 1)) == 0, FG_ERR_VALIDATION,
               "GGUF: general.alignment %llu is not a power of two", (unsigned long long)alignment);
    r.what = "tensor table";
    tensors.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors; ++i) {
      Tensor &t = tensors[i];
      t.name = r.str();
      t.ndim = r.get<uint32_t>();
      FG_REQUIRE(t.ndim >= 1 && t.ndim <= 4, FG_ERR_VALIDATION, "GGUF: %s has %u dimensions", t.name.c_str(), t.ndim);
      int64_t rows = 1;
      for (uint32_t d = 0; d < t.ndim; ++d) {
        const uint64_t v = r.get<uint64_t>();
        FG_REQUIRE(v >= 1 && v < (1ull << 40), FG_ERR_VALIDATION, "GGUF: %s has a bad dimension", t.name.c_str());
        t.ne[d] = (int64_t)v;
        if (d) {
          FG_REQUIRE(rows <= (1ll << 40) / t.ne[d], FG_ERR_VALIDATION, "GGUF: %s is too large", t.name.c_str());
          rows *= t.ne[d];
        }
      }
      FG_REQUIRE(rows <= (1ll << 48) / t.ne[0], FG_ERR_VALIDATION, "GGUF: %s is too large", t.name.c_str());
      t.type = r.get<uint32_t>();
      t.offset = r.get<uint64_t>();
      t.bytes = type_bytes(t.type, t.ne[0], rows);
      index[t.name] = i;
    }
    const uint64_t head = (uint64_t)(r.p - (const unsigned char *)map);
    const uint64_t data0 = (head + alignment - 1) / alignment * alignment;
    for (Tensor &t : tensors) {
      if (!t.bytes) continue;  // a type this build does not read: listed, not loadable
      FG_REQUIRE(t.offset % alignment == 0 && data0 + t.offset <= size && t.bytes <= size - data0 - t.offset,
                 FG_ERR_VALIDATION, "GGUF: %s lies outside the file", t.name.c_str());
      t.data = (const unsigned char *)map + data0 + t.offset;
    }
  }
};

namespace {

int set_gerr(int st, const char *msg) {
  fg::g_last_error = msg;
  return st;
}

#define FG_GAPI_BEGIN try {
#define FG_GAPI_END                                                   \
  }                                                                   \
  catch (const fg::Error &e) {                                        \
    return set_gerr(e.status, e.what());                              \
  }                                                                   \
  catch (const std::bad_alloc &) {                                    \
    return set_gerr(FG_ERR_OUT_OF_MEMORY, "host allocation failed");  \
  }                                                                   \
  catch (const std::exception &e) {                                   \
    return set_gerr(FG_ERR_INTERNAL_GPU, e.what());                   \
  }                                                                   \
  return FG_OK;

int32_t to_fg_type(uint32_t t) {
  switch (t) {
    case kGgmlF32: return FG_F32;
    case kGgmlF16: return FG_F16;
    case kGgmlQ4_0: return FG_Q4_0;
    case kGgmlQ8_0: return FG_Q8_0;
    case kGgmlQ4_K: return FG_Q4_K;
    case kGgmlQ6_K: return FG_Q6_K;
    default: return -1;
  }
}

}  // namespace

extern "C" {

int fg_gguf_open(const char *path, fg_gguf **out) {
  FG_GAPI_BEGIN
  FG_REQUIRE(path && out, FG_ERR_VALIDATION, "fg_gguf_open: null argument");
  *out = nullptr;
  std::unique_ptr<fg_gguf> g(new fg_gguf);
  g->fd = open(path, O_RDONLY);
  FG_REQUIRE(g->fd >= 0, FG_ERR_VALIDATION, "GGUF: cannot open %s", path);
  struct stat st;
  FG_REQUIRE(fstat(g->fd, &st) == 0 && st.st_size > 0, FG_ERR_VALIDATION, "GGUF: cannot stat %s", path);
  g->size = (size_t)st.st_size;
  g->map = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
  FG_REQUIRE(g->map != MAP_FAILED, FG_ERR_VALIDATION, "GGUF: cannot map %s", path);
  g->parse();
  *out = g.release();
  FG_GAPI_END
}

int fg_gguf_close(fg_gguf *g) {
  delete g;
  return FG_OK;
}

int fg_gguf_tensor_count(const fg_gguf *g, int64_t *n) {
  FG_GAPI_BEGIN
  FG_REQUIRE(g && n, FG_ERR_VALIDATION, "fg_gguf_tensor_count: null argument");
  *n = (int64_t)g->tensors.size();
  FG_GAPI_END
}

int fg_gguf_tensor_info(const fg_gguf *g, int64_t i, const char **name, int32_t *dtype, int32_t *ndim, int64_t *dims,
                        const void **data, uint64_t *bytes) {
  FG_GAPI_BEGIN
  FG_REQUIRE(g && i >= 0 && i < (int64_t)g->tensors.size(), FG_ERR_VALIDATION, "fg_gguf_tensor_info: bad index");
  const Tensor &t = g->tensors[(size_t)i];
  if (name) *name = t.name.c_str();
  if (dtype) *dtype = to_fg_type(t.type);
  if (ndim) *ndim = (int32_t)t.ndim;
  if (dims)
    for (uint32_t d = 0; d < 4; ++d) dims[d] = t.ne[d];
  if (data) *data = t.data;
  if (bytes) *bytes = t.data ? t.bytes : 0;
  FG_GAPI_END
}

int fg_gguf_meta_number(const fg_gguf *g, const char *key, double *value) {
  FG_GAPI_BEGIN
  FG_REQUIRE(g && key && value, FG_ERR_VALIDATION, "fg_gguf_meta_number: null argument");
  *value = g->num(key, 0, true);
  FG_GAPI_END
}

int fg_gguf_meta_string(const fg_gguf *g, const char *key, const char **value) {
  FG_GAPI_BEGIN
  FG_REQUIRE(g && key && value, FG_ERR_VALIDATION, "fg_gguf_meta_string: null argument");
  const Meta *m = g->find(key);
  FG_REQUIRE(m && m->type == GV_STR, FG_ERR_VALIDATION, "GGUF: missing string metadata %s", key);
  *value = m->str.c_str();
  FG_GAPI_END
}

int fg_gguf_llama_config(const fg_gguf *g, int32_t max_position, int32_t max_batch, fg_llama_config *cfg) {
  FG_GAPI_BEGIN
  FG_REQUIRE(g && cfg, FG_ERR_VALIDATION, "fg_gguf_llama_config: null argument");
  const Meta *arch = g->find("general.architecture");
  FG_REQUIRE(arch && arch->type == GV_STR && arch->str == "llama", FG_ERR_UNSUPPORTED_OP,
             "GGUF: general.architecture must be \"llama\"");
  fg_llama_config c{};
  c.hidden_size = (int32_t)g->num("llama.embedding_length", 0, true);
  c.intermediate_size = (int32_t)g->num("llama.feed_forward_length", 0, true);
  c.num_hidden_layers = (int32_t)g->num("llama.block_count", 0, true);
  c.num_attention_heads = (int32_t)g->num("llama.attention.head_count", 0, true);
  c.num_key_value_heads = (int32_t)g->num("llama.attention.head_count_kv", c.num_attention_heads, false);
  c.rms_norm_eps = (float)g->num("llama.attention.layer_norm_rms_epsilon", 1e-5, false);
  c.rope_theta = (float)g->num("llama.rope.freq_base", 10000.0, false);
  const Tensor *emb = g->tensor("token_embd.weight");
  FG_REQUIRE(emb && emb->ndim == 2, FG_ERR_VALIDATION, "GGUF: token_embd.weight missing");
  c.vocab_size = (int32_t)emb->ne[1];
  const Tensor *q = g->tensor("blk.0.attn_q.weight");
  FG_REQUIRE(q, FG_ERR_VALIDATION, "GGUF: blk.0.attn_q.weight missing");
  c.qtype = to_fg_type(q->type);
  if (c.qtype == FG_Q6_K) c.qtype = FG_Q4_K;  // a k-quant model: each Linear Q4_K or Q6_K
  FG_REQUIRE(c.qtype == FG_Q4_0 || c.qtype == FG_Q8_0 || c.qtype == FG_Q4_K, FG_ERR_DTYPE,
             "GGUF: the Linear weights must be Q4_0, Q8_0 or Q4_K / Q6_K (blk.0.attn_q.weight has ggml type %u)",
             q->type);
  c.max_position_embeddings =
      max_position > 0 ? max_position : (int32_t)g->num("llama.context_length", 2048, false);
  c.max_batch = max_batch > 0 ? max_batch : 1;
  *cfg = c;
  FG_GAPI_END
}

int fg_llama_load_gguf(fg_llama *m, const fg_gguf *g) {
  FG_GAPI_BEGIN
  FG_REQUIRE(m && g, FG_ERR_VALIDATION, "fg_llama_load_gguf: null argument");
  fg_llama_config c{};
  if (int st = fg_llama_get_config(m, &c)) return st;
  const int H = c.hidden_size, V = c.vocab_size, L = c.num_hidden_layers;
  auto need = [&](const std::string &name, const std::vector<int64_t> &ne) -> const Tensor & {
    const Tensor *t = g->tensor(name);
    FG_REQUIRE(t, FG_ERR_VALIDATION, "GGUF: tensor %s missing", name.c_str());
    FG_REQUIRE(t->ndim == ne.size(), FG_ERR_SHAPE, "GGUF: %s has %u dimensions, expected %zu", name.c_str(), t->ndim,
               ne.size());
    for (size_t d = 0; d < ne.size(); ++d)
      FG_REQUIRE(t->ne[d] == ne[d], FG_ERR_SHAPE, "GGUF: %s dimension %zu is %lld, expected %lld", name.c_str(), d,
                 (long long)t->ne[d], (long long)ne[d]);
    FG_REQUIRE(t->data, FG_ERR_DTYPE, "GGUF: %s has ggml type %u, which this build does not read", name.c_str(),
               t->type);
    return *t;
  };
  auto load = [&](const char *as, int layer, const Tensor &t) {
    if (int st = fg_llama_load(m, as, layer, t.data, t.bytes)) fg::raise(st, "%s", fg::g_last_error.c_str());
  };
  auto load_f32 = [&](const char *as, int layer, const Tensor &t) {
    if (t.type == kGgmlF32) return load(as, layer, t);
    FG_REQUIRE(t.type == kGgmlF16, FG_ERR_DTYPE, "GGUF: %s must be F32 or F16", t.name.c_str());
    std::vector<float> f((size_t)t.ne[0]);
    const __half *h = (const __half *)t.data;
    for (size_t i = 0; i < f.size(); ++i) f[i] = __half2float(h[i]);
    if (int st = fg_llama_load(m, as, layer, f.data(), f.size() * 4)) fg::raise(st, "%s", fg::g_last_error.c_str());
  };
  auto load_q = [&](const char *as, int layer, const Tensor &t) {
    const int ft = to_fg_type(t.type);
    const bool ok = c.qtype == FG_Q4_K ? (ft == FG_Q4_K || ft == FG_Q6_K) : ft == c.qtype;
    FG_REQUIRE(ok, FG_ERR_DTYPE, "GGUF: %s is ggml type %u, the model's Linears are %s", t.name.c_str(), t.type,
               c.qtype == FG_Q4_0 ? "Q4_0" : c.qtype == FG_Q8_0 ? "Q8_0" : "Q4_K / Q6_K");
    load(as, layer, t);
  };
  {  // the embedding table is kept in fp16
    const Tensor &e = need("token_embd.weight", {H, V});
    if (e.type == kGgmlF16) {
      load("embed", -1, e);
    } else {
      FG_REQUIRE(e.type == kGgmlF32, FG_ERR_DTYPE, "GGUF: token_embd.weight must be F16 or F32");
      std::vector<__half> h((size_t)H * V);
      const float *f = (const float *)e.data;
      for (size_t i = 0; i < h.size(); ++i) h[i] = __float2half_rn(f[i]);
      if (int st = fg_llama_load(m, "embed", -1, h.data(), h.size() * 2)) fg::raise(st, "%s", fg::g_last_error.c_str());
    }
  }
  load_f32("norm", -1, need("output_norm.weight", {H}));
  // llama.cpp omits output.weight when it is tied to the embedding; that needs a quantized copy
  const Tensor *out = g->tensor("output.weight");
  FG_REQUIRE(out, FG_ERR_UNSUPPORTED_OP, "GGUF: output.weight missing (a tied embedding is not supported)");
  load_q("lm_head", -1, need("output.weight", {H, V}));
  const int d = H / c.num_attention_heads, nq = c.num_attention_heads * d, nkv = c.num_key_value_heads * d;
  for (int l = 0; l < L; ++l) {
    const std::string b = "blk." + std::to_string(l) + ".";
    load_f32("attn_norm", l, need(b + "attn_norm.weight", {H}));
    load_f32("ffn_norm", l, need(b + "ffn_norm.weight", {H}));
    load_q("q", l, need(b + "attn_q.weight", {H, nq}));
    load_q("k", l, need(b + "attn_k.weight", {H, nkv}));
    load_q("v", l, need(b + "attn_v.weight", {H, nkv}));
    load_q("o", l, need(b + "attn_output.weight", {nq, H}));
    load_q("gate", l, need(b + "ffn_gate.weight", {H, c.intermediate_size}));
    load_q("up", l, need(b + "ffn_up.weight", {H, c.intermediate_size}));
    load_q("down", l, need(b + "ffn_down.weight", {c.intermediate_size, H}));
  }
  FG_GAPI_END
}

}  // extern "C"
