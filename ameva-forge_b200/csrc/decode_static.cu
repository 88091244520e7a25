// fg_attention_decode_static: split-KV decode attention that allocates nothing.
//
// The context path (the Llama decode step) gives the split-KV kernel a scratch
// area taken from the context's stream-ordered pool.  Some callers cannot
// allocate at the moment they need one decode-attention step:
//  * a host whose device memory is already committed to its own KV-cache
//    pages under a hard VRAM quota, where any further allocation fails or
//    evicts a live cache;
//  * a decode loop on a latency-critical thread, where cudaMalloc/cudaFree
//    may synchronise the device and stall every stream in the process;
//  * a host that owns its buffers and stream but no fg_ctx (no pool exists).
// This entry point runs the same kernel with its scratch in the file-scope
// array below, so a call performs no cudaMalloc/cudaFree and uses no
// allocating library.
//
// Scratch layout (same as the pooled path): per-(sequence, KV head) arrival
// counters first, then the per-split partial results.  The counters must be
// zero when a launch starts: the array is zero-initialised when the module
// loads and every launch leaves the counters it used at zero (the last CTA of
// each head resets its counter after the merge).  The partials need no
// initial value.  Because every call uses the same array, calls on one device
// must not overlap: two launches in flight at once (on different streams, or
// from different host threads without ordering) race on the counters and
// partials and give wrong results.  Calls queued on one stream are ordered
// and safe.
#include <mutex>

#include "runtime.cuh"

namespace fg {
extern thread_local std::string g_last_error;
}

using namespace fg;

namespace {

// Static scratch limit: 2 MiB.  The split count grows until about two CTAs
// per SM are busy, so the partials peak at a few hundred (sequence, KV head,
// split) units: for Llama-2-7B (32 KV heads, d 128) at most 0.3 MB and for
// TinyLlama-1.1B (4 KV heads, group 8, d 64) at most 1.3 MB, at any batch
// and context.  Shapes whose partials need more (several hundred KV heads of
// group 8 and d 128) are rejected.
constexpr uint64_t kStaticScratchBytes = 2ull << 20;
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_addr_mu;
void *g_addr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};

// Device address of g_decode_scratch and the SM count of the current device,
// looked up once per device.  The first lookup may load this module on the
// device (lazy module loading), so the first call on each device must not be
// made while a stream is being captured.
void *scratch_address(int dev, int *num_sms) {
  FG_REQUIRE(dev >= 0 && dev < kMaxDevices, FG_ERR_VALIDATION, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_addr_mu);
  if (!g_addr[dev]) {
    void *p = nullptr;
    FG_CUDA(cudaGetSymbolAddress(&p, g_decode_scratch));
    FG_CUDA(cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev));
    g_addr[dev] = p;
  }
  *num_sms = g_sms[dev];
  return g_addr[dev];
}

}  // namespace

extern "C" int fg_attention_decode_static(const float *q, const void *k_cache, const void *v_cache, float *out,
                                          int32_t batch, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                          int64_t cache_capacity, int32_t n_kv, float scale, void *stream) {
  try {
    FG_REQUIRE(q && k_cache && v_cache && out, FG_ERR_VALIDATION, "attention_decode_static: null buffer");
    // the kernel copies K/V in 16-byte chunks (cp.async) and reads q / writes out as fp32 words; a
    // misaligned pointer would fault on the device instead of returning a status
    FG_REQUIRE((((uintptr_t)k_cache | (uintptr_t)v_cache) & 15) == 0, FG_ERR_VALIDATION,
               "attention_decode_static: k_cache and v_cache must be 16-byte aligned");
    FG_REQUIRE((((uintptr_t)q | (uintptr_t)out) & 3) == 0, FG_ERR_VALIDATION,
               "attention_decode_static: q and out must be 4-byte aligned");
    FG_REQUIRE(batch >= 1 && heads >= 1 && kv_heads >= 1, FG_ERR_SHAPE,
               "attention_decode_static: batch %d, heads %d, kv_heads %d must be >= 1", batch, heads, kv_heads);
    FG_REQUIRE(heads % kv_heads == 0, FG_ERR_SHAPE,
               "Query heads %d must be divisible by KV heads %d (GQA requirement)", heads, kv_heads);
    FG_REQUIRE(n_kv >= 1 && n_kv <= cache_capacity, FG_ERR_SHAPE,
               "attention_decode_static: n_kv %d outside [1, cache_capacity %lld]", n_kv, (long long)cache_capacity);
    AttnArgs a;
    a.q = q;
    a.k = k_cache;
    a.v = v_cache;
    a.o = out;
    a.q_f16 = 0;
    a.kv_f16 = 1;
    a.B = batch;
    a.H = heads;
    a.Hkv = kv_heads;
    a.Nq = 1;
    a.d = head_dim;
    a.q_sb = (int64_t)heads * head_dim;
    a.q_sh = head_dim;
    a.q_si = a.q_sb;
    a.o_sb = a.q_sb;
    a.o_sh = a.q_sh;
    a.o_si = a.q_si;
    a.kv_sb = (int64_t)kv_heads * cache_capacity * head_dim;
    a.kv_sh = cache_capacity * head_dim;
    a.n_kv = n_kv;
    a.scale = scale;
    a.causal = 0;
    a.scratch_batch = batch;
    FG_REQUIRE(attn_decode_supported(a), FG_ERR_SHAPE,
               "attention_decode_static: head_dim %d (64 or 128) or GQA group %d (1, 2, 4 or 8) unsupported",
               head_dim, heads / kv_heads);
    int dev = 0;
    FG_CUDA(cudaGetDevice(&dev));
    int num_sms = 0;
    void *scratch = scratch_address(dev, &num_sms);
    const int splits = attn_decode_splits(a, n_kv, num_sms, kStaticScratchBytes);
    const uint64_t need = attn_decode_scratch_bytes(a, splits);
    FG_REQUIRE(need <= kStaticScratchBytes, FG_ERR_VALIDATION,
               "attention_decode_static: batch %d x kv_heads %d x %d splits needs %llu bytes of scratch; the static "
               "scratch holds %llu bytes (use the context path for this shape)",
               batch, kv_heads, splits, (unsigned long long)need, (unsigned long long)kStaticScratchBytes);
    launch_attention_decode(a, splits, scratch, (cudaStream_t)stream);
    FG_LAUNCH_CHECK();
  } catch (const fg::Error &e) {
    fg::g_last_error = e.what();
    return e.status;
  } catch (const std::exception &e) {
    fg::g_last_error = e.what();
    return FG_ERR_INTERNAL_GPU;
  }
  return FG_OK;
}
