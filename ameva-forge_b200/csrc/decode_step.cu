// Persistent decode step: one cooperative launch runs a whole greedy decode
// step of a Llama-shaped decoder at batch 1 (tensor parallelism 1, Q4_0
// weights, fp16 KV cache) -- the per-layer sequence of llama.py:149-165 plus
// the embedding, the final norm + lm_head and the greedy pick:
//
//   EMBED | L x (QKV, ATTN, O, GATEUP, DOWN) | LM_HEAD | ARGMAX
//
// with a grid-wide barrier between phases.  The point of one launch is that
// the weights and the KV cache -- which do not depend on this step's
// activations -- stream continuously: every CTA holds two "virtual CTAs"
// (a producer thread + 8 consumer warps + a 4-stage shared-memory ring), and
// each producer walks the whole phase list ahead of its consumers, so while
// the consumers wait at a barrier or stage the next activation vector, the
// rings keep filling with the next phase's tiles.
//
// Phases:
//  * GEMV phases use the Q4_0 integer-MMA GEMV of q4_gemv.cuh with the fused
//    epilogues of the layered path (RMSNorm fused into x staging, RoPE + KV
//    append, SwiGLU, residual add), split over the 2 x gridDim virtual CTAs
//    exactly as the stand-alone GEMV splits them (same sums, same order);
//  * ATTN: split-KV attention over the cache.  Unit (KV head, split) covers a
//    run of 32-key tiles of keys [0, pos) (streamed through the ring: K tile
//    and V tile, one bulk copy each); the unit of the last split adds key
//    pos -- this step's K/V, written by the QKV phase -- from global memory,
//    so the producer never waits on this step's results.  Every unit of a
//    head publishes its partial (max, sum, output), waits for the head's
//    other splits on a per-head counter, and merges its own slice of the
//    head's outputs;
//  * ARGMAX: every CTA reduces a slice of the logits to a 64-bit key (value,
//    then lowest index; the sampler's NaN rules, sampling.ts:45-55) and
//    atomicMax-es it; after one more barrier CTA 0 writes the token, logs it
//    and advances the position.
//
// Every wait is bounded (2 s): a barrier that times out sets the device error
// word, and all threads then leave without further waiting.
#include <type_traits>

#include "q4_gemv.cuh"
#include "tmap.cuh"

namespace fg {

namespace {

constexpr int kStepStages = 4;                                   // ring stages per virtual CTA
constexpr int kStepGroups = 2;                                   // virtual CTAs per CTA
constexpr int kStepConsumers = kStepGroups * kGroupThreads;      // 512
constexpr int kStepThreads = kStepConsumers + kStepGroups * 32;  // + one producer warp per group
constexpr int kKeysPerTile = 32;
constexpr int kBoxBytes = kKeysPerTile * 128;  // one [32 keys][64 dims] fp16 box of an attention tile
// GQA groups of 4 and 8 fill half or all of the 8 columns of the attention tile on tensor cores: they take it
// (groups of 1 and 2 take the CUDA-core tile).
template <int G>
constexpr bool kMmaAttn = G >= 4;
constexpr int kBarConsumers = 3;                                 // named barrier of all consumer warps

enum Phase { PH_EMBED, PH_QKV, PH_ATTN, PH_O, PH_GATEUP, PH_DOWN, PH_LM, PH_ARGMAX };

// Phases of a layer: QKV, ATTN, O, GATEUP, DOWN; under tensor parallelism O and DOWN produce partial
// sums that every rank exchanges (see fold_index).
__device__ __forceinline__ Phase phase_kind(int p, int L, int per) {
  if (p == 0) return PH_EMBED;
  if (p <= per * L) return (Phase)(PH_QKV + (p - 1) % per);
  return p == per * L + 1 ? PH_LM : PH_ARGMAX;
}
// Tensor parallelism: the phase after an exchange adds the ranks' partial sums to the residual while it
// stages its input -- GATEUP folds its layer's o_proj exchange 2l, QKV of layer l + 1 and LM the
// down_proj exchange 2l + 1.  -1: no fold.
__device__ __forceinline__ int fold_index(int p, int L) {
  if (p == 5 * L + 1) return 2 * L - 1;
  if (p < 1 || p > 5 * L) return -1;
  const int l = (p - 1) / 5, k = (p - 1) % 5;
  if (k == 3) return 2 * l;
  if (k == 0 && l > 0) return 2 * l - 1;
  return -1;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_volatile_int(const int *p) { return *reinterpret_cast<const volatile int *>(p); }
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Flag words of rank r's exchange region: key[8] at word 8 and kflag[8] at word 16 (the greedy pick), the
// exchange counter at word kXcnt (every CTA of every rank adds one per exchange).
constexpr int kXcnt = 24;
__device__ __forceinline__ unsigned long long *xflag_words(const StepArgs &A, int r) {
  return reinterpret_cast<unsigned long long *>(reinterpret_cast<unsigned char *>(A.xr[r]) + A.xflags);
}
// Wait until every other rank has published sequence `seq` in this rank's word array w[8] (bounded).
__device__ __noinline__ bool wait_peers(const StepArgs &A, const unsigned long long *w, unsigned long long seq) {
  const uint64_t t0 = global_ns();
  for (int r = 0; r < A.tp; ++r) {
    if (r == A.rank) continue;
    while (ld_acquire_sys_u64(w + r) < seq) {
      if (ld_volatile_int(A.err) != 0) return false;
      if (global_ns() - t0 > kWaitTimeoutNs) {
        atomicCAS(A.err, 0, DEVERR_GRID);
        return false;
      }
    }
  }
  return true;
}

// Wait (bounded acquire poll at system scope) until this rank's exchange counter reaches `target`.
__device__ __noinline__ bool wait_xcnt(const StepArgs &A, unsigned long long target) {
  const unsigned long long *c = xflag_words(A, A.rank) + kXcnt;
  if (ld_acquire_sys_u64(c) >= target) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (ld_acquire_sys_u64(c) >= target) return true;
    if (ld_volatile_int(A.err) != 0) return false;
    if (global_ns() - t0 > kWaitTimeoutNs) {
      atomicCAS(A.err, 0, DEVERR_GRID);
      return false;
    }
  }
}

// Work index of this CTA's group grp.  Single GPU: group-major (group 0 of every CTA, then group 1), so a
// phase with fewer units than virtual CTAs puts at most one of them on an SM until every SM has one,
// instead of filling both groups of the first SMs while the last ones idle.  The tensor-parallel instance
// keeps CTA-major indices (2 b + grp).
template <bool TP>
__device__ __forceinline__ int work_index(int grp) {
  return TP ? (int)blockIdx.x * kStepGroups + grp : grp * (int)gridDim.x + (int)blockIdx.x;
}

// Grid-wide barrier, one calling thread per CTA (after a CTA-wide barrier).
// bar[0] counts arrivals and is never reset; bar[1] counts launches (the
// epoch).  Barrier k of the launch with epoch E completes when the count
// reaches (E * barriers_per_launch + k + 1) * CTAs, so an arrival is one
// posted atomic add and the wait is a bounded acquire poll.
__device__ bool grid_sync(unsigned long long *count, unsigned long long target, int *err) {
  // release: this CTA's phase results (ordered before this thread by the CTA barrier) are visible
  // to every CTA that acquires the count
  asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(count) : "memory");
  if (ld_acquire_u64(count) >= target) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    __nanosleep(32);
    if (ld_acquire_u64(count) >= target) return true;
    if (ld_volatile_int(err) != 0) return false;
    if (global_ns() - t0 > kWaitTimeoutNs) {
      atomicCAS(err, 0, DEVERR_GRID);
      return false;
    }
  }
}

// Wait (bounded acquire poll) until the counter reaches `target`.
__device__ bool wait_count(const unsigned long long *cnt, unsigned long long target, int *err) {
  if (ld_acquire_u64(cnt) >= target) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (ld_acquire_u64(cnt) >= target) return true;
    if (ld_volatile_int(err) != 0) return false;
    if (global_ns() - t0 > kWaitTimeoutNs) {
      atomicCAS(err, 0, DEVERR_GRID);
      return false;
    }
  }
}


// Split of the attention phase: units = KV heads x splits, at most one unit per
// virtual CTA; split s of a head covers tiles [s*nt/S, (s+1)*nt/S) of keys
// [0, npos); the last split also takes key npos.
struct AttnSplit {
  int S, nt, units;
};
__device__ __forceinline__ AttnSplit attn_split(int npos, int Hkv, int P) {
  AttnSplit a;
  a.nt = (npos + kKeysPerTile - 1) / kKeysPerTile;
  // splits per head: enough units for every group, but at least 2 tiles per unit (a split's fixed cost
  // -- q load, first-tile latency, its share of the merge -- outweighs a single tile; 2 tiles per unit
  // measured faster than 4 or 8 on short contexts); <= 512 so the merge weights [S][G] fit the 8 G D o area
  a.S = max(1, min(min(P / Hkv, 512), max(1, a.nt / 2)));
  a.units = Hkv * a.S;
  return a;
}

}  // namespace

// The greedy pick over every rank's vocabulary shard: publish this rank's best key to the others,
// wait for theirs, return the maximum (or `key` unchanged and false on a timeout).
__device__ __noinline__ bool exchange_keys(const StepArgs &A, unsigned long long kseq, unsigned long long &key) {
  for (int r = 0; r < A.tp; ++r) {
    if (r == A.rank) continue;
    unsigned long long *wr = xflag_words(A, r);
    wr[8 + A.rank] = key;
    st_release_sys_u64(wr + 16 + A.rank, kseq);
  }
  const unsigned long long *wl = xflag_words(A, A.rank);
  if (!wait_peers(A, wl + 16, kseq)) return false;
  for (int r = 0; r < A.tp; ++r)
    if (r != A.rank) {
      const unsigned long long kr = *reinterpret_cast<const volatile unsigned long long *>(wl + 8 + r);
      key = kr > key ? kr : key;
    }
  return true;
}

// GEMV operand of phase p (layer l, whose weights and cache `lay` describes; unused for LM_HEAD).
__device__ __forceinline__ void gemv_phase(const StepArgs &A, Phase ph, int l, const StepLayer *lay, QMat &w,
                                           const float *&x, const float *&gamma, Epilogue &ep) {
  const auto xchg = [&](Epilogue &e, int xi) {  // partial sums to every rank's part[xi % 2][this rank]
    e.mode = EPI_XCHG;
    e.xdst = A.xr;
    e.xoff = ((int64_t)(xi & 1) * A.tp + A.rank) * A.H;
    e.nx = A.tp;
  };
  ep = Epilogue();
  if (ph == PH_LM) {
    w = A.lm_head;
    x = A.h;
    gamma = A.norm;
    ep.mode = EPI_PLAIN;
    ep.y = A.logits;
    ep.ldy = A.vocab_l;
    return;
  }
  const StepLayer &Ly = *lay;
  switch (ph) {
    case PH_QKV:
      w = Ly.qkv;
      x = A.h;
      gamma = Ly.attn_norm;
      ep.mode = EPI_QKV;
      ep.q_out = A.q;
      ep.k_cache = Ly.k;
      ep.v_cache = Ly.v;
      ep.n_q = A.Hq * A.d;
      ep.n_kv = A.Hkv * A.d;
      ep.head_dim = A.d;
      ep.cap = A.cap;
      ep.tokens_per_seq = 1;
      ep.pos = A.pos;
      ep.inv_freq = A.inv_freq;
      break;
    case PH_O:
      w = Ly.o;
      x = A.att;
      gamma = nullptr;
      ep.mode = EPI_PLAIN;
      ep.y = A.h;
      ep.resid = A.h;
      ep.ldy = A.H;
      if (A.tp > 1) xchg(ep, 2 * l);
      break;
    case PH_GATEUP:
      w = Ly.gateup;
      x = A.h;
      gamma = Ly.ffn_norm;
      ep.mode = EPI_SWIGLU;
      ep.y = A.ffn;
      ep.ldy = A.I;
      break;
    default:  // PH_DOWN
      w = Ly.down;
      x = A.ffn;
      gamma = nullptr;
      ep.mode = EPI_PLAIN;
      ep.y = A.h;
      ep.resid = A.h;
      ep.ldy = A.H;
      if (A.tp > 1) xchg(ep, 2 * l + 1);
      break;
  }
}

namespace {

// The ring stages one virtual CTA's producer fills over a whole launch, in consumption order: GEMV phases
// give the tiles of its strips (one contiguous copy each), ATTN phases the 32-key tiles of its unit (K and V
// as swizzled tensor boxes).
template <int D, int G>
struct StepCursor {
  const StepArgs *A;
  int p, nphase, L, vk, P, npos;
  int kind;  // 0: between phases, 1: GEMV strips, 2: attention tiles
  const unsigned char *src;
  int nq, u, u1, q0;
  const CUtensorMap *km, *vm;  // the unit's layer's K and V cache maps
  int hk, t, t1, l_;

  __device__ void init(const StepArgs &a, int vk_, int P_, int npos_) {
    A = &a;
    p = -1;
    L = a.L;
    nphase = 5 * L + 3;
    vk = vk_;
    P = P_;
    npos = npos_;
    kind = 0;
  }
  // The next stage: a GEMV tile (a, ba), an attention tile of contiguous rows (K rows at a, V rows at b,
  // ba = bb bytes each; GQA groups of 1 and 2) or an attention tile of tensor boxes (keys [y, y + 32) of KV head
  // z in kmap and vmap, ba bytes in all; GQA groups of 4 and 8); false after the last stage.
  __device__ bool next(const void *&a, uint32_t &ba, const void *&b, uint32_t &bb, const CUtensorMap *&kmap,
                       const CUtensorMap *&vmap, int &y, int &z) {
    for (;;) {
      if (kind == 1 && u < u1) {
        a = src + ((int64_t)u * nq + q0) * kQ4QuadBytes;
        ba = (uint32_t)min(kQ4TileQuads, nq - q0) * kQ4QuadBytes;
        b = nullptr;
        bb = 0;
        kmap = vmap = nullptr;
        q0 += kQ4TileQuads;
        if (q0 >= nq) {
          q0 = 0;
          ++u;
        }
        return true;
      }
      if (kind == 2 && t < t1) {
        if constexpr (kMmaAttn<G>) {
          a = b = nullptr;
          ba = 2u * (D / 64) * kBoxBytes;  // whole boxes land, keys past the cache included (as zeros)
          bb = 0;
          kmap = km;
          vmap = vm;
          y = t * kKeysPerTile;
          z = hk;
        } else {
          const int nk = min(kKeysPerTile, npos - t * kKeysPerTile);
          const int64_t off = ((int64_t)hk * A->cap + (int64_t)t * kKeysPerTile) * D;
          a = A->layers[l_].k + off;
          b = A->layers[l_].v + off;
          ba = bb = (uint32_t)nk * D * 2;
          kmap = vmap = nullptr;
        }
        ++t;
        return true;
      }
      if (++p >= nphase) return false;
      const Phase ph = phase_kind(p, L, 5);
      const int l = (p - 1) / 5;
      kind = 0;
      if (ph == PH_ATTN) {
        const AttnSplit sp = attn_split(npos, A->Hkv, P);
        if (vk < sp.units) {
          const int s = vk % sp.S;
          hk = vk / sp.S;
          t = s * sp.nt / sp.S;
          t1 = (s + 1) * sp.nt / sp.S;
          km = static_cast<const CUtensorMap *>(A->kv_maps) + 2 * l;
          vm = km + 1;
          l_ = l;
          kind = 2;
        }
      } else if (ph >= PH_QKV && ph <= PH_LM) {
        QMat w;
        const float *x, *gm;
        Epilogue ep;
        gemv_phase(*A, ph, l, A->layers + l, w, x, gm, ep);
        const Sched sc = make_sched(w.N, kQ4StripRows, 1, vk, P);
        src = reinterpret_cast<const unsigned char *>(w.qs);
        nq = (int)w.row_words;
        u = sc.u0;
        u1 = sc.u1;
        q0 = 0;
        kind = 1;
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Attention consumer: one unit (KV head hk, keys of tiles [t0, t1) + the
// current key when `last`) on the 8 warps of a group, on tensor cores
// (mma.sync m16n8k16, fp16 operands, fp32 accumulation).
//
// Ring slot layout (TMA tensor boxes, 128-byte swizzle): K as D/64 boxes of
// [32 keys][64 dims] fp16, 4 KB each, then V the same way.  Row r of a box
// holds its 16-byte chunk c at chunk position c ^ (r & 7), so the eight rows
// of an ldmatrix 8x8 block sit in eight different bank groups.  Rows past the
// tile's valid keys hold other cache positions (or zeros past the cache):
// their scores are masked and their V entries zeroed in registers.
//
// Warp w takes key block kb = w & 1 (keys 16 kb .. 16 kb + 15 of every tile)
// and output dims [dset D/4, (dset + 1) D/4), dset = w >> 1.  Per tile:
//   S^T[16 keys][8 g] = K_kb q^T   (A = K rows by ldmatrix, B = q fragments,
//                                   q = qh + ql as two fp16 halves, two MMAs
//                                   per 16 dims: q keeps ~22 bits)
//   online softmax per g over the warp's keys (running max, per-lane partial
//   sums reduced once at the end);
//   O^T[dims][g] += V^T[dims][16 keys] P^T (A = V rows by ldmatrix.trans,
//                                   B = P^T by movmatrix; P = ph + pl, two MMAs)
// The four warps of a key block compute the same scores and softmax state, so
// the unit ends with a two-way merge (kb 0, kb 1) per output dim.  Columns
// g >= G are padding (q = 0) and are never stored.
// ---------------------------------------------------------------------------
constexpr int r4(int x) { return (x + 3) & ~3; }

template <int D, int G>
struct AttnCfgM {
  static_assert(D == 64 || D == 128, "head_dim");
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "GQA group");
  static constexpr int NCH = D / 16;   // 16-dim chunks of a key row
  static constexpr int NPC = NCH / 4;  // chunks of output dims per warp
  static constexpr int NB = D / 64;    // boxes per K (or V) tile
  // shared scratch (floats): q fragments [NCH][32 lanes][4 words], warp states (m, l) [8 warps][8 g][2],
  // o [2 kb][G][D], and this step's key as a one-key tile in the ring layout with 16-row boxes (K, then V)
  static constexpr int SM_QF = 0, SM_ML = NCH * 32 * 4, SM_O = SM_ML + 8 * 8 * 2, SM_KV = r4(SM_O + 2 * G * D),
                       SM_END = SM_KV + 2 * NB * (kBoxBytes / 2) / 4;
};
static_assert(2 * 2 * kBoxBytes <= kQ4TileBytes, "attention tile fits a ring slot");

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}
// Shared-memory address of 16-byte chunk cc (dims 8 cc .. 8 cc + 7) of row `row` of a tile of 128-byte rows in
// boxes of `box` bytes (64 dims per box, 128-byte swizzle).
__device__ __forceinline__ uint32_t swz_chunk(uint32_t tile, int box, int row, int cc) {
  return tile + (uint32_t)((cc >> 3) * box + row * 128 + (((cc & 7) ^ (row & 7)) << 4));
}

// A warp's running state: max and per-lane partial sum of its two g columns, O^T fragments of its dims.
template <int D, int G>
struct WarpAttnM {
  float m[2], l[2];
  float o[AttnCfgM<D, G>::NPC][4];
};

template <int D, int G>
__device__ __forceinline__ void attn_warp_init_m(WarpAttnM<D, G> &W) {
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    W.m[j] = -INFINITY;
    W.l[j] = 0.0f;
  }
#pragma unroll
  for (int c = 0; c < AttnCfgM<D, G>::NPC; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) W.o[c][j] = 0.0f;
}

// One tile for warp w: key block kb = w & 1 of the K tile at ktile and the V tile at vtile (shared-memory
// addresses, boxes of `box` bytes), nk valid keys.
template <int D, int G>
__device__ __forceinline__ void attn_mma_tile(uint32_t ktile, uint32_t vtile, int box, int nk, const uint4 *qf,
                                              WarpAttnM<D, G> &W, int w, int lane) {
  using C = AttnCfgM<D, G>;
  const int kb = w & 1, dset = w >> 1;
  const int mi = lane >> 3, r8 = lane & 7;
  // ---- scores S^T of keys 16 kb + (lane / 4, + 8), columns g = 2 (lane % 4) + (0, 1)
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  {
    const int row = kb * 16 + r8 + (mi & 1) * 8;
#pragma unroll
    for (int ch = 0; ch < C::NCH; ++ch) {
      uint32_t a[4];
      ldsm_x4(a, swz_chunk(ktile, box, row, 2 * ch + (mi >> 1)));
      const uint4 q = qf[ch * 32 + lane];
      mma_f16(s, a, q.x, q.y);
      mma_f16(s, a, q.z, q.w);
    }
  }
  const int key0 = kb * 16 + (lane >> 2);
  const bool v0 = key0 < nk, v1 = key0 + 8 < nk;
  const float sv[4] = {v0 ? s[0] : -INFINITY, v0 ? s[1] : -INFINITY, v1 ? s[2] : -INFINITY, v1 ? s[3] : -INFINITY};
  float tm[2] = {fmaxf(sv[0], sv[2]), fmaxf(sv[1], sv[3])};
#pragma unroll
  for (int o = 4; o < 32; o <<= 1)
#pragma unroll
    for (int j = 0; j < 2; ++j) tm[j] = fmaxf(tm[j], __shfl_xor_sync(0xffffffffu, tm[j], o));
  float al[2], p[4];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float mn = fmaxf(W.m[j], tm[j]);
    al[j] = mn == -INFINITY ? 1.0f : expf(W.m[j] - mn);
    p[j] = sv[j] == -INFINITY ? 0.0f : expf(sv[j] - mn);
    p[j + 2] = sv[j + 2] == -INFINITY ? 0.0f : expf(sv[j + 2] - mn);
    W.l[j] = W.l[j] * al[j] + (p[j] + p[j + 2]);
    W.m[j] = mn;
  }
  // ---- P^T as the B operand: fp16 hi and lo parts, rows = keys turned into columns by movmatrix
  const uint32_t h0 = pack_h2(p[0], p[1]), h1 = pack_h2(p[2], p[3]);
  const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&h0));
  const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&h1));
  const uint32_t l0 = pack_h2(p[0] - f0.x, p[1] - f0.y), l1 = pack_h2(p[2] - f1.x, p[3] - f1.y);
  const uint32_t bh0 = movm_t(h0), bh1 = movm_t(h1), bl0 = movm_t(l0), bl1 = movm_t(l1);
  // ---- O^T += V^T P^T over this warp's dims
  const int vrow = kb * 16 + r8 + (mi >> 1) * 8;
  const int kc = kb * 16 + 2 * (lane & 3);  // keys of this lane's A elements: kc, kc + 1 (a0, a1), + 8 (a2, a3)
  const bool partial = nk < 32;
#pragma unroll
  for (int c = 0; c < C::NPC; ++c) {
    uint32_t a[4];
    ldsm_x4_t(a, swz_chunk(vtile, box, vrow, 2 * (dset * C::NPC + c) + (mi & 1)));
    if (partial) {  // rows past the valid keys: zero their V entries (p is 0 there, but 0 * inf is not)
      const uint32_t m01 = (kc < nk ? 0x0000FFFFu : 0u) | (kc + 1 < nk ? 0xFFFF0000u : 0u);
      const uint32_t m23 = (kc + 8 < nk ? 0x0000FFFFu : 0u) | (kc + 9 < nk ? 0xFFFF0000u : 0u);
      a[0] &= m01;
      a[1] &= m01;
      a[2] &= m23;
      a[3] &= m23;
    }
    W.o[c][0] *= al[0];
    W.o[c][1] *= al[1];
    W.o[c][2] *= al[0];
    W.o[c][3] *= al[1];
    mma_f16(W.o[c], a, bh0, bh1);
    mma_f16(W.o[c], a, bl0, bl1);
  }
}

// ---------------------------------------------------------------------------
// Attention consumer for GQA groups of 1 and 2 (CUDA cores): one unit on the
// 8 warps of a group; ring slot = K rows [32][D] fp16 then V rows [32][D]
// fp16, contiguous (one bulk copy each).  Warp w takes keys [4w, 4w + 4) of
// every tile and keeps its own online softmax (running max, sum and output
// in registers), so no group barrier runs inside a unit; the eight warp
// states merge once at its end.  With one or two query rows per KV head the
// tensor-core tile below would leave 7 or 6 of its 8 columns empty; this
// path issues fewer instructions per key there.
// ---------------------------------------------------------------------------
template <int D, int G>
struct AttnCfgS {
  static_assert(D == 64 || D == 128, "head_dim");
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "GQA group");
  static constexpr int NV = D / 64;              // q.k: lane 8 kk + c takes 16-byte chunks c + 8 v (v < NV) of key kk
  static constexpr int DL = D / 32;              // p.V: lane takes dims [DL lane, DL lane + DL)
  static constexpr int GL = 8 / G;               // lanes of a key that end the score reduction with the same g
  static constexpr bool QREG = G * NV * 8 <= 32;  // this lane's q slice lives in registers
  // shared scratch (floats): q [G][D] (chunk halves swizzled), per-warp p [8][G][4] + alpha [8][G],
  // warp states (m, l) [8][G], o [8][G][D] and the K and V rows of this step's key (D fp16 each)
  static constexpr int SM_Q = 0, SM_P = G * D, SM_ML = r4(SM_P + 8 * G * 5), SM_O = r4(SM_ML + 16 * G),
                       SM_KV = SM_O + 8 * G * D, SM_END = SM_KV + D;
};

// Offset of q element dd of a row: the two float4 halves of 8-dim chunk k swap places when bit 2 of k is
// set, so the eight lanes of a key read their chunks' first halves from eight distinct bank groups.
__device__ __forceinline__ int q_swz(int dd) {
  const int k = dd >> 3;
  return (k << 3) | (((dd & 7) + (((k >> 2) & 1) << 2)) & 7);
}

template <int D, int G>
struct WarpAttnS {
  using C = AttnCfgS<D, G>;
  float q[C::QREG ? G * C::NV * 8 : 1];  // q[g][chunk c + 8 v][e] of this lane
  float m, l;                           // running max and sum of this lane's g (= c / GL)
  float o[G][C::DL];                    // output dims [DL lane, DL lane + DL) of every g
};

// q element e of chunk (c + 8 v) of row g, read from shared memory (swizzled) or this lane's registers.
template <int D, int G>
__device__ __forceinline__ void attn_q8s(const WarpAttnS<D, G> &W, const float *sq, int g, int v, int c, float (&qv)[8]) {
  using C = AttnCfgS<D, G>;
  if constexpr (C::QREG) {
#pragma unroll
    for (int e = 0; e < 8; ++e) qv[e] = W.q[(g * C::NV + v) * 8 + e];
  } else {
    const int k = c + 8 * v, h = (k >> 2) & 1;
    const float4 a = *reinterpret_cast<const float4 *>(sq + g * D + k * 8 + 4 * h);
    const float4 b = *reinterpret_cast<const float4 *>(sq + g * D + k * 8 + 4 * (h ^ 1));
    qv[0] = a.x, qv[1] = a.y, qv[2] = a.z, qv[3] = a.w, qv[4] = b.x, qv[5] = b.y, qv[6] = b.z, qv[7] = b.w;
  }
}

template <int D, int G>
__device__ __forceinline__ void attn_warp_init_s(WarpAttnS<D, G> &W, const float *sq, int lane) {
  using C = AttnCfgS<D, G>;
  if constexpr (C::QREG) {
    const int c = lane & 7;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int v = 0; v < C::NV; ++v) {
        const int k = c + 8 * v, h = (k >> 2) & 1;
        const float4 a = *reinterpret_cast<const float4 *>(sq + g * D + k * 8 + 4 * h);
        const float4 b = *reinterpret_cast<const float4 *>(sq + g * D + k * 8 + 4 * (h ^ 1));
        float *d = &W.q[(g * C::NV + v) * 8];
        d[0] = a.x, d[1] = a.y, d[2] = a.z, d[3] = a.w, d[4] = b.x, d[5] = b.y, d[6] = b.z, d[7] = b.w;
      }
  }
  W.m = -INFINITY;
  W.l = 0.0f;
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int t = 0; t < C::DL; ++t) W.o[g][t] = 0.0f;
}

// Keys [4w, 4w + 4) of one tile for warp w: key j's K row at kt + j D, its V row at vt + j D; keys
// j >= nk are masked and their rows never read.  GLB: the rows are in global memory, written by
// other CTAs of this launch (read through L2).  sp: this warp's p / alpha exchange area (G >= 4).
template <int D, int G, bool GLB>
__device__ __forceinline__ void attn_warp_tile(const __half *kt, const __half *vt, int nk, const float *sq, float *sp,
                                               WarpAttnS<D, G> &W, int w, int lane) {
  using C = AttnCfgS<D, G>;
  const int kk = lane >> 3, c = lane & 7, j = 4 * w + kk;
  const bool valid = j < nk;
  // ---- partial dots of this lane's chunks for every g (two chains each)
  float sa[G], sb[G];
#pragma unroll
  for (int g = 0; g < G; ++g) sa[g] = sb[g] = 0.0f;
#pragma unroll
  for (int v = 0; v < C::NV; ++v) {
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (valid) {
      const uint4 *src = reinterpret_cast<const uint4 *>(kt + (int64_t)j * D + (c + 8 * v) * 8);
      raw = GLB ? __ldcg(src) : *src;
    }
    float kf[8];
    const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h2[e]);
      kf[2 * e] = f.x;
      kf[2 * e + 1] = f.y;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float qv[8];
      attn_q8s<D, G>(W, sq, g, v, c, qv);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        sa[g] = fmaf(qv[e], kf[e], sa[g]);
        sb[g] = fmaf(qv[e + 1], kf[e + 1], sb[g]);
      }
    }
  }
  // ---- reduce over the 8 lanes of the key, scattering g: while more than one g is left, each xor round
  // halves them (the lane with the bit set keeps the upper half); then plain butterfly sums
  float s[G];
#pragma unroll
  for (int g = 0; g < G; ++g) s[g] = sa[g] + sb[g];
  {
    int cnt = G;
#pragma unroll
    for (int bit = 4; bit >= 1; bit >>= 1) {
      if (cnt > 1) {
        const int h = cnt / 2;
        const bool up = (c & bit) != 0;
#pragma unroll
        for (int i2 = 0; i2 < G / 2; ++i2) {
          if (i2 < h) {
            const float send = up ? s[i2] : s[i2 + h];
            const float keep = up ? s[i2 + h] : s[i2];
            s[i2] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
          }
        }
        cnt = h;
      } else {
        s[0] += __shfl_xor_sync(0xffffffffu, s[0], bit);
      }
    }
  }
  // ---- online softmax of this lane's g over the warp's 4 keys
  const float sv = valid ? s[0] : -INFINITY;
  float tm = fmaxf(sv, __shfl_xor_sync(0xffffffffu, sv, 8));
  tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 16));
  const float mn = fmaxf(W.m, tm);
  const float al = mn == -INFINITY ? 1.0f : expf(W.m - mn);
  const float p = valid ? expf(sv - mn) : 0.0f;
  float ps = p + __shfl_xor_sync(0xffffffffu, p, 8);
  ps += __shfl_xor_sync(0xffffffffu, ps, 16);
  W.l = W.l * al + ps;
  W.m = mn;
  // ---- every g's p of the 4 keys and alpha, to every lane
  float pk[G][4], ag[G];
  if constexpr (G <= 2) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) pk[g][k2] = __shfl_sync(0xffffffffu, p, 8 * k2 + g * C::GL);
      ag[g] = __shfl_sync(0xffffffffu, al, g * C::GL);
    }
  } else {
    __syncwarp();  // the previous tile's reads of sp are done
    if (c % C::GL == 0) {
      sp[(c / C::GL) * 4 + kk] = p;
      if (kk == 0) sp[G * 4 + c / C::GL] = al;
    }
    __syncwarp();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float4 t = *reinterpret_cast<const float4 *>(sp + g * 4);
      pk[g][0] = t.x, pk[g][1] = t.y, pk[g][2] = t.z, pk[g][3] = t.w;
      ag[g] = sp[G * 4 + g];
    }
  }
  // ---- o = o alpha + p V over the warp's valid keys
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int t = 0; t < C::DL; ++t) W.o[g][t] *= ag[g];
#pragma unroll
  for (int k2 = 0; k2 < 4; ++k2) {
    const int jj = 4 * w + k2;
    if (jj < nk) {
      float vf[C::DL];
      const __half *vr = vt + (int64_t)jj * D + lane * C::DL;
      if constexpr (C::DL == 4) {
        const uint2 *src = reinterpret_cast<const uint2 *>(vr);
        const uint2 raw = GLB ? __ldcg(src) : *src;
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
        vf[0] = a.x, vf[1] = a.y, vf[2] = b.x, vf[3] = b.y;
      } else {
        const unsigned *src = reinterpret_cast<const unsigned *>(vr);
        const unsigned raw = GLB ? __ldcg(src) : *src;
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw));
        vf[0] = a.x, vf[1] = a.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int t = 0; t < C::DL; ++t) W.o[g][t] = fmaf(pk[g][k2], vf[t], W.o[g][t]);
    }
  }
}

template <int D, int G>
using AttnCfg = typename std::conditional<kMmaAttn<G>, AttnCfgM<D, G>, AttnCfgS<D, G>>::type;

}  // namespace

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
// TP: the tensor-parallel instance (O / DOWN partial sums exchanged over NVLink, COMB phases, the
// greedy pick across vocabulary shards); the single-GPU instance carries none of that code.
template <int D, int G, bool TP>
__global__ void __launch_bounds__(kStepThreads, 1) k_decode_step(const __grid_constant__ StepArgs A) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);  // swizzled boxes: 1 KB
  __shared__ __align__(8) uint64_t full[kStepGroups][kStepStages], empty[kStepGroups][kStepStages];
  __shared__ float s_sum[(kStepConsumers / 32)];
  __shared__ int s_last[kStepGroups];
  __shared__ int s_abort;
  __shared__ unsigned long long s_key[kStepConsumers / 32];
  __shared__ float s_rope[128];  // cos / sin of every RoPE frequency at this step's position (head_dim <= 128)
  // descriptors of layer l in slot l & 1: copied ahead of the barrier before the layer's first phase, so the
  // phase starts without a global-memory round trip
  __shared__ __align__(16) StepLayer s_layer[2];
  static_assert(sizeof(StepLayer) % 16 == 0 && sizeof(StepLayer) / 16 <= kStepConsumers, "layer copy");

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int per = 5;  // QKV, ATTN, O, GATEUP, DOWN (tensor parallelism folds its exchanges into staging)
  const int L = A.L, nphase = per * L + 3;
  const int P = kStepGroups * gridDim.x;
  unsigned char *rings = base;                                            // [2][stages][18 KB]
  unsigned char *xarea = base + kStepGroups * kStepStages * kQ4TileBytes;  // staged x / attention scratch
  float *reds = reinterpret_cast<float *>(xarea + A.xarea_bytes);         // [2 groups][2 buffers][128]
  const int npos = A.pos[0];                                              // keys already in the cache
  const unsigned long long epoch = *reinterpret_cast<volatile unsigned long long *>(A.bar + 1);
  // arrivals every head's attention counter received in earlier launches (each launch adds L S)
  const unsigned long long abase = *reinterpret_cast<volatile unsigned long long *>(A.bar + 2);
  // exchange sequence base of this launch (2 L exchanges per launch; tensor parallelism only)
  const unsigned long long xbase = TP ? *reinterpret_cast<volatile unsigned long long *>(A.xep) : 0ull;

  if (tid == 0) {
    for (int g = 0; g < kStepGroups; ++g)
      for (int s = 0; s < kStepStages; ++s) {
        mbar_init(&full[g][s], 1);
        mbar_init(&empty[g][s], kGroupWarps);
      }
    s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // =========================== producers ===========================
  if (tid >= kStepConsumers) {
    const int grp = (tid - kStepConsumers) >> 5;
    if (lane != 0) return;
    const int vk = work_index<TP>(grp);
    unsigned char *ring = rings + grp * kStepStages * kQ4TileBytes;
    uint64_t *fl = full[grp], *em = empty[grp];
    const uint64_t pol = l2_evict_first_policy();
    StepCursor<D, G> ld;
    ld.init(A, vk, P, npos);
    const void *a, *b;
    uint32_t ba, bb;
    const CUtensorMap *kmap, *vmap;
    int y = 0, z = 0;
    int i = 0;
    while (ld.next(a, ba, b, bb, kmap, vmap, y, z)) {
      const int st = i % kStepStages;
      if (i >= kStepStages && !mbar_wait(&em[st], (uint32_t)(i / kStepStages - 1) & 1, A.err, DEVERR_GEMV_EMPTY))
        break;
      unsigned char *slot = ring + st * kQ4TileBytes;
      mbar_arrive_expect_tx(&fl[st], ba + bb);
      if (!kmap) {
        bulk_g2s(slot, a, ba, &fl[st], pol);
        if (bb) bulk_g2s(slot + kKeysPerTile * D * 2, b, bb, &fl[st], pol);
      } else {
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx) {
          tma_load_3d(slot + bx * kBoxBytes, kmap, 64 * bx, y, z, &fl[st], pol);
          tma_load_3d(slot + (D / 64 + bx) * kBoxBytes, vmap, 64 * bx, y, z, &fl[st], pol);
        }
      }
      ++i;
    }
    drain_ring<kStepStages>(fl, i, A.err);
    return;
  }

  // =========================== consumers ===========================
  // the QKV epilogues' RoPE factors, once per launch (the first QKV phase follows at least one barrier)
  for (int f = tid; f < A.d / 2; f += kStepConsumers) {
    float sn, cs;
    sincosf(rope_theta(A.inv_freq[f], npos), &sn, &cs);
    s_rope[f] = cs;
    s_rope[A.d / 2 + f] = sn;
  }
  if (tid < (int)(sizeof(StepLayer) / 16))
    reinterpret_cast<uint4 *>(&s_layer[0])[tid] = reinterpret_cast<const uint4 *>(A.layers)[tid];
  const int grp = warp / kGroupWarps, gw = warp % kGroupWarps, gtid = tid % kGroupThreads;
  const int vk = work_index<TP>(grp);
  const int gbar = 1 + grp;
  unsigned char *ring = rings + grp * kStepStages * kQ4TileBytes;
  uint64_t *fl = full[grp], *em = empty[grp];
  float *red = reds + grp * 2 * kGroupWarps * kQ4StripRows;
  int i = 0;  // ring stages consumed

  for (int p = 0; p < nphase; ++p) {
    const Phase ph = phase_kind(p, L, per);
    const int l = (p - 1) / per;
    bool ok = true;
    if (ph == PH_EMBED) {
      const int id = A.ids[0];
      const bool valid = id >= 0 && id < A.vocab;
      for (int j = blockIdx.x * kStepConsumers + tid; j < A.H; j += gridDim.x * kStepConsumers)
        A.h[j] = valid ? __half2float(A.embed[(int64_t)id * A.H + j]) : 0.0f;
    } else if (ph == PH_ATTN) {
      using Cf = AttnCfg<D, G>;
      const AttnSplit sp = attn_split(npos, A.Hkv, P);
      float *sm = reinterpret_cast<float *>(xarea) + grp * Cf::SM_END;
      if (vk < sp.units) {
        const int hk = vk / sp.S, s = vk % sp.S;
        const int t0 = s * sp.nt / sp.S, t1 = (s + 1) * sp.nt / sp.S;
        const bool last = s == sp.S - 1;
        if constexpr (kMmaAttn<G>) {
          // q fragments (the B operand of the scores): lane L of chunk ch holds the fp16 (hi, lo) pairs of
          // q[g = L / 4] at dims ch 16 + 2 (L % 4) (+ 1) and + 8, times the softmax scale; rows g >= G are zero
          uint4 *qf = reinterpret_cast<uint4 *>(sm + Cf::SM_QF);
          for (int e = gtid; e < Cf::NCH * 32; e += kGroupThreads) {
            const int ch = e >> 5, ln = e & 31, g = ln >> 2, k0 = ch * 16 + 2 * (ln & 3);
            uint4 f = make_uint4(0u, 0u, 0u, 0u);
            if (g < G) {
              const float *qg = A.q + (int64_t)(hk * G + g) * D;
              const float2 a = __ldcg(reinterpret_cast<const float2 *>(qg + k0));
              const float2 b = __ldcg(reinterpret_cast<const float2 *>(qg + k0 + 8));
              const float q0 = a.x * A.scale, q1 = a.y * A.scale, q2 = b.x * A.scale, q3 = b.y * A.scale;
              f.x = pack_h2(q0, q1);
              f.y = pack_h2(q2, q3);
              const float2 h0 = __half22float2(*reinterpret_cast<const __half2 *>(&f.x));
              const float2 h1 = __half22float2(*reinterpret_cast<const __half2 *>(&f.y));
              f.z = pack_h2(q0 - h0.x, q1 - h0.y);
              f.w = pack_h2(q2 - h1.x, q3 - h1.y);
            }
            qf[e] = f;
          }
          const uint32_t kv1 = smem_u32(sm + Cf::SM_KV);  // the one-key tile: K boxes, then V boxes, 16 rows each
          if (last && gtid < D / 4) {  // key npos (written by this launch's QKV phase) into row 0 (unswizzled)
            const int64_t row = ((int64_t)hk * A.cap + npos) * D;
            const int kv = gtid / (D / 8), cc = gtid % (D / 8);
            const __half *src = (kv == 0 ? s_layer[l & 1].k : s_layer[l & 1].v) + row + cc * 8;
            const uint32_t dst = swz_chunk(kv1 + kv * Cf::NB * (kBoxBytes / 2), kBoxBytes / 2, 0, cc);
            const uint4 val = __ldcg(reinterpret_cast<const uint4 *>(src));
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(val.x), "r"(val.y), "r"(val.z),
                         "r"(val.w)
                         : "memory");
          }
          named_sync_id(gbar, kGroupThreads);
          WarpAttnM<D, G> W;
          attn_warp_init_m<D, G>(W);
          for (int t = t0; t < t1; ++t, ++i) {
            const int sl = i % kStepStages;
            ok = ok && mbar_wait(&fl[sl], (uint32_t)(i / kStepStages) & 1, A.err, DEVERR_GEMV_FULL);
            if (ok) {
              const uint32_t kt = smem_u32(ring + sl * kQ4TileBytes);
              attn_mma_tile<D, G>(kt, kt + Cf::NB * kBoxBytes, kBoxBytes, min(kKeysPerTile, npos - t * kKeysPerTile),
                                  qf, W, gw, lane);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&em[sl]);
          }
          if (last && (gw & 1) == 0 && ok)  // key npos: the one-key tile, on the key-block-0 warps
            attn_mma_tile<D, G>(kv1, kv1 + Cf::NB * (kBoxBytes / 2), kBoxBytes / 2, 1, qf, W, gw, lane);
          // ---- merge the two key blocks' states into the unit's (m, l, o)
          float *wml = sm + Cf::SM_ML, *wo = sm + Cf::SM_O;
          {
            float lt[2] = {W.l[0], W.l[1]};
  #pragma unroll
            for (int o = 4; o < 32; o <<= 1)
  #pragma unroll
              for (int j = 0; j < 2; ++j) lt[j] += __shfl_xor_sync(0xffffffffu, lt[j], o);
            const int g0 = 2 * (lane & 3);
            if (lane < 4) {
              wml[(gw * 8 + g0) * 2] = W.m[0];
              wml[(gw * 8 + g0) * 2 + 1] = lt[0];
              wml[(gw * 8 + g0 + 1) * 2] = W.m[1];
              wml[(gw * 8 + g0 + 1) * 2 + 1] = lt[1];
            }
            const int kb = gw & 1, dset = gw >> 1;
  #pragma unroll
            for (int c = 0; c < Cf::NPC; ++c) {
              const int d0 = (dset * Cf::NPC + c) * 16 + (lane >> 2);
  #pragma unroll
              for (int j = 0; j < 2; ++j)
                if (g0 + j < G) {
                  wo[(kb * G + g0 + j) * D + d0] = W.o[c][j];
                  wo[(kb * G + g0 + j) * D + d0 + 8] = W.o[c][2 + j];
                }
            }
          }
          named_sync_id(gbar, kGroupThreads);
          float *part = A.attn_part + ((int64_t)hk * sp.S + s) * G * (D + 2);
          for (int e = gtid; e < G * D; e += kGroupThreads) {
            const int g = e / D, c = e % D, w0 = 2 * (c / (D / 4));
            const float m0 = wml[(w0 * 8 + g) * 2], l0 = wml[(w0 * 8 + g) * 2 + 1];
            const float m1 = wml[((w0 + 1) * 8 + g) * 2], l1 = wml[((w0 + 1) * 8 + g) * 2 + 1];
            const float M = fmaxf(m0, m1);
            const float f0 = m0 == -INFINITY ? 0.0f : expf(m0 - M), f1 = m1 == -INFINITY ? 0.0f : expf(m1 - M);
            const float Ls = fmaf(l1, f1, l0 * f0);
            const float O = fmaf(wo[(G + g) * D + c], f1, wo[g * D + c] * f0);
            if (sp.S == 1) {
              A.att[(int64_t)(hk * G + g) * D + c] = O / fmaxf(Ls, 1e-12f);
            } else {
              part[g * (D + 2) + 2 + c] = O;
              if (c == 0) {
                part[g * (D + 2)] = M;
                part[g * (D + 2) + 1] = Ls;
              }
            }
          }
        } else {
          for (int e = gtid; e < G * D; e += kGroupThreads)
            sm[Cf::SM_Q + (e / D) * D + q_swz(e % D)] = __ldcg(A.q + (int64_t)hk * G * D + e) * A.scale;
          if (last && gtid < D / 4) {  // key npos (written by this launch's QKV phase): K then V row, 16 B each
            const int64_t row = ((int64_t)hk * A.cap + npos) * D;
            const __half *src = (gtid < D / 8 ? s_layer[l & 1].k : s_layer[l & 1].v) + row + (gtid % (D / 8)) * 8;
            reinterpret_cast<uint4 *>(sm + Cf::SM_KV)[gtid] = __ldcg(reinterpret_cast<const uint4 *>(src));
          }
          named_sync_id(gbar, kGroupThreads);
          WarpAttnS<D, G> W;
          attn_warp_init_s<D, G>(W, sm + Cf::SM_Q, lane);
          float *wp = sm + Cf::SM_P + gw * G * 5;
          for (int t = t0; t < t1; ++t, ++i) {
            const int sl = i % kStepStages;
            ok = ok && mbar_wait(&fl[sl], (uint32_t)(i / kStepStages) & 1, A.err, DEVERR_GEMV_FULL);
            if (ok) {
              const __half *kt = reinterpret_cast<const __half *>(ring + sl * kQ4TileBytes);
              attn_warp_tile<D, G, false>(kt, kt + kKeysPerTile * D, min(kKeysPerTile, npos - t * kKeysPerTile),
                                          sm + Cf::SM_Q, wp, W, gw, lane);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&em[sl]);
          }
          if (last && gw == 0 && ok) {  // key npos: this step's K/V, staged with q
            const __half *kv = reinterpret_cast<const __half *>(sm + Cf::SM_KV);
            attn_warp_tile<D, G, false>(kv, kv + D, 1, sm + Cf::SM_Q, wp, W, 0, lane);
          }
          // ---- merge the eight warp states into the unit's (m, l, o)
          float *wml = sm + Cf::SM_ML, *wo = sm + Cf::SM_O;
          {
            const int c = lane & 7;
            if (lane < 8 && c % Cf::GL == 0) {
              wml[(gw * G + c / Cf::GL) * 2] = W.m;
              wml[(gw * G + c / Cf::GL) * 2 + 1] = W.l;
            }
  #pragma unroll
            for (int g = 0; g < G; ++g) {
              float *dst = wo + (gw * G + g) * D + lane * Cf::DL;
              if constexpr (Cf::DL == 4)
                *reinterpret_cast<float4 *>(dst) = make_float4(W.o[g][0], W.o[g][1], W.o[g][2], W.o[g][3]);
              else
                *reinterpret_cast<float2 *>(dst) = make_float2(W.o[g][0], W.o[g][1]);
            }
          }
          named_sync_id(gbar, kGroupThreads);
          float *part = A.attn_part + ((int64_t)hk * sp.S + s) * G * (D + 2);
          for (int e = gtid; e < G * D; e += kGroupThreads) {
            const int g = e / D, c = e % D;
            float M = -INFINITY;
  #pragma unroll
            for (int w = 0; w < kGroupWarps; ++w) M = fmaxf(M, wml[(w * G + g) * 2]);
            float Ls = 0.0f, O = 0.0f;
  #pragma unroll
            for (int w = 0; w < kGroupWarps; ++w) {
              const float mw = wml[(w * G + g) * 2];
              const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
              Ls = fmaf(wml[(w * G + g) * 2 + 1], f, Ls);
              O = fmaf(wo[(w * G + g) * D + c], f, O);
            }
            if (sp.S == 1) {
              A.att[(int64_t)(hk * G + g) * D + c] = O / fmaxf(Ls, 1e-12f);
            } else {
              part[g * (D + 2) + 2 + c] = O;
              if (c == 0) {
                part[g * (D + 2)] = M;
                part[g * (D + 2) + 1] = Ls;
              }
            }
          }
        }
        if (sp.S > 1) {
          // every split of the head publishes its partial (one release add on the head's counter, which
          // only grows: abase counts the arrivals of earlier launches), waits until all S have, and then
          // merges its own slice [s G D / S, (s + 1) G D / S) of the head's outputs -- one round of loads
          // instead of a lone last split walking all S partials
          named_sync_id(gbar, kGroupThreads);
          if (gtid == 0) {
            unsigned long long *cnt = A.attn_cnt + hk;
            asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(cnt) : "memory");
            s_last[grp] = wait_count(cnt, abase + (unsigned long long)(l + 1) * sp.S, A.err) ? 1 : 0;
          }
          named_sync_id(gbar, kGroupThreads);
          ok = ok && s_last[grp] != 0;
          const float *hp = A.attn_part + (int64_t)hk * sp.S * G * (D + 2);
          const int o0 = s * G * D / sp.S, o1 = (s + 1) * G * D / sp.S;
          // a team of TS lanes per output (TS a power of two <= 16, >= S when S <= 16)
          const int TS = sp.S > 8 ? 16 : (sp.S > 4 ? 8 : (sp.S > 2 ? 4 : 2));
          const int team = gtid / TS, tl = gtid % TS, nteams = kGroupThreads / TS;
          const int npass = (o1 - o0 + nteams - 1) / nteams;
          for (int pass = 0; pass < npass; ++pass) {
            const int o = o0 + pass * nteams + team;
            const bool valid = ok && o < o1;
            const int g = valid ? o / D : 0, c = valid ? o % D : 0;
            float m = -INFINITY, ls = 0.0f, os = 0.0f;
            if (valid) {
              for (int j = tl; j < sp.S; j += TS) {
                const float *pj = hp + (j * G + g) * (D + 2);
                const float mj = __ldcg(pj), lj = __ldcg(pj + 1), oj = __ldcg(pj + 2 + c);
                const float mn = fmaxf(m, mj);
                const float f0 = m == -INFINITY ? 0.0f : expf(m - mn), f1 = mj == -INFINITY ? 0.0f : expf(mj - mn);
                ls = ls * f0 + lj * f1;
                os = os * f0 + oj * f1;
                m = mn;
              }
            }
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1) {
              if (off < TS) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
                const float l2 = __shfl_xor_sync(0xffffffffu, ls, off);
                const float o2 = __shfl_xor_sync(0xffffffffu, os, off);
                const float mn = fmaxf(m, m2);
                const float f0 = m == -INFINITY ? 0.0f : expf(m - mn), f1 = m2 == -INFINITY ? 0.0f : expf(m2 - mn);
                ls = ls * f0 + l2 * f1;
                os = os * f0 + o2 * f1;
                m = mn;
              }
            }
            if (valid && tl == 0) A.att[(int64_t)(hk * G + g) * D + c] = os / fmaxf(ls, 1e-12f);
          }
        }
      }
    } else if (ph == PH_ARGMAX) {
      // slice of the logits -> one key per CTA -> atomicMax (global vocabulary index)
      unsigned long long best = 0;
      const int V = A.vocab_l;
      for (int j = blockIdx.x * kStepConsumers + tid; j < V; j += gridDim.x * kStepConsumers) {
        const float v = __ldcg(A.logits + j);
        const int jg = j + A.vbase;
        unsigned long long key;
        if (v != v) {
          key = jg == 0 ? ~0ull : 0ull;  // a NaN never wins, except at index 0 (the sampler keeps index 0)
        } else {
          uint32_t bits = __float_as_uint(v);
          bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
          key = ((unsigned long long)bits << 32) | (0xFFFFFFFFull - (unsigned long long)jg);
        }
        best = key > best ? key : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      if (lane == 0) s_key[warp] = best;
      named_sync_id(kBarConsumers, kStepConsumers);
      if (tid == 0) {
        unsigned long long b = 0;
        for (int w = 0; w < kStepConsumers / 32; ++w) b = s_key[w] > b ? s_key[w] : b;
        atomicMax(A.argkey, b);
      }
    } else {
      // ---------------- GEMV phase
      QMat w;
      const float *x, *gm;
      Epilogue ep;
      gemv_phase(A, ph, l, &s_layer[l & 1], w, x, gm, ep);
      if (ph == PH_QKV) {
        ep.rope_cs = s_rope;
        ep.pos0 = npos;
      }
      const Sched sc = make_sched(w.N, kQ4StripRows, 1, vk, P);  // units = 16-row strips
      const int nq = (int)w.row_words;
      Q4X<1> X;
      X.carve(xarea, (int)(w.K >> 5), nq * 4);
      if constexpr (TP) {
        const int fx = fold_index(p, L);
        if (fx >= 0) {
          // h(out) = h(in) + every rank's partial sums of exchange fx in rank order (the same on every rank,
          // so h stays bit-identical across ranks); h alternates between two buffers, one per exchange parity
          // every CTA of every rank has stored its partial sums of exchange fx (all ranks run the same grid size)
          if (tid == 0)
            s_last[0] = wait_xcnt(A, (xbase * (2 * L) + fx + 1) * (unsigned long long)A.tp * gridDim.x) ? 1 : 0;
          named_sync_id(kBarConsumers, kStepConsumers);
          ok = s_last[0] != 0;
          if (ok)
            q4_stage_x_fold(X, (fx & 1) ? A.h2 : A.h, A.xr[A.rank] + (int64_t)(fx & 1) * A.tp * A.H, A.tp, A.H,
                            (fx & 1) ? A.h : A.h2, (int)((int64_t)blockIdx.x * A.H / gridDim.x),
                            (int)((int64_t)(blockIdx.x + 1) * A.H / gridDim.x), gm, tid, kStepConsumers, s_sum);
        } else {
          q4_stage_x<1>(X, x, w.K, gm, tid, kStepConsumers, s_sum);
        }
      } else if (gm) {
        q4_stage_x<1>(X, x, w.K, gm, tid, kStepConsumers, s_sum);
      } else {  // no norm (O, DOWN): six items' loads in flight, one L2 round trip for K <= 12288
        q4_stage_x<1, 6>(X, x, w.K, nullptr, tid, kStepConsumers, s_sum);
      }
      named_sync_id(kBarConsumers, kStepConsumers);
      // every thread forms 1/rms from the warps' sums (s_sum is rewritten only after the phase's barrier)
      const float inv = rms_inv(s_sum, kStepConsumers / 32, 1, 0, w.K, A.eps, gm != nullptr);
      Q4Lane<1> Ln;
      Ln.init(X, lane);
      float2 acc[1] = {make_float2(0.0f, 0.0f)};
      for (int u = sc.u0; u < sc.u1; ++u) {
        for (int q0 = 0; q0 < nq; q0 += kQ4TileQuads, ++i) {
          const int sl = i % kStepStages;
          ok = ok && mbar_wait(&fl[sl], (uint32_t)(i / kStepStages) & 1, A.err, DEVERR_GEMV_FULL);
          if (ok) q4_tile<1>(ring + sl * kQ4TileBytes, q0, min(kQ4TileQuads, nq - q0), gw, Ln, acc);
          __syncwarp();
          if (lane == 0) mbar_arrive(&em[sl]);
        }
        // two partial buffers in turn: a warp refills this one two strips later, after the next
        // strip's barrier, which the finishing threads reach only once they have read it
        float *rb = red + ((u - sc.u0) & 1) * (kGroupWarps * kQ4StripRows);
        q4_group_red<1>(rb, acc, gw, lane);
        named_sync_id(gbar, kGroupThreads);
        if (ok) finish_strip<1, TP>(w, ep, u, rb, &inv, gtid, kGroupThreads);
      }
    }
    // ---------------- end of phase: grid barrier
    if (!ok) s_abort = 1;
    if (ph == PH_DOWN && l + 1 < L && tid < (int)(sizeof(StepLayer) / 16))  // the next layer's descriptors
      reinterpret_cast<uint4 *>(&s_layer[(l + 1) & 1])[tid] = reinterpret_cast<const uint4 *>(A.layers + l + 1)[tid];
    named_sync_id(kBarConsumers, kStepConsumers);
    const bool xphase = TP && (ph == PH_O || ph == PH_DOWN);
    const unsigned long long btarget = (epoch * (unsigned long long)nphase + p + 1) * gridDim.x;
    if (xphase) {
      // exchange phase: one arrival at every rank's exchange counter after one system-scope release fence,
      // which orders this CTA's partial sums (stored into every rank's region, before the CTA barrier above)
      // before the arrivals; the phase that folds the exchange waits on its counter, which implies every CTA
      // of this rank has finished too, so the grid barrier only takes the arrival (its count stays that of a
      // barrier per phase) and nobody waits on it.  One fence and relaxed adds: 561 tokens/s at TP 2 against
      // 499 with a release on every add and 514 with the barrier-then-flag exchange (same box)
      if (tid == 0 && !s_abort) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int r = 0; r < A.tp; ++r)
          asm volatile("red.relaxed.sys.global.add.u64 [%0], 1;" ::"l"(xflag_words(A, r) + kXcnt) : "memory");
        asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;" ::"l"(A.bar) : "memory");
      }
    } else if (tid == 0 && !s_abort && !grid_sync(A.bar, btarget, A.err)) {
      s_abort = 1;
    }
    named_sync_id(kBarConsumers, kStepConsumers);
    if (s_abort) return;
  }
  // ---------------- the token: CTA 0, after the ARGMAX barrier
  if (blockIdx.x == 0 && tid == 0) {
    unsigned long long key = *reinterpret_cast<volatile unsigned long long *>(A.argkey);
    if constexpr (TP) {  // the greedy pick over every rank's vocabulary shard
      if (!exchange_keys(A, xbase + 1, key)) return;
      *A.xep = xbase + 1;
    }
    const int32_t id = (int32_t)(0xFFFFFFFFull - (key & 0xFFFFFFFFull));
    A.ids[0] = id;
    const int st = *A.step;
    if (A.token_log && st < A.log_steps) A.token_log[st] = id;
    *A.step = st + 1;
    A.pos[0] = npos + 1;
    *A.argkey = 0ull;
    const AttnSplit sp = attn_split(npos, A.Hkv, 2 * gridDim.x);
    A.bar[2] = abase + (sp.S > 1 ? (unsigned long long)L * sp.S : 0ull);  // this launch's counter arrivals
    A.bar[1] = epoch + 1;  // every CTA has passed every barrier of this launch
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {
template <int D, int G>
size_t step_attn_floats() {
  return (size_t)kStepGroups * AttnCfg<D, G>::SM_END;
}
template <int D, int G>
const void *step_kernel(bool tp) {
  return tp ? (const void *)k_decode_step<D, G, true> : (const void *)k_decode_step<D, G, false>;
}
const void *pick_kernel(int D, int G, bool tp) {
  if (D == 128) {
    switch (G) {
      case 1: return step_kernel<128, 1>(tp);
      case 2: return step_kernel<128, 2>(tp);
      case 4: return step_kernel<128, 4>(tp);
      case 8: return step_kernel<128, 8>(tp);
    }
  } else if (D == 64) {
    switch (G) {
      case 1: return step_kernel<64, 1>(tp);
      case 2: return step_kernel<64, 2>(tp);
      case 4: return step_kernel<64, 4>(tp);
      case 8: return step_kernel<64, 8>(tp);
    }
  }
  return nullptr;
}
size_t attn_floats(int D, int G) {
  if (D == 128) {
    switch (G) {
      case 1: return step_attn_floats<128, 1>();
      case 2: return step_attn_floats<128, 2>();
      case 4: return step_attn_floats<128, 4>();
      default: return step_attn_floats<128, 8>();
    }
  }
  switch (G) {
    case 1: return step_attn_floats<64, 1>();
    case 2: return step_attn_floats<64, 2>();
    case 4: return step_attn_floats<64, 4>();
    default: return step_attn_floats<64, 8>();
  }
}
}  // namespace

bool decode_step_supported(int d, int G, int qtype, int64_t H, int64_t I, int64_t qdim) {
  if (qtype != FG_Q4_0 || !pick_kernel(d, G, false)) return false;
  const size_t smem = decode_step_smem(d, G, H, I, qdim);
  return smem <= 220 * 1024;  // 227 KB per block, less the kernel's static shared memory
}

size_t decode_step_xarea(int d, int G, int64_t H, int64_t I, int64_t qdim) {
  int64_t kmax = std::max(H, std::max(I, qdim));
  const int nbx = (int)q4_quads(kmax) * 4;
  const size_t xb = align_up(Q4X<1>::bytes(nbx), 16);
  const size_t ab = align_up(attn_floats(d, G) * 4, 16);
  return std::max(xb, ab);
}

size_t decode_step_smem(int d, int G, int64_t H, int64_t I, int64_t qdim) {
  return 1024 + (size_t)kStepGroups * kStepStages * kQ4TileBytes + decode_step_xarea(d, G, H, I, qdim) +
         (size_t)kStepGroups * 2 * kGroupWarps * kQ4StripRows * 4;
}

int decode_step_vctas(int num_sms) { return kStepGroups * num_sms; }

void launch_decode_step(const StepArgs &A, int num_sms, cudaStream_t s) {
  const void *kern = pick_kernel(A.d, A.Hq / A.Hkv, A.tp > 1);
  FG_REQUIRE(kern, FG_ERR_SHAPE, "decode step: head_dim %d / GQA group %d unsupported", A.d, A.Hq / A.Hkv);
  const size_t smem = decode_step_smem(A.d, A.Hq / A.Hkv, A.H, A.I, (int64_t)A.Hq * A.d);
  FG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)num_sms);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barriers rely on it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void *args[] = {const_cast<StepArgs *>(&A)};
  FG_CUDA(cudaLaunchKernelExC(&cfg, kern, args));
}

}  // namespace fg
