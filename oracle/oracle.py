"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for the forge_b200 parity tests.

Python face of ``oracle/forge_oracle.c`` (built by ``oracle/Makefile``) plus
a numpy restatement of the reference Llama forward
(packages/forge-py/src/forge/models/llama.py:45-248) built on those C
primitives.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module; the product (``ameva-forge_b200/``) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libforge_oracle.so")
_lib = None

Q4_0 = 4
Q8_0 = 8
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34}

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64 = ctypes.c_int64


def build() -> str:
    """Compile the C oracle (idempotent)."""
    src = os.path.join(_HERE, "forge_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        L.fo_splitmix64.restype = ctypes.c_uint64
        L.fo_splitmix64.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.fo_normal.restype = ctypes.c_float
        L.fo_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        L.fo_fill_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, _i64, ctypes.c_float, ctypes.c_float, _f32p]
        L.fo_f32_to_f16.restype = ctypes.c_uint16
        L.fo_f32_to_f16.argtypes = [ctypes.c_float]
        L.fo_f32_to_f16_array.argtypes = [_f32p, _i64, _u16p]
        L.fo_f16_to_f32_array.argtypes = [_u16p, _i64, _f32p]
        L.fo_quantize_q4_0.argtypes = [_f32p, _i64, _u8p]
        L.fo_quantize_q8_0.argtypes = [_f32p, _i64, _u8p]
        L.fo_gguf_to_ref.argtypes = [ctypes.c_int, _u8p, _i64, _u32p, _f32p, _f32p]
        L.fo_unpack_quant.argtypes = [_u32p, _f32p, _f32p, ctypes.c_int, _i64, _i64, _f32p]
        L.fo_dequant.argtypes = [ctypes.c_int, _u8p, _i64, _f32p]
        L.fo_qmatmul.argtypes = [ctypes.c_int, _u8p, _i64, _i64, _f32p, _i64, _f32p]
        L.fo_dequant_q4k.argtypes = [_u8p, _i64, _f32p]
        L.fo_qmatmul_q4k.argtypes = [_u8p, _i64, _i64, _f32p, _i64, _f32p]
        L.fo_dequant_q6k.argtypes = [_u8p, _i64, _f32p]
        L.fo_qmatmul_q6k.argtypes = [_u8p, _i64, _i64, _f32p, _i64, _f32p]
        L.fo_matmul.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p]
        L.fo_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                   ctypes.c_float, ctypes.c_int]
        L.fo_rmsnorm.argtypes = [_f32p, _f32p, _i64, _i64, ctypes.c_float, _f32p]
        L.fo_rope_inv_freq.argtypes = [ctypes.c_float, _i64, _f32p]
        L.fo_rope.argtypes = [_f32p, _i64, _i64, _i64, ctypes.c_float, _i64, _f32p]
        L.fo_swiglu.argtypes = [_f32p, _f32p, _i64, _f32p]
        L.fo_embedding.argtypes = [_f32p, _i64, _i64, _i32p, _i64, _f32p]
        L.fo_argmax.restype = ctypes.c_int64
        L.fo_argmax.argtypes = [_f32p, _i64]
        L.fo_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


# ----------------------------------------------------------------- generator
def splitmix64(seed: int, i: int) -> int:
    return int(lib().fo_splitmix64(seed & (2**64 - 1), i & (2**64 - 1)))


def normal(seed: int, offset: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().fo_fill_normal(seed & (2**64 - 1), offset, n, mean, std, _p(out, _f32p))
    return out


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().fo_f32_to_f16_array(_p(x.reshape(-1), _f32p), x.size, _p(out.reshape(-1), _u16p))
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().fo_f16_to_f32_array(_p(h.reshape(-1), _u16p), h.size, _p(out.reshape(-1), _f32p))
    return out


def round_f16(x: np.ndarray) -> np.ndarray:
    return f16_to_f32(f32_to_f16(x))


# ----------------------------------------------------------------- quant
def quantize(qtype: int, w: np.ndarray) -> np.ndarray:
    """fp32 [rows, cols] -> GGUF blocks uint8 [rows, cols/32*block_bytes]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    assert cols % 32 == 0
    nb = rows * cols // 32
    out = np.empty((rows, cols // 32 * BLOCK_BYTES[qtype]), dtype=np.uint8)
    fn = lib().fo_quantize_q4_0 if qtype == Q4_0 else lib().fo_quantize_q8_0
    fn(_p(w, _f32p), nb, _p(out, _u8p))
    return out


def gguf_to_ref(qtype: int, blocks: np.ndarray):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    nb = blocks.size // BLOCK_BYTES[qtype]
    words = nb * (4 if qtype == Q4_0 else 8)
    packed = np.empty(words, dtype=np.uint32)
    scales = np.empty(nb, dtype=np.float32)
    zeros = np.empty(nb, dtype=np.float32)
    lib().fo_gguf_to_ref(qtype, _p(blocks.reshape(-1), _u8p), nb, _p(packed, _u32p), _p(scales, _f32p),
                         _p(zeros, _f32p))
    return packed, scales, zeros


def unpack_quant(packed, scales, zeros, bits: int, group_size: int, n: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    zeros = np.ascontiguousarray(zeros, dtype=np.float32)
    out = np.empty(n, dtype=np.float32)
    lib().fo_unpack_quant(_p(packed, _u32p), _p(scales, _f32p), _p(zeros, _f32p), bits, group_size, n,
                          _p(out, _f32p))
    return out


def dequant(qtype: int, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty((rows, cols), dtype=np.float32)
    lib().fo_dequant(qtype, _p(blocks.reshape(-1), _u8p), rows * cols // 32, _p(out, _f32p))
    return out


def dequant_q4k(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """GGUF Q4_K super-blocks [rows, cols / 256 * 144] -> fp32 [rows, cols] (forge_oracle.c)."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty((rows, cols), dtype=np.float32)
    lib().fo_dequant_q4k(_p(blocks.reshape(-1), _u8p), rows * cols // 256, _p(out, _f32p))
    return out


def qmatmul_q4k(blocks: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.size // K
    y = np.empty((M, N), dtype=np.float32)
    lib().fo_qmatmul_q4k(_p(np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1), _u8p), N, K,
                         _p(x.reshape(-1), _f32p), M, _p(y, _f32p))
    return y.reshape(x.shape[:-1] + (N,))


def random_q4k(rows: int, cols: int, seed: int, d_scale: float = 1e-3) -> np.ndarray:
    """Random valid Q4_K blocks: finite positive fp16 d / dmin, random 6-bit packs and nibbles."""
    rng = np.random.default_rng(seed)
    nb = rows * cols // 256
    b = rng.integers(0, 256, size=(nb, 144), dtype=np.uint8)
    d = (rng.random(nb) * d_scale + d_scale / 8).astype(np.float16).view(np.uint16)
    dm = (rng.random(nb) * d_scale + d_scale / 8).astype(np.float16).view(np.uint16)
    b[:, 0], b[:, 1] = d & 0xFF, d >> 8
    b[:, 2], b[:, 3] = dm & 0xFF, dm >> 8
    return b.reshape(rows, cols // 256 * 144)


def dequant_q6k(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """GGUF Q6_K super-blocks [rows, cols / 256 * 210] -> fp32 [rows, cols] (forge_oracle.c)."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty((rows, cols), dtype=np.float32)
    lib().fo_dequant_q6k(_p(blocks.reshape(-1), _u8p), rows * cols // 256, _p(out, _f32p))
    return out


def qmatmul_q6k(blocks: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.size // K
    y = np.empty((M, N), dtype=np.float32)
    lib().fo_qmatmul_q6k(_p(np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1), _u8p), N, K,
                         _p(x.reshape(-1), _f32p), M, _p(y, _f32p))
    return y.reshape(x.shape[:-1] + (N,))


def random_q6k(rows: int, cols: int, seed: int, d_scale: float = 1e-3) -> np.ndarray:
    """Random valid Q6_K blocks: random ql / qh / int8 scales, finite positive fp16 d."""
    rng = np.random.default_rng(seed)
    nb = rows * cols // 256
    b = rng.integers(0, 256, size=(nb, 210), dtype=np.uint8)
    d = (rng.random(nb) * d_scale + d_scale / 8).astype(np.float16).view(np.uint16)
    b[:, 208], b[:, 209] = d & 0xFF, d >> 8
    return b.reshape(rows, cols // 256 * 210)


def qmatmul(qtype: int, blocks: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    M = x.size // K
    y = np.empty((M, N), dtype=np.float32)
    lib().fo_qmatmul(qtype, _p(np.ascontiguousarray(blocks).reshape(-1), _u8p), N, K, _p(x.reshape(-1), _f32p),
                     M, _p(y, _f32p))
    return y.reshape(x.shape[:-1] + (N,))


def matmul(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    C = np.empty((M, N), dtype=np.float32)
    lib().fo_matmul(_p(A, _f32p), _p(B, _f32p), M, K, N, _p(C, _f32p))
    return C


def attention(Q, K, V, scale=None, causal=False, n_kv=None):
    """Q [B,H,Nq,d]; K/V [B,Hkv,S,d] with the first n_kv rows live."""
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    B, H, Nq, d = Q.shape
    Hkv, S = K.shape[1], K.shape[2]
    n_kv = S if n_kv is None else n_kv
    if scale is None:
        scale = 1.0 / np.sqrt(d)
    O = np.empty_like(Q)
    lib().fo_attention(_p(Q, _f32p), _p(K, _f32p), _p(V, _f32p), _p(O, _f32p), B, H, Hkv, Nq, n_kv, d, S * d,
                       float(scale), 1 if causal else 0)
    return O


def rmsnorm(x, gamma=None, eps=1e-5):
    x = np.ascontiguousarray(x, dtype=np.float32)
    dim = x.shape[-1]
    out = np.empty_like(x)
    g = None if gamma is None else _p(np.ascontiguousarray(gamma, dtype=np.float32), _f32p)
    lib().fo_rmsnorm(_p(x, _f32p), g, x.size // dim, dim, eps, _p(out, _f32p))
    return out


def rope_inv_freq(base: float, d: int) -> np.ndarray:
    out = np.empty(d // 2, dtype=np.float32)
    lib().fo_rope_inv_freq(base, d, _p(out, _f32p))
    return out


def rope(x, base=10000.0, offset=0):
    """x [..., N, d] (rows = product of leading dims)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    N, d = x.shape[-2], x.shape[-1]
    out = np.empty_like(x)
    lib().fo_rope(_p(x, _f32p), x.size // (N * d), N, d, base, offset, _p(out, _f32p))
    return out


def swiglu(gate, up):
    gate = np.ascontiguousarray(gate, dtype=np.float32)
    up = np.ascontiguousarray(up, dtype=np.float32)
    out = np.empty_like(gate)
    lib().fo_swiglu(_p(gate, _f32p), _p(up, _f32p), gate.size, _p(out, _f32p))
    return out


def embedding(table, ids):
    table = np.ascontiguousarray(table, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    vocab, dim = table.shape
    out = np.empty(ids.shape + (dim,), dtype=np.float32)
    lib().fo_embedding(_p(table, _f32p), vocab, dim, _p(ids.reshape(-1), _i32p), ids.size, _p(out, _f32p))
    return out


def argmax(logits) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().fo_argmax(_p(logits, _f32p), logits.size))


def xorshift32_first(seed: int) -> float:
    """The first output of the reference's Xorshift32 generator / 2^32
    (packages/forge/src/tensor/sampling.ts:20-28: s = (seed >>> 0) || 1)."""
    x = (int(seed) & 0xFFFFFFFF) or 1
    x ^= (x << 13) & 0xFFFFFFFF
    x ^= x >> 17
    x ^= (x << 5) & 0xFFFFFFFF
    return x / 4294967296.0


def sample(logits, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0, seed: int = 0) -> int:
    """LLMSampler.sample with a seed (packages/forge/src/tensor/sampling.ts:35-128),
    statement by statement: greedy below temperature 1e-5 (:45-55); the
    partial selection sort with swaps for k <= 128 (:62-76), else a stable
    descending sort (:78-80); double-precision softmax stored as float32
    (:82-96); top-p prefix (:98-109); categorical pick on the first
    Xorshift32 draw (:111-127).  Pure Python: small vocabularies only."""
    import math
    lg = np.asarray(logits, dtype=np.float32).reshape(-1)
    V = lg.size
    if V == 0:
        raise ValueError("Logits array cannot be empty")
    if temperature <= 1e-5:
        best, bv = 0, lg[0]
        for i in range(1, V):
            if lg[i] > bv:
                bv, best = lg[i], i
        return best
    K = top_k if 0 < top_k < V else V
    idx = list(range(V))
    if K < V and K <= 128:
        for i in range(K):
            mp, mv = i, lg[idx[i]]
            for j in range(i + 1, V):
                if lg[idx[j]] > mv:
                    mv, mp = lg[idx[j]], j
            idx[i], idx[mp] = idx[mp], idx[i]
    else:
        idx.sort(key=lambda a: -float(lg[a]))  # stable, as Array.prototype.sort
    mx = float(lg[idx[0]]) / temperature
    cand = np.empty(K, np.float32)
    tot = 0.0
    for i in range(K):
        p = math.exp(float(lg[idx[i]]) / temperature - mx)
        cand[i] = p
        tot += p
    inv = 1.0 / max(tot, 1e-12)
    for i in range(K):
        cand[i] = float(cand[i]) * inv
    cutoff = K
    if top_p < 1.0:
        cs = 0.0
        for i in range(K):
            cs += float(cand[i])
            if cs >= top_p:
                cutoff = i + 1
                break
    fs = 0.0
    for i in range(cutoff):
        fs += float(cand[i])
    invf = 1.0 / max(fs, 1e-12)
    r = xorshift32_first(seed)
    acc = 0.0
    for i in range(cutoff):
        acc += float(cand[i]) * invf
        if r <= acc:
            return idx[i]
    return idx[cutoff - 1]


def num_threads() -> int:
    return int(lib().fo_num_threads())


# ----------------------------------------------------------------- Llama
# Tensor ids of the synthetic weight recipe: seed = splitmix64(model_seed,
# layer * 16 + tid); value (r, c) of an [N, K] matrix = std * normal(seed, r*K + c).
TID = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6, "attn_norm": 7, "ffn_norm": 8}
GLOBAL_LAYER = 0xFFFF
GID = {"embed": 0, "norm": 1, "lm_head": 2}


@dataclass
class LlamaShape:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0

    @property
    def head_dim(self):
        return self.hidden_size // self.num_attention_heads


def tensor_seed(model_seed: int, layer: int, tid: int) -> int:
    return splitmix64(model_seed, layer * 16 + tid)


def synth_matrix(model_seed, layer, tid, rows, cols, std=0.02, row0=0, nrows=None):
    nrows = rows if nrows is None else nrows
    s = tensor_seed(model_seed, layer, tid)
    return normal(s, row0 * cols, nrows * cols, 0.0, std).reshape(nrows, cols)


@dataclass
class LlamaWeights:
    """Host copy of a synthetic model: GGUF Q4_0 blocks for every Linear
    (incl. lm_head), fp16 embedding table, fp32 norm gains."""
    shape: LlamaShape
    qtype: int
    embed_f16: np.ndarray
    norm: np.ndarray
    lm_head: np.ndarray
    layers: list = field(default_factory=list)


def synth_llama(shape: LlamaShape, seed: int, qtype: int = Q4_0, std: float = 0.02) -> LlamaWeights:
    H, I, V = shape.hidden_size, shape.intermediate_size, shape.vocab_size
    d = shape.head_dim
    kvd = shape.num_key_value_heads * d
    emb = f32_to_f16(synth_matrix(seed, GLOBAL_LAYER, GID["embed"], V, H, std))
    norm = normal(tensor_seed(seed, GLOBAL_LAYER, GID["norm"]), 0, H, 1.0, 0.1)
    lm = quantize(qtype, synth_matrix(seed, GLOBAL_LAYER, GID["lm_head"], V, H, std))
    w = LlamaWeights(shape, qtype, emb, norm, lm)
    dims = {"q": (H, H), "k": (kvd, H), "v": (kvd, H), "o": (H, H), "gate": (I, H), "up": (I, H), "down": (H, I)}
    for l in range(shape.num_hidden_layers):
        L = {}
        for name, (r, c) in dims.items():
            L[name] = quantize(qtype, synth_matrix(seed, l, TID[name], r, c, std))
        L["attn_norm"] = normal(tensor_seed(seed, l, TID["attn_norm"]), 0, H, 1.0, 0.1)
        L["ffn_norm"] = normal(tensor_seed(seed, l, TID["ffn_norm"]), 0, H, 1.0, 0.1)
        w.layers.append(L)
    return w


# A k-quant model in the type mix of a llama.cpp Q4_K_M file: Q6_K for attn_v, ffn_down and the output
# matrix, Q4_K for the other Linears.  Each Linear is (type name, GGUF blocks); embedding and norms follow
# synth_llama's recipe.
KQ_MIX = {"q": "Q4_K", "k": "Q4_K", "v": "Q6_K", "o": "Q4_K", "gate": "Q4_K", "up": "Q4_K", "down": "Q6_K"}


def kquant_llama(shape: LlamaShape, seed: int, d_scale: float = 1e-4) -> LlamaWeights:
    H, I, V = shape.hidden_size, shape.intermediate_size, shape.vocab_size
    kvd = shape.num_key_value_heads * shape.head_dim
    emb = f32_to_f16(synth_matrix(seed, GLOBAL_LAYER, GID["embed"], V, H, 0.02))
    norm = normal(tensor_seed(seed, GLOBAL_LAYER, GID["norm"]), 0, H, 1.0, 0.1)
    rnd = {"Q4_K": random_q4k, "Q6_K": random_q6k}
    lm = ("Q6_K", random_q6k(V, H, tensor_seed(seed, GLOBAL_LAYER, GID["lm_head"]) & 0xFFFFFFFF, d_scale))
    w = LlamaWeights(shape, -1, emb, norm, lm)
    dims = {"q": (H, H), "k": (kvd, H), "v": (kvd, H), "o": (H, H), "gate": (I, H), "up": (I, H), "down": (H, I)}
    for l in range(shape.num_hidden_layers):
        L = {}
        for name, (r, c) in dims.items():
            t = KQ_MIX[name]
            L[name] = (t, rnd[t](r, c, tensor_seed(seed, l, TID[name]) & 0xFFFFFFFF, d_scale))
        L["attn_norm"] = normal(tensor_seed(seed, l, TID["attn_norm"]), 0, H, 1.0, 0.1)
        L["ffn_norm"] = normal(tensor_seed(seed, l, TID["ffn_norm"]), 0, H, 1.0, 0.1)
        w.layers.append(L)
    return w


class LlamaRef:
    """numpy restatement of LlamaForCausalLM (packages/forge-py/src/forge/
    models/llama.py:69-248) over quantized weights: pre-norm decoder, KV
    append, GQA by head grouping, causal SDPA with scale 1/sqrt(d), greedy
    argmax with the lowest-index tie rule.  ``kv_f16`` stores the cache
    rounded to fp16 (the build's cache format); False keeps fp32 as the
    reference does."""

    def __init__(self, w: LlamaWeights, max_seq: int, batch: int = 1, kv_f16: bool = True):
        self.w, self.s = w, w.shape
        s = self.s
        self.kv_f16 = kv_f16
        self.batch = batch
        self.k = [np.zeros((batch, s.num_key_value_heads, max_seq, s.head_dim), np.float32)
                  for _ in range(s.num_hidden_layers)]
        self.v = [np.zeros_like(self.k[0]) for _ in range(s.num_hidden_layers)]
        self.pos = 0
        self.embed = f16_to_f32(w.embed_f16)

    def synthesize_kv(self, seed: int, length: int, std: float = 1.0):
        """The cache fill of fg_llama_synthesize_kv: key (b, h, p, c) of layer l
        = fp16(std * N01(splitmix64(seed, l*16 + 9), ((b*Hkv + h)*length + p)*d + c)),
        values with l*16 + 10; the cache length becomes `length`."""
        s = self.s
        n = self.batch * s.num_key_value_heads * length * s.head_dim
        shp = (self.batch, s.num_key_value_heads, length, s.head_dim)
        for li in range(s.num_hidden_layers):
            self.k[li][:, :, :length] = round_f16(normal(tensor_seed(seed, li, 9), 0, n, 0.0, std).reshape(shp))
            self.v[li][:, :, :length] = round_f16(normal(tensor_seed(seed, li, 10), 0, n, 0.0, std).reshape(shp))
        self.pos = length

    def _lin(self, blocks, N, K, x):
        if isinstance(blocks, tuple):  # a k-quant Linear: (type name, GGUF blocks)
            t, b = blocks
            return qmatmul_q4k(b, N, K, x) if t == "Q4_K" else qmatmul_q6k(b, N, K, x)
        return qmatmul(self.w.qtype, blocks, N, K, x)

    def forward(self, ids: np.ndarray) -> np.ndarray:
        """ids [B, L] -> logits [B, L, vocab]; appends L positions to the cache."""
        s, w = self.s, self.w
        B, L = ids.shape
        Hd, H, Hkv, d, I = s.hidden_size, s.num_attention_heads, s.num_key_value_heads, s.head_dim, s.intermediate_size
        off = self.pos
        h = embedding(self.embed, ids)  # [B, L, H]
        for li, lw in enumerate(w.layers):
            x = rmsnorm(h, lw["attn_norm"], s.rms_norm_eps)
            q = self._lin(lw["q"], H * d, Hd, x).reshape(B, L, H, d).transpose(0, 2, 1, 3)
            k = self._lin(lw["k"], Hkv * d, Hd, x).reshape(B, L, Hkv, d).transpose(0, 2, 1, 3)
            v = self._lin(lw["v"], Hkv * d, Hd, x).reshape(B, L, Hkv, d).transpose(0, 2, 1, 3)
            q = rope(q, s.rope_theta, off)
            k = rope(k, s.rope_theta, off)
            if self.kv_f16:
                k, v = round_f16(k), round_f16(v)
            self.k[li][:, :, off:off + L] = k
            self.v[li][:, :, off:off + L] = v
            a = attention(q, self.k[li], self.v[li], 1.0 / np.sqrt(d), True, n_kv=off + L)
            a = np.ascontiguousarray(a.transpose(0, 2, 1, 3)).reshape(B, L, Hd)
            h = h + self._lin(lw["o"], Hd, Hd, a)
            x = rmsnorm(h, lw["ffn_norm"], s.rms_norm_eps)
            g = self._lin(lw["gate"], I, Hd, x)
            u = self._lin(lw["up"], I, Hd, x)
            h = h + self._lin(lw["down"], Hd, I, swiglu(g, u))
        self.pos += L
        hn = rmsnorm(h, w.norm, s.rms_norm_eps)
        return self._lin(w.lm_head, s.vocab_size, Hd, hn)

    def generate(self, prompt: np.ndarray, new_tokens: int):
        """Greedy decode (llama.py:212-248): returns (tokens [B, new], last logits)."""
        logits = self.forward(prompt)
        out = []
        nxt = np.array([argmax(logits[b, -1]) for b in range(prompt.shape[0])], np.int32)
        out.append(nxt)
        for _ in range(1, new_tokens):
            logits = self.forward(nxt[:, None])
            nxt = np.array([argmax(logits[b, -1]) for b in range(prompt.shape[0])], np.int32)
            out.append(nxt)
        return np.stack(out, 1), logits
