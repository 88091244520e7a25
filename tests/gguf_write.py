"""Minimal GGUF v3 writer for the tests (the published container layout:
header, metadata key/values, tensor table, aligned data section).  Writes a
Llama model with llama.cpp tensor names from the oracle's host weights."""
import struct

import numpy as np

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 0, 1, 2, 8, 12, 14
KQ_GGML = {"Q4_K": GGML_Q4_K, "Q6_K": GGML_Q6_K}
V_U32, V_F32, V_STR, V_ARR = 4, 6, 8, 9


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key, vtype, value) -> bytes:
    out = _str(key) + struct.pack("<I", vtype)
    if vtype == V_U32:
        return out + struct.pack("<I", value)
    if vtype == V_F32:
        return out + struct.pack("<f", value)
    if vtype == V_STR:
        return out + _str(value)
    if vtype == V_ARR:  # array of strings
        return out + struct.pack("<IQ", V_STR, len(value)) + b"".join(_str(v) for v in value)
    raise ValueError(vtype)


def write(path, meta, tensors, alignment=32, version=3):
    """meta: [(key, vtype, value)]; tensors: [(name, ggml_type, dims (ne0 first), raw bytes)]."""
    kv = b"".join(_kv(k, t, v) for k, t, v in meta)
    table, blobs, off = b"", [], 0
    for name, gt, dims, raw in tensors:
        raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1).tobytes()
        table += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        table += struct.pack("<IQ", gt, off)
        blobs.append(raw)
        off += len(raw)
        off = (off + alignment - 1) // alignment * alignment
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(meta)) + kv + table
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * ((-len(head)) % alignment))
        for raw in blobs:
            f.write(raw)
            f.write(b"\0" * ((-len(raw)) % alignment))


def write_llama(path, w, context_length=256):
    """The oracle's LlamaWeights (GGUF Q4_0/Q8_0 blocks, or per-Linear (k-quant type, blocks) pairs of
    oracle.kquant_llama; fp16 embedding, fp32 gains)."""
    s = w.shape
    H, I, V, d = s.hidden_size, s.intermediate_size, s.vocab_size, s.head_dim
    qt = GGML_Q4_0 if w.qtype == 4 else GGML_Q8_0
    meta = [("general.architecture", V_STR, "llama"), ("general.alignment", V_U32, 32),
            ("llama.context_length", V_U32, context_length), ("llama.embedding_length", V_U32, H),
            ("llama.feed_forward_length", V_U32, I), ("llama.block_count", V_U32, s.num_hidden_layers),
            ("llama.attention.head_count", V_U32, s.num_attention_heads),
            ("llama.attention.head_count_kv", V_U32, s.num_key_value_heads),
            ("llama.rope.freq_base", V_F32, s.rope_theta),
            ("llama.attention.layer_norm_rms_epsilon", V_F32, s.rms_norm_eps),
            ("tokenizer.ggml.tokens", V_ARR, [f"t{i}" for i in range(8)])]
    kvd = s.num_key_value_heads * d
    t = [("token_embd.weight", GGML_F16, (H, V), w.embed_f16),
         ("output_norm.weight", GGML_F32, (H,), w.norm.astype(np.float32)),
         ("output.weight", *_lin(qt, (H, V), w.lm_head))]
    names = {"q": ("attn_q", (H, H)), "k": ("attn_k", (H, kvd)), "v": ("attn_v", (H, kvd)),
             "o": ("attn_output", (H, H)), "gate": ("ffn_gate", (H, I)), "up": ("ffn_up", (H, I)),
             "down": ("ffn_down", (I, H))}
    for l, L in enumerate(w.layers):
        t.append((f"blk.{l}.attn_norm.weight", GGML_F32, (H,), L["attn_norm"].astype(np.float32)))
        t.append((f"blk.{l}.ffn_norm.weight", GGML_F32, (H,), L["ffn_norm"].astype(np.float32)))
        for k, (gname, dims) in names.items():
            t.append((f"blk.{l}.{gname}.weight", *_lin(qt, dims, L[k])))
    write(path, meta, t)


def _lin(qt, dims, blocks):
    """(ggml type, dims, raw bytes) of a Linear: a k-quant (type name, blocks) pair, or blocks of the
    model's Q4_0 / Q8_0 type."""
    if isinstance(blocks, tuple):
        return KQ_GGML[blocks[0]], dims, blocks[1]
    return qt, dims, blocks
