"""LlamaConfig / LlamaForCausalLM over the forge_b200 C ABI, mirroring
packages/forge-py/src/forge/models/llama.py:30-248 (forward with a KV cache
and greedy generate).  The model state (quantized weights, fp16 KV cache,
decode CUDA graph) lives in the library; Python passes token ids and reads
logits / next ids.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _capi as C
from .gpu_core import QTYPES, Context, default


@dataclass
class LlamaConfig:
    """llama.py:30-42 plus the build's fields: KV heads are already there;
    ``max_batch`` sequences decode together; ``qtype`` quantizes every Linear."""
    vocab_size: int = 32000
    hidden_size: int = 256
    intermediate_size: int = 688
    num_hidden_layers: int = 4
    num_attention_heads: int = 8
    num_key_value_heads: int = 8
    max_position_embeddings: int = 2048
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    max_batch: int = 1
    qtype: str = "Q4_0"

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def to_c(self) -> C.LlamaConfigC:
        c = C.LlamaConfigC()
        c.vocab_size, c.hidden_size, c.intermediate_size = self.vocab_size, self.hidden_size, self.intermediate_size
        c.num_hidden_layers, c.num_attention_heads = self.num_hidden_layers, self.num_attention_heads
        c.num_key_value_heads, c.max_position_embeddings = self.num_key_value_heads, self.max_position_embeddings
        c.max_batch, c.rms_norm_eps, c.rope_theta = self.max_batch, self.rms_norm_eps, self.rope_theta
        c.qtype = QTYPES[self.qtype]
        return c


# The shapes the benchmarks are quoted on.
TINYLLAMA_1_1B = dict(vocab_size=32000, hidden_size=2048, intermediate_size=5632, num_hidden_layers=22,
                      num_attention_heads=32, num_key_value_heads=4, rope_theta=10000.0)
LLAMA2_7B = dict(vocab_size=32000, hidden_size=4096, intermediate_size=11008, num_hidden_layers=32,
                 num_attention_heads=32, num_key_value_heads=32, rope_theta=10000.0)


class LlamaForCausalLM:
    def __init__(self, config: LlamaConfig, ctx: Context | None = None):
        self.config = config
        self.ctx = ctx or default()
        p = ctypes.c_void_p()
        cfg = config.to_c()
        C.call("fg_llama_create", self.ctx.ptr, ctypes.byref(cfg), ctypes.byref(p))
        self._p = p

    def close(self):
        if self._p is not None:
            C.call("fg_llama_destroy", self._p)
            self._p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------- weights
    def synthesize(self, seed: int, std: float = 0.02):
        """Seeded random-init weights (N(0, std) quantized Linears)."""
        C.call("fg_llama_synthesize", self._p, seed & (2**64 - 1), std)

    @classmethod
    def from_gguf(cls, path: str, ctx: Context | None = None, max_position_embeddings: int = 0, max_batch: int = 1):
        """A model with the configuration and weights of a llama.cpp-named
        GGUF file (Q4_0/Q8_0 Linears; each tensor-parallel rank keeps its shard)."""
        from .gguf import GGUFFile
        with GGUFFile(path) as g:
            m = cls(g.llama_config(max_position_embeddings, max_batch), ctx)
            C.call("fg_llama_load_gguf", m._p, g._p)
        return m

    def load(self, name: str, data: np.ndarray, layer: int = -1):
        """One weight of the full model: GGUF blocks for Linears, fp16 [V, H]
        embedding, fp32 norm gains.  Each TP rank keeps its shard."""
        a = np.ascontiguousarray(data)
        C.call("fg_llama_load", self._p, name.encode(), layer, a.ctypes.data_as(ctypes.c_void_p), a.nbytes)

    def reset(self):
        C.call("fg_llama_reset", self._p)

    def set_position(self, batch: int, pos: int):
        """Cache length `pos` for sequences [0, batch) without a prefill (the
        cache keeps its contents: zeros after creation)."""
        C.call("fg_llama_set_position", self._p, batch, pos)

    def synthesize_kv(self, seed: int, length: int, batch: int = 1, std: float = 1.0):
        """Seeded fp16 values in cache positions [0, length) of every layer for
        sequences [0, batch), and cache length `length` (a prefilled context
        without a prefill)."""
        C.call("fg_llama_synthesize_kv", self._p, seed & (2**64 - 1), batch, length, std)

    def decode_path(self, batch: int = 1) -> str:
        """'step' when a decode step of `batch` sequences runs the persistent
        one-launch kernel, 'layered' for the per-op kernels."""
        v = ctypes.c_int32()
        C.call("fg_llama_decode_path", self._p, batch, ctypes.byref(v))
        return "step" if v.value == 1 else "layered"

    @property
    def position(self) -> int:
        v = ctypes.c_int32()
        C.call("fg_llama_position", self._p, ctypes.byref(v))
        return v.value

    # ---------------------------------------------------------- forward / decode
    def forward(self, input_ids, return_logits: bool = True):
        """forward(input_ids) with the cache (llama.py:199-210): ids [B, L];
        appends L positions; returns (last-position logits [B, V], next ids [B])."""
        ids = np.ascontiguousarray(np.atleast_2d(np.asarray(input_ids, dtype=np.int32)))
        B, L = ids.shape
        nxt = np.empty(B, np.int32)
        logits = np.empty((B, self.config.vocab_size), np.float32) if return_logits else None
        C.call("fg_llama_forward", self._p, ids.ctypes.data_as(ctypes.c_void_p), B, L,
               logits.ctypes.data_as(ctypes.c_void_p) if logits is not None else None,
               nxt.ctypes.data_as(ctypes.c_void_p))
        return logits, nxt

    def decode(self, ids, return_logits: bool = False):
        """One greedy decode step (one CUDA graph launch)."""
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        B = ids.size
        nxt = np.empty(B, np.int32)
        logits = np.empty((B, self.config.vocab_size), np.float32) if return_logits else None
        C.call("fg_llama_decode", self._p, ids.ctypes.data_as(ctypes.c_void_p), B,
               nxt.ctypes.data_as(ctypes.c_void_p),
               logits.ctypes.data_as(ctypes.c_void_p) if logits is not None else None)
        return (nxt, logits) if return_logits else nxt

    def generate_device(self, batch: int, steps: int, read: bool = True):
        """`steps` greedy steps with ids kept on the device; returns [steps, batch]
        (with read=False only enqueues them; read_tokens() fetches them later)."""
        C.call("fg_llama_generate_device", self._p, batch, steps)
        return self.read_tokens(batch, steps) if read else None

    def read_tokens(self, batch: int, steps: int) -> np.ndarray:
        out = np.empty((steps, batch), np.int32)
        C.call("fg_llama_tokens", self._p, out.ctypes.data_as(ctypes.c_void_p), out.size)
        return out

    def generate(self, prompt_tokens, max_new_tokens: int = 20):
        """Greedy generation (llama.py:212-248): prefill, then decode steps.
        prompt_tokens: list of ids (one sequence) or [B, L]."""
        ids = np.atleast_2d(np.asarray(prompt_tokens, dtype=np.int32))
        self.reset()
        _, nxt = self.forward(ids, return_logits=False)
        out = [nxt.copy()]
        for _ in range(1, max_new_tokens):
            nxt = self.decode(nxt)
            out.append(nxt.copy())
        gen = np.stack(out, 1)
        if ids.shape[0] == 1:
            return list(ids[0]) + [int(t) for t in gen[0]]
        return np.concatenate([ids, gen], 1)
