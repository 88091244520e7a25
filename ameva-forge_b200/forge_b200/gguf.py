"""GGUF files over the forge_b200 C ABI (fg_gguf_*): the memory-mapped,
validated container reader and the Llama weight loader.  No parsing happens
in Python; this wraps the library's reader so the Python, C++ and N-API hosts
all load files the same way."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _capi as C

_FG_TO_NAME = {0: "F32", 1: "F16", 16: "Q4_0", 17: "Q8_0", 18: "Q4_K", 19: "Q6_K", -1: "unsupported"}


class GGUFFile:
    """An open GGUF file: tensor table, metadata lookups and zero-copy views
    of tensor bytes (valid while the file is open)."""

    def __init__(self, path: str):
        p = ctypes.c_void_p()
        C.call("fg_gguf_open", str(path).encode(), ctypes.byref(p))
        self._p = p

    def close(self):
        if self._p is not None:
            C.call("fg_gguf_close", self._p)
            self._p = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        n = ctypes.c_int64()
        C.call("fg_gguf_tensor_count", self._p, ctypes.byref(n))
        return n.value

    def tensor(self, i: int) -> dict:
        name, dt, nd = ctypes.c_char_p(), ctypes.c_int32(), ctypes.c_int32()
        dims, data, nb = (ctypes.c_int64 * 4)(), ctypes.c_void_p(), ctypes.c_uint64()
        C.call("fg_gguf_tensor_info", self._p, i, ctypes.byref(name), ctypes.byref(dt), ctypes.byref(nd), dims,
               ctypes.byref(data), ctypes.byref(nb))
        raw = None
        if data.value and nb.value:
            raw = np.ctypeslib.as_array((ctypes.c_uint8 * nb.value).from_address(data.value))
        return {"name": name.value.decode(), "dtype": _FG_TO_NAME.get(dt.value, "unsupported"),
                "dims": tuple(dims[k] for k in range(nd.value)), "bytes": raw}

    def tensors(self):
        return [self.tensor(i) for i in range(len(self))]

    def number(self, key: str) -> float:
        v = ctypes.c_double()
        C.call("fg_gguf_meta_number", self._p, key.encode(), ctypes.byref(v))
        return v.value

    def string(self, key: str) -> str:
        v = ctypes.c_char_p()
        C.call("fg_gguf_meta_string", self._p, key.encode(), ctypes.byref(v))
        return v.value.decode()

    def llama_config(self, max_position_embeddings: int = 0, max_batch: int = 1):
        from .llama import LlamaConfig
        c = C.LlamaConfigC()
        C.call("fg_gguf_llama_config", self._p, max_position_embeddings, max_batch, ctypes.byref(c))
        return LlamaConfig(vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                           num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads,
                           num_key_value_heads=c.num_key_value_heads,
                           max_position_embeddings=c.max_position_embeddings, rms_norm_eps=c.rms_norm_eps,
                           rope_theta=c.rope_theta, max_batch=c.max_batch,
                           qtype={16: "Q4_0", 17: "Q8_0", 18: "Q4_K"}[c.qtype])
