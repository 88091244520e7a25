"""Host-side op API over the C ABI, mirroring the reference's gpuCore object
(packages/forge/src/tensor/gpuCore.ts:1448-1467) and the tensor lifecycle of
its bridge (init / read / dispose / getTensorInfo, pyodideBridge.ts:31-58).

Handles are strings ``"tensor_<hex>"`` as in the reference (types.ts:19);
errors are the reference's typed errors (forge_b200.errors).  Every op runs
on the GPU through libforge_b200.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _capi as C
from .errors import AMEVAForgeDisposedError, AMEVAForgeDTypeError

_NP_TO_FG = {np.dtype(np.float32): C.FG_F32, np.dtype(np.float16): C.FG_F16, np.dtype(np.int32): C.FG_I32,
             np.dtype(np.uint32): C.FG_U32, np.dtype(np.uint8): C.FG_U8}
_FG_TO_NP = {C.FG_F32: np.float32, C.FG_F16: np.float16, C.FG_I32: np.int32, C.FG_U32: np.uint32, C.FG_U8: np.uint8}
QTYPES = {"Q4_0": C.FG_Q4_0, "Q8_0": C.FG_Q8_0, "Q4_K": C.FG_Q4_K, "Q6_K": C.FG_Q6_K, C.FG_Q4_0: C.FG_Q4_0,
          C.FG_Q8_0: C.FG_Q8_0, C.FG_Q4_K: C.FG_Q4_K, C.FG_Q6_K: C.FG_Q6_K}
GGUF_BLOCK_BYTES = {C.FG_Q4_0: 18, C.FG_Q8_0: 34, C.FG_Q4_K: 144, C.FG_Q6_K: 210}
GGUF_BLOCK_VALUES = {C.FG_Q4_0: 32, C.FG_Q8_0: 32, C.FG_Q4_K: 256, C.FG_Q6_K: 256}


def _h(handle: str) -> int:
    if not isinstance(handle, str) or not handle.startswith("tensor_"):
        raise AMEVAForgeDisposedError(f"Tensor not found: {handle!r}")
    return int(handle[7:], 16)


def _s(h: int) -> str:
    return "tensor_%016x" % h


def nccl_unique_id() -> bytes:
    buf = (ctypes.c_uint8 * 128)()
    C.call("fg_nccl_unique_id", buf)
    return bytes(buf)


def device_count() -> int:
    n = ctypes.c_int32(0)
    C.call("fg_device_count", ctypes.byref(n))
    return n.value


class Context:
    """One device context (gpuCore.init): a CUDA device, its stream, the handle
    registry and the VRAM quota.  Under tensor parallelism each rank owns one."""

    def __init__(self, device: int = 0, vram_limit_bytes: int = 0, tp_rank: int = 0, tp_size: int = 1,
                 nccl_id: bytes | None = None):
        opts = C.InitOpts()
        opts.device, opts.tp_rank, opts.tp_size = device, tp_rank, tp_size
        opts.vram_limit_bytes = vram_limit_bytes
        if nccl_id is not None:
            ctypes.memmove(opts.nccl_id, nccl_id, 128)
        p = ctypes.c_void_p()
        C.call("fg_init", ctypes.byref(opts), ctypes.byref(p))
        self._p = p
        self.device, self.tp_rank, self.tp_size = device, tp_rank, tp_size

    @property
    def ptr(self):
        if self._p is None:
            raise AMEVAForgeDisposedError("context was shut down")
        return self._p

    def shutdown(self):
        if self._p is not None:
            C.call("fg_shutdown", self._p)
            self._p = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.shutdown()

    # ---------------------------------------------------------- lifecycle
    def upload(self, array, dtype=None) -> str:
        a = np.ascontiguousarray(array if dtype is None else np.asarray(array, dtype=dtype))
        if a.dtype not in _NP_TO_FG:
            raise AMEVAForgeDTypeError(f"unsupported upload dtype {a.dtype}")
        shape = (ctypes.c_int64 * max(1, a.ndim))(*a.shape)
        h = ctypes.c_uint64()
        C.call("fg_upload", self.ptr, a.ctypes.data_as(ctypes.c_void_p), a.nbytes, shape, a.ndim,
               _NP_TO_FG[a.dtype], ctypes.byref(h))
        return _s(h.value)

    uploadFloat32Array = upload

    def upload_quant(self, qtype, blocks: np.ndarray, rows: int, cols: int) -> str:
        qt = QTYPES[qtype]
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        h = ctypes.c_uint64()
        C.call("fg_upload_quant", self.ptr, qt, b.ctypes.data_as(ctypes.c_void_p), b.nbytes, rows, cols,
               ctypes.byref(h))
        return _s(h.value)

    def empty(self, shape, dtype=np.float32) -> str:
        shp = (ctypes.c_int64 * max(1, len(shape)))(*shape)
        h = ctypes.c_uint64()
        C.call("fg_empty", self.ptr, shp, len(shape), _NP_TO_FG[np.dtype(dtype)], ctypes.byref(h))
        return _s(h.value)

    def info(self, handle: str) -> dict:
        ti = C.TensorInfo()
        C.call("fg_info", self.ptr, _h(handle), ctypes.byref(ti))
        return {"shape": tuple(ti.shape[i] for i in range(ti.ndim)), "dtype": ti.dtype, "bytes": ti.bytes,
                "device_ptr": ti.device_ptr}

    getTensorInfo = info

    def read(self, handle: str) -> np.ndarray:
        inf = self.info(handle)
        if inf["dtype"] not in _FG_TO_NP:
            raise AMEVAForgeDTypeError("quantized tensors are read with read_quant_gguf")
        out = np.empty(inf["shape"], dtype=_FG_TO_NP[inf["dtype"]])
        C.call("fg_read", self.ptr, _h(handle), out.ctypes.data_as(ctypes.c_void_p), out.nbytes)
        return out

    def read_quant_gguf(self, handle: str) -> np.ndarray:
        inf = self.info(handle)
        rows, cols = inf["shape"]
        dt = inf["dtype"]
        out = np.empty((rows, cols // GGUF_BLOCK_VALUES[dt] * GGUF_BLOCK_BYTES[dt]), dtype=np.uint8)
        C.call("fg_read_quant_gguf", self.ptr, _h(handle), out.ctypes.data_as(ctypes.c_void_p), out.nbytes)
        return out

    def dispose(self, handle: str):
        C.call("fg_dispose", self.ptr, _h(handle))

    def dispose_batch(self, handles):
        arr = (ctypes.c_uint64 * len(handles))(*[_h(x) for x in handles])
        C.call("fg_dispose_batch", self.ptr, arr, len(handles))

    disposeBatch = dispose_batch

    def synchronize(self):
        C.call("fg_synchronize", self.ptr)

    def quota(self) -> dict:
        q = C.Quota()
        C.call("fg_quota_snapshot", self.ptr, ctypes.byref(q))
        return {"limit": q.limit_bytes, "active": q.active_bytes, "pending": q.pending_bytes,
                "peak": q.peak_bytes, "live_tensors": q.live_tensors}

    getQuotaSnapshot = quota

    def configure_runtime(self, allow_non_finite: bool = False):
        C.call("fg_set_allow_non_finite", self.ptr, 1 if allow_non_finite else 0)

    # ---------------------------------------------------------- ops
    def _op(self, name, *args) -> str:
        h = ctypes.c_uint64()
        C.call(name, self.ptr, *args, ctypes.byref(h))
        return _s(h.value)

    def unpackQuant(self, packed, scales, zeros, bits: int = 4, groupSize: int = 128, numElements: int = 0) -> str:
        return self._op("fg_unpack_quant", _h(packed), _h(scales), _h(zeros), bits, groupSize, numElements)

    def dequant(self, w) -> str:
        return self._op("fg_dequant", _h(w))

    def qmatmul(self, x, w) -> str:
        return self._op("fg_qmatmul", _h(x), _h(w))

    def qmatmul_into(self, x, w, out) -> str:
        C.call("fg_qmatmul_into", self.ptr, _h(x), _h(w), _h(out))
        return out

    def stream_ptr(self) -> int:
        s = ctypes.c_void_p()
        C.call("fg_get_stream", self.ptr, ctypes.byref(s))
        return s.value

    def matmul(self, a, b) -> str:
        return self._op("fg_matmul", _h(a), _h(b))

    def flashAttention(self, q, k, v, scale=None, isCausal: bool = False) -> str:
        return self._op("fg_flash_attention", _h(q), _h(k), _h(v), 0.0 if scale is None else float(scale),
                        0 if scale is None else 1, 1 if isCausal else 0)

    def rmsNorm(self, x, gamma=None, eps: float = 1e-5) -> str:
        return self._op("fg_rmsnorm", _h(x), 0 if gamma is None else _h(gamma), eps)

    def rope(self, x, base: float = 1e4, offset: int = 0) -> str:
        return self._op("fg_rope", _h(x), base, offset)

    def swiglu(self, gate, up) -> str:
        return self._op("fg_swiglu", _h(gate), _h(up))

    def embedding(self, weight, index) -> str:
        return self._op("fg_embedding", _h(weight), _h(index))

    def add(self, a, b) -> str:
        return self._op("fg_add", _h(a), _h(b))

    def argmax(self, logits) -> str:
        return self._op("fg_argmax", _h(logits))

    def sample(self, logits, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0, seed=None) -> str:
        """LLMSampler.sample (sampling.ts:35-128) per row: I32 [rows]."""
        return self._op("fg_sample", _h(logits), float(temperature), int(top_k), float(top_p),
                        0 if seed is None else 1, 0 if seed is None else int(seed) & 0xFFFFFFFF)

    def cast(self, x, dtype) -> str:
        return self._op("fg_cast", _h(x), _NP_TO_FG[np.dtype(dtype)])

    def synth_normal(self, shape, dtype=np.float32, seed: int = 0, offset: int = 0, mean: float = 0.0,
                     std: float = 1.0) -> str:
        shp = (ctypes.c_int64 * max(1, len(shape)))(*shape)
        return self._op("fg_synth_normal", shp, len(shape), _NP_TO_FG[np.dtype(dtype)], seed & (2**64 - 1), offset,
                        mean, std)

    def synth_quant(self, qtype, rows: int, cols: int, seed: int, row0: int = 0, std: float = 0.02) -> str:
        return self._op("fg_synth_quant", QTYPES[qtype], rows, cols, seed & (2**64 - 1), row0, std)

    # snake_case aliases (forge-py naming)
    unpack_quant = unpackQuant
    flash_attention = flashAttention
    rms_norm = rmsNorm


_default: Context | None = None


def init(device: int = 0, vram_limit_bytes: int = 0) -> Context:
    """gpuCore.init: create (once) the process-wide default context."""
    global _default
    if _default is None:
        _default = Context(device=device, vram_limit_bytes=vram_limit_bytes)
    return _default


def default() -> Context:
    return init()
