"""ctypes binding of libforge_b200.so (include/forge_b200.h).

This is the Python twin of the N-API shim a TypeScript host would use: plain
C types in, status codes out, messages from fg_last_error().  The library is
the in-tree build (forge_b200/_lib); there is no fallback -- if it is missing
or cannot be loaded, every call fails loudly.
"""
import ctypes
import os

from . import errors

_HERE = os.path.dirname(os.path.abspath(__file__))
# FORGE_B200_LIBRARY selects another build of the same library (profiling
# experiments); by default the in-tree build is used.
LIB_PATH = os.environ.get("FORGE_B200_LIBRARY") or os.path.join(_HERE, "_lib", "libforge_b200.so")

FG_F32, FG_F16, FG_I32, FG_U8, FG_U32, FG_Q4_0, FG_Q8_0, FG_Q4_K, FG_Q6_K = 0, 1, 3, 4, 5, 16, 17, 18, 19
MAX_DIMS = 8

c_i32, c_i64, c_u64, c_f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float
c_vp = ctypes.c_void_p
c_h = ctypes.c_uint64
P = ctypes.POINTER


class InitOpts(ctypes.Structure):
    _fields_ = [("device", c_i32), ("tp_rank", c_i32), ("tp_size", c_i32), ("reserved", c_i32),
                ("vram_limit_bytes", c_u64), ("nccl_id", ctypes.c_uint8 * 128)]


class TensorInfo(ctypes.Structure):
    _fields_ = [("dtype", c_i32), ("ndim", c_i32), ("shape", c_i64 * MAX_DIMS), ("bytes", c_u64),
                ("device_ptr", c_u64)]


class Quota(ctypes.Structure):
    _fields_ = [("limit_bytes", c_u64), ("active_bytes", c_u64), ("pending_bytes", c_u64),
                ("peak_bytes", c_u64), ("live_tensors", c_u64)]


class LlamaConfigC(ctypes.Structure):
    _fields_ = [("vocab_size", c_i32), ("hidden_size", c_i32), ("intermediate_size", c_i32),
                ("num_hidden_layers", c_i32), ("num_attention_heads", c_i32), ("num_key_value_heads", c_i32),
                ("max_position_embeddings", c_i32), ("max_batch", c_i32), ("rms_norm_eps", c_f32),
                ("rope_theta", c_f32), ("qtype", c_i32), ("reserved", c_i32)]


# name -> (argtypes) ; every function returns int status unless listed in _RESTYPE
_SIGS = {
    "fg_version": [],
    "fg_last_error": [],
    "fg_status_name": [ctypes.c_int],
    "fg_device_count": [P(c_i32)],
    "fg_init": [P(InitOpts), P(c_vp)],
    "fg_shutdown": [c_vp],
    "fg_nccl_unique_id": [ctypes.c_uint8 * 128],
    "fg_synchronize": [c_vp],
    "fg_get_stream": [c_vp, P(c_vp)],
    "fg_quota_snapshot": [c_vp, P(Quota)],
    "fg_upload": [c_vp, c_vp, c_u64, P(c_i64), c_i32, c_i32, P(c_h)],
    "fg_upload_quant": [c_vp, c_i32, c_vp, c_u64, c_i64, c_i64, P(c_h)],
    "fg_empty": [c_vp, P(c_i64), c_i32, c_i32, P(c_h)],
    "fg_read": [c_vp, c_h, c_vp, c_u64],
    "fg_read_quant_gguf": [c_vp, c_h, c_vp, c_u64],
    "fg_info": [c_vp, c_h, P(TensorInfo)],
    "fg_dispose": [c_vp, c_h],
    "fg_dispose_batch": [c_vp, P(c_h), c_i32],
    "fg_set_allow_non_finite": [c_vp, c_i32],
    "fg_unpack_quant": [c_vp, c_h, c_h, c_h, c_i32, c_i64, c_i64, P(c_h)],
    "fg_dequant": [c_vp, c_h, P(c_h)],
    "fg_qmatmul": [c_vp, c_h, c_h, P(c_h)],
    "fg_qmatmul_into": [c_vp, c_h, c_h, c_h],
    "fg_matmul": [c_vp, c_h, c_h, P(c_h)],
    "fg_flash_attention": [c_vp, c_h, c_h, c_h, c_f32, c_i32, c_i32, P(c_h)],
    "fg_attention_decode_static": [c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i64, c_i32, c_f32, c_vp],
    "fg_rmsnorm": [c_vp, c_h, c_h, c_f32, P(c_h)],
    "fg_rope": [c_vp, c_h, c_f32, c_i64, P(c_h)],
    "fg_swiglu": [c_vp, c_h, c_h, P(c_h)],
    "fg_embedding": [c_vp, c_h, c_h, P(c_h)],
    "fg_add": [c_vp, c_h, c_h, P(c_h)],
    "fg_argmax": [c_vp, c_h, P(c_h)],
    "fg_cast": [c_vp, c_h, c_i32, P(c_h)],
    "fg_synth_normal": [c_vp, P(c_i64), c_i32, c_i32, c_u64, c_u64, c_f32, c_f32, P(c_h)],
    "fg_synth_quant": [c_vp, c_i32, c_i64, c_i64, c_u64, c_i64, c_f32, P(c_h)],
    "fg_llama_create": [c_vp, P(LlamaConfigC), P(c_vp)],
    "fg_llama_destroy": [c_vp],
    "fg_llama_load": [c_vp, ctypes.c_char_p, c_i32, c_vp, c_u64],
    "fg_llama_synthesize": [c_vp, c_u64, c_f32],
    "fg_llama_reset": [c_vp],
    "fg_llama_position": [c_vp, P(c_i32)],
    "fg_llama_forward": [c_vp, c_vp, c_i32, c_i32, c_vp, c_vp],
    "fg_llama_decode": [c_vp, c_vp, c_i32, c_vp, c_vp],
    "fg_llama_generate_device": [c_vp, c_i32, c_i32],
    "fg_llama_tokens": [c_vp, c_vp, c_i64],
    "fg_llama_get_config": [c_vp, P(LlamaConfigC)],
    "fg_llama_set_position": [c_vp, c_i32, c_i32],
    "fg_llama_synthesize_kv": [c_vp, c_u64, c_i32, c_i32, c_f32],
    "fg_llama_decode_path": [c_vp, c_i32, P(c_i32)],
    "fg_sample": [c_vp, c_h, ctypes.c_double, c_i32, ctypes.c_double, c_i32, ctypes.c_uint32, P(c_h)],
    "fg_gguf_open": [ctypes.c_char_p, P(c_vp)],
    "fg_gguf_close": [c_vp],
    "fg_gguf_tensor_count": [c_vp, P(c_i64)],
    "fg_gguf_tensor_info": [c_vp, c_i64, P(ctypes.c_char_p), P(c_i32), P(c_i32), P(c_i64), P(c_vp), P(ctypes.c_uint64)],
    "fg_gguf_meta_number": [c_vp, ctypes.c_char_p, P(ctypes.c_double)],
    "fg_gguf_meta_string": [c_vp, ctypes.c_char_p, P(ctypes.c_char_p)],
    "fg_gguf_llama_config": [c_vp, c_i32, c_i32, P(LlamaConfigC)],
    "fg_llama_load_gguf": [c_vp, c_vp],
    "fg_execute_graph": [c_vp, ctypes.c_char_p, P(c_vp), P(c_u64), c_i32, P(c_i64), P(c_h), c_i32, P(c_i32)],
    "fg_configure_graph": [c_vp, c_i64, c_i32, c_i64],
}
_RESTYPE = {"fg_version": ctypes.c_char_p, "fg_last_error": ctypes.c_char_p, "fg_status_name": ctypes.c_char_p}

_lib = None


def lib():
    """Load the in-tree library once; raise if it is absent (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise errors.AMEVAForgeWebGPUUnavailableError(
                f"forge_b200 native library not built: {LIB_PATH} (run ameva-forge_b200/build.py)")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, ctypes.c_int)
        _lib = L
    return _lib


def check(status: int):
    if status != 0:
        msg = lib().fg_last_error().decode("utf-8", "replace")
        errors.raise_for(status, msg)


def call(name: str, *args):
    check(getattr(lib(), name)(*args))
