"""fg_attention_decode_static: decode attention for callers that cannot
allocate device memory while they decode (a host whose VRAM is committed to
its own KV cache, a latency-critical thread where cudaMalloc would
synchronise the device, a host that owns its buffers but no fg_ctx).  It
keeps its split-KV scratch in a static device array instead.

Each call is checked against the oracle (oracle.attention on the same fp16
cache values, the reference's online softmax in double accumulation) and
against fg_flash_attention, the pooled entry point, on the same inputs; two
calls run in a row on the same static array.  Both kernels compute in fp32;
the tolerance is 1e-4 * ||ref||_inf.

The file sorts last so that it also runs after every other GPU test of the
session (the static counters must still be zero then); it passes alone too.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err
from forge_b200 import _capi as C
from forge_b200.errors import AMEVAForgeShapeError, AMEVAForgeValidationError

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _case(seed, B, H, Hkv, d, cap):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, H, d), dtype=np.float32)
    kc = rng.standard_normal((B, Hkv, cap, d), dtype=np.float32).astype(np.float16)
    vc = rng.standard_normal((B, Hkv, cap, d), dtype=np.float32).astype(np.float16)
    return q, kc, vc


def _ptr(ctx, h):
    return ctypes.c_void_p(ctx.info(h)["device_ptr"])


def _static_call(ctx, hq, hk, hv, hout, B, H, Hkv, d, cap, n_kv, scale):
    C.call("fg_attention_decode_static", _ptr(ctx, hq), _ptr(ctx, hk), _ptr(ctx, hv), _ptr(ctx, hout), B, H, Hkv, d,
           cap, n_kv, scale, ctypes.c_void_p(ctx.stream_ptr()))


def _pooled_ref(ctx, q, kc, vc, n_kv, scale):
    B, H, d = q.shape
    hq = ctx.upload(q.reshape(B, H, 1, d))
    hk = ctx.upload(np.ascontiguousarray(kc[:, :, :n_kv].astype(np.float32)))
    hv = ctx.upload(np.ascontiguousarray(vc[:, :, :n_kv].astype(np.float32)))
    ho = ctx.flashAttention(hq, hk, hv, scale=scale)
    out = ctx.read(ho).reshape(B, H, d)
    ctx.dispose_batch([hq, hk, hv, ho])
    return out


@pytest.mark.parametrize("B,H,Hkv,d,cap,n_kvs", [
    (1, 32, 32, 128, 4096, (1000, 4096)),   # Llama-2-7B decode, two lengths (different split counts)
    (3, 32, 4, 64, 2048, (777, 2048)),      # TinyLlama-1.1B GQA group 8, batch 3
    (2, 8, 4, 128, 300, (300, 1)),          # group 2, single key on the second call
])
def test_two_calls_match_flash_attention(ctx, B, H, Hkv, d, cap, n_kvs):
    q, kc, vc = _case(B * 1000 + H + d, B, H, Hkv, d, cap)
    hq, hk, hv = ctx.upload(q), ctx.upload(kc), ctx.upload(vc)
    hout = ctx.empty((B, H, d), np.float32)
    scale = float(1.0 / np.sqrt(d))
    quota0 = ctx.quota()
    for n_kv in n_kvs:  # two calls in a row reuse the same static scratch
        _static_call(ctx, hq, hk, hv, hout, B, H, Hkv, d, cap, n_kv, scale)
        out = ctx.read(hout)
        oref = O.attention(q.reshape(B, H, 1, d), kc.astype(np.float32), vc.astype(np.float32), scale,
                           n_kv=n_kv).reshape(B, H, d)
        err = max_rel_err(out, oref)
        assert err < TOL, ("oracle", n_kv, err)
        err = max_rel_err(out, _pooled_ref(ctx, q, kc, vc, n_kv, scale))
        assert err < TOL, ("fg_flash_attention", n_kv, err)
    # the pooled reference disposed what it made; the static calls added nothing
    assert ctx.quota()["live_tensors"] == quota0["live_tensors"]
    ctx.dispose_batch([hq, hk, hv, hout])


def test_shape_beyond_static_scratch_runs_with_fewer_splits(ctx):
    # 280 KV heads of group 8 and d 128 split in two would need 2.3 MB of partials: the call takes
    # fewer splits (one needs no scratch) and still matches the oracle
    B, H, Hkv, d, cap = 1, 2240, 280, 128, 256
    q, kc, vc = _case(7, B, H, Hkv, d, cap)
    hq, hk, hv = ctx.upload(q), ctx.upload(kc), ctx.upload(vc)
    hout = ctx.empty((B, H, d), np.float32)
    _static_call(ctx, hq, hk, hv, hout, B, H, Hkv, d, cap, cap, 0.088)
    oref = O.attention(q.reshape(B, H, 1, d), kc.astype(np.float32), vc.astype(np.float32), 0.088,
                       n_kv=cap).reshape(B, H, d)
    assert max_rel_err(ctx.read(hout), oref) < TOL
    with pytest.raises(AMEVAForgeShapeError, match="n_kv"):
        _static_call(ctx, hq, hk, hv, hout, B, H, Hkv, d, cap, cap + 1, 0.088)
    ctx.dispose_batch([hq, hk, hv, hout])
    # a supported call still works after the rejection
    test_two_calls_match_flash_attention(ctx, 1, 8, 8, 64, 512, (512, 100))


def test_rejects_misaligned_cache_pointer(ctx):
    # a K cache that starts 8 bytes into a buffer (e.g. a slice at an odd token offset of a head_dim-4 row
    # layout) cannot be copied in 16-byte chunks: the call must return a status, not fault
    B, H, Hkv, d, cap = 1, 8, 8, 64, 128
    q, kc, vc = _case(9, B, H, Hkv, d, cap)
    hq, hk, hv = ctx.upload(q), ctx.upload(kc), ctx.upload(vc)
    hout = ctx.empty((B, H, d), np.float32)
    bad = ctypes.c_void_p(ctx.info(hk)["device_ptr"] + 8)
    with pytest.raises(AMEVAForgeValidationError, match="16-byte aligned"):
        C.call("fg_attention_decode_static", _ptr(ctx, hq), bad, _ptr(ctx, hv), _ptr(ctx, hout), B, H, Hkv, d,
               cap - 8, 64, 0.125, ctypes.c_void_p(ctx.stream_ptr()))
    badq = ctypes.c_void_p(ctx.info(hq)["device_ptr"] + 2)
    with pytest.raises(AMEVAForgeValidationError, match="4-byte aligned"):
        C.call("fg_attention_decode_static", badq, _ptr(ctx, hk), _ptr(ctx, hv), _ptr(ctx, hout), B, H, Hkv, d,
               cap, 64, 0.125, ctypes.c_void_p(ctx.stream_ptr()))
    ctx.dispose_batch([hq, hk, hv, hout])
