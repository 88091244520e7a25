"""Flash attention vs the reference fixtures (fp32, atol 1e-4 as the
reference's own suite) and the oracle (fp16 inputs, 2e-3 * ||ref||_inf)."""
import numpy as np
import pytest

import inputs as I
import oracle as O
from conftest import max_rel_err
from forge_b200.errors import AMEVAForgeShapeError

pytestmark = pytest.mark.gpu


def test_mha_golden(ctx, golden):
    q, k, v = I.mha()
    out = ctx.read(ctx.flashAttention(ctx.upload(q), ctx.upload(k), ctx.upload(v), isCausal=False))
    np.testing.assert_allclose(out, golden["mha_out"], atol=1e-4)


def test_gqa_causal_golden(ctx, golden):
    q, k, v = I.gqa()
    out = ctx.read(ctx.flashAttention(ctx.upload(q), ctx.upload(k), ctx.upload(v), isCausal=True))
    np.testing.assert_allclose(out, golden["gqa_out"], atol=1e-4)


@pytest.mark.parametrize("B,H,Hkv,Nq,Nkv,d,causal", [
    (1, 4, 4, 1, 37, 64, True),      # decode row against a KV offset
    (2, 8, 2, 5, 70, 128, True),     # chunked prefill with KV offset
    (1, 2, 1, 33, 33, 256, False),   # max head dim
    (1, 2, 2, 3, 2, 8, True),        # fewer keys than queries: early rows see none
    (3, 2, 2, 17, 17, 32, True),
])
def test_fp32_ragged_vs_oracle(ctx, B, H, Hkv, Nq, Nkv, d, causal):
    q = O.normal(1, 0, B * H * Nq * d).reshape(B, H, Nq, d)
    k = O.normal(2, 0, B * Hkv * Nkv * d).reshape(B, Hkv, Nkv, d)
    v = O.normal(3, 0, B * Hkv * Nkv * d).reshape(B, Hkv, Nkv, d)
    out = ctx.read(ctx.flashAttention(ctx.upload(q), ctx.upload(k), ctx.upload(v), isCausal=causal))
    np.testing.assert_allclose(out, O.attention(q, k, v, causal=causal), atol=2e-5)


def test_fp16_prefill_vs_oracle(ctx):
    B, H, S, d = 1, 4, 512, 128
    q16 = O.f32_to_f16(O.normal(11, 0, B * H * S * d)).reshape(B, H, S, d)
    k16 = O.f32_to_f16(O.normal(12, 0, B * H * S * d)).reshape(B, H, S, d)
    v16 = O.f32_to_f16(O.normal(13, 0, B * H * S * d)).reshape(B, H, S, d)
    out = ctx.read(ctx.flashAttention(ctx.upload(q16.view(np.float16)), ctx.upload(k16.view(np.float16)),
                                      ctx.upload(v16.view(np.float16)), scale=1 / np.sqrt(d), isCausal=True))
    ref = O.attention(O.f16_to_f32(q16), O.f16_to_f32(k16), O.f16_to_f32(v16), 1 / np.sqrt(d), True)
    assert max_rel_err(out, ref) <= 2e-3


@pytest.mark.parametrize("B,H,Hkv,Nq,Nkv,d,causal", [
    (1, 2, 2, 128, 128, 128, True),    # one query block, one key block, diagonal mask
    (1, 4, 1, 200, 333, 64, True),     # GQA 4:1, ragged blocks, KV offset 133
    (2, 2, 2, 256, 256, 128, False),   # non-causal, two batches
    (1, 2, 2, 130, 100, 128, True),    # more queries than keys: the first 30 rows see none
    (1, 8, 2, 16, 700, 128, True),     # a 16-token chunk over a 700-token cache
    (1, 2, 1, 640, 640, 64, True),     # five query blocks, O rescaled across five key blocks
])
def test_fp16_tensor_core_vs_oracle(ctx, B, H, Hkv, Nq, Nkv, d, causal):
    """fp16 Q/K/V with head_dim 64/128 take the tcgen05 kernel (attention_tc.cu)."""
    q16 = O.f32_to_f16(O.normal(21, 0, B * H * Nq * d)).reshape(B, H, Nq, d)
    k16 = O.f32_to_f16(O.normal(22, 0, B * Hkv * Nkv * d)).reshape(B, Hkv, Nkv, d)
    v16 = O.f32_to_f16(O.normal(23, 0, B * Hkv * Nkv * d)).reshape(B, Hkv, Nkv, d)
    out = ctx.read(ctx.flashAttention(ctx.upload(q16.view(np.float16)), ctx.upload(k16.view(np.float16)),
                                      ctx.upload(v16.view(np.float16)), isCausal=causal))
    ref = O.attention(O.f16_to_f32(q16), O.f16_to_f32(k16), O.f16_to_f32(v16), 1 / np.sqrt(d), causal)
    assert np.isfinite(out).all()
    assert max_rel_err(out, ref) <= 2e-3


@pytest.mark.parametrize("B,H,Hkv,Nq,Nkv,d,causal,mag", [
    (1, 2, 2, 128, 128, 128, True, 1.0),    # one query block, one key block, diagonal mask
    (1, 4, 1, 200, 333, 64, True, 1.0),     # GQA 4:1, ragged blocks, KV offset 133
    (2, 2, 2, 256, 256, 128, False, 1.0),   # non-causal, two batches
    (1, 2, 2, 130, 100, 128, True, 1.0),    # more queries than keys: the first 30 rows see none
    (1, 8, 2, 16, 700, 128, True, 1.0),     # a 16-token chunk over a 700-token cache
    (1, 2, 1, 640, 640, 64, True, 1.0),     # five query blocks, O rescaled across five key blocks
    (1, 2, 2, 300, 300, 128, True, 1000.0),  # magnitudes past fp16's range: the per-head / per-row scales
    (1, 2, 2, 300, 300, 128, True, 1e-3),    # small magnitudes: the lo halves stay normal
])
def test_fp32_tensor_core_vs_oracle(ctx, B, H, Hkv, Nq, Nkv, d, causal, mag):
    """fp32 Q/K/V (the executeGraph path) with head_dim 64/128 take attention_tc32.cu: scores from fp16
    hi/lo splits (three tensor-core passes), P V in fp16; bar 1e-3 * ||ref||_inf (fp32 accumulation)."""
    q = O.normal(31, 0, B * H * Nq * d).reshape(B, H, Nq, d) * np.float32(mag)
    k = O.normal(32, 0, B * Hkv * Nkv * d).reshape(B, Hkv, Nkv, d) * np.float32(mag)
    v = O.normal(33, 0, B * Hkv * Nkv * d).reshape(B, Hkv, Nkv, d) * np.float32(mag)
    scale = 1 / np.sqrt(d) / mag  # keeps the scores' spread at N(0, 1)-like values
    out = ctx.read(ctx.flashAttention(ctx.upload(q), ctx.upload(k), ctx.upload(v), scale=scale, isCausal=causal))
    ref = O.attention(q, k, v, scale, causal)
    assert np.isfinite(out).all()
    assert max_rel_err(out, ref) <= 1e-3


def test_fp32_tensor_core_wide_scores(ctx):
    """Scores spread far wider than N(0, 1) (|s scale| up to ~40): the split keeps fp32-class accuracy
    where fp16-rounded operands would not."""
    B, H, Nq, d = 1, 2, 256, 128
    q = O.normal(41, 0, B * H * Nq * d).reshape(B, H, Nq, d) * np.float32(4.0)
    k = O.normal(42, 0, B * H * Nq * d).reshape(B, H, Nq, d) * np.float32(4.0)
    v = O.normal(43, 0, B * H * Nq * d).reshape(B, H, Nq, d)
    out = ctx.read(ctx.flashAttention(ctx.upload(q), ctx.upload(k), ctx.upload(v), isCausal=True))
    ref = O.attention(q, k, v, 1 / np.sqrt(d), True)
    assert max_rel_err(out, ref) <= 1e-3


def test_validation_messages(ctx):
    q = ctx.upload(np.zeros((1, 3, 4, 8), np.float32))
    k = ctx.upload(np.zeros((1, 2, 4, 8), np.float32))
    with pytest.raises(AMEVAForgeShapeError, match="divisible"):
        ctx.flashAttention(q, k, k)
    big = ctx.upload(np.zeros((1, 1, 1, 264), np.float32))
    with pytest.raises(AMEVAForgeShapeError, match="256"):
        ctx.flashAttention(big, big, big)
