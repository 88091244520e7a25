"""Parity at the configurations the benchmarks time, against the oracle.

* The persistent decode-step kernel (k_decode_step) at the Llama-2-7B shape
  (d 128, MHA) with the KV cache filled to 4100 positions: 129 key tiles, the
  last one partial, 9 attention splits per KV head -- the split the 7B
  decode benchmark runs -- and at the TinyLlama-1.1B shape (d 64, GQA 8:1)
  at context 2048.  Two layers plus lm_head each; four greedy steps; logits
  within 2e-3 * ||ref||_inf and identical tokens (the decode tolerance of
  the north-star spec).  The cache is filled with seeded fp16 values on both
  sides (fg_llama_synthesize_kv / LlamaRef.synthesize_kv), so attention sees
  real score spreads, not a zero cache.
* The tcgen05 flash-attention prefill kernel (k_attn_tc) at the benchmark
  shape B4 H32 S4096 d128 causal, fp16 Q/K/V ~ N(0, 1): sampled (batch, head)
  pairs with every key, and query rows that include the first 16, a middle
  block and the last 16 (the longest rows, which exercise the lazy rescale
  over 32 key blocks).  Bound 2e-3 * ||ref||_inf (fp16 inputs).

The causal limit and the 1/max(l, 1e-12) normalisation follow
packages/forge/src/tensor/kernels/flash_attention.wgsl.ts:92-96, 160; the
decoder follows packages/forge-py/src/forge/models/llama.py:86-188.
"""
import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu

L7B2 = O.LlamaShape(32000, 4096, 11008, 2, 32, 32)
TINY2 = O.LlamaShape(32000, 2048, 5632, 2, 32, 4)


@pytest.mark.parametrize("name,shape,ctx_len,cap", [
    ("llama7b_2layer_ctx4100", L7B2, 4100, 4112),
    ("tinyllama_2layer_ctx2048", TINY2, 2048, 2064),
])
def test_step_kernel_vs_oracle_at_bench_context(ctx, name, shape, ctx_len, cap):
    import forge_b200
    cfg = forge_b200.LlamaConfig(max_position_embeddings=cap, max_batch=1, **shape.__dict__)
    m = forge_b200.LlamaForCausalLM(cfg, ctx)
    try:
        m.synthesize(5)
        m.synthesize_kv(77, ctx_len)
        assert m.decode_path(1) == "step"
        ref = O.LlamaRef(O.synth_llama(shape, 5), max_seq=cap, kv_f16=True)
        ref.synthesize_kv(77, ctx_len)
        tok = np.array([1234], np.int32)
        for step in range(4):
            nxt, lg = m.decode(tok, return_logits=True)
            rl = ref.forward(tok.reshape(1, 1))[:, -1]
            err = max_rel_err(lg, rl)
            assert err <= 2e-3, (step, err)
            assert int(nxt[0]) == O.argmax(rl[0]), step
            tok = nxt
        assert m.position == ctx_len + 4
    finally:
        m.close()


def test_attention_prefill_tc_bench_shape_vs_oracle(ctx):
    B, H, S, d = 4, 32, 4096, 128
    n = B * H * S * d
    q16 = O.f32_to_f16(O.normal(31, 0, n)).reshape(B, H, S, d)
    k16 = O.f32_to_f16(O.normal(32, 0, n)).reshape(B, H, S, d)
    v16 = O.f32_to_f16(O.normal(33, 0, n)).reshape(B, H, S, d)
    hq, hk, hv = (ctx.upload(t.view(np.float16)) for t in (q16, k16, v16))
    ho = ctx.flashAttention(hq, hk, hv, scale=1 / np.sqrt(d), isCausal=True)
    out = ctx.read(ho)
    ctx.dispose_batch([hq, hk, hv, ho])
    assert np.isfinite(out).all()
    for b, h in ((0, 0), (1, 17), (2, 5), (3, 31)):
        for i0, i1 in ((0, 16), (2040, 2056), (4080, 4096)):
            # rows [i0, i1) against keys [0, i1): the oracle's causal limit j < i1 - (i1 - i0) + i + 1 is the
            # full-sequence limit of row i0 + i
            q = O.f16_to_f32(q16[b:b + 1, h:h + 1, i0:i1])
            k = O.f16_to_f32(k16[b:b + 1, h:h + 1, :i1])
            v = O.f16_to_f32(v16[b:b + 1, h:h + 1, :i1])
            ref = O.attention(q, k, v, 1 / np.sqrt(d), True)
            err = max_rel_err(out[b:b + 1, h:h + 1, i0:i1], ref)
            assert err <= 2e-3, (b, h, i0, err)
