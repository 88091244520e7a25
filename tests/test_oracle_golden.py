"""Pins the CPU oracle to the reference: every fixture in tests/golden was
produced by the reference's own code (forge-py CPU path) or, for the unpack
known answers, by the input formulas of the reference's unpack test."""
import numpy as np
import pytest

import inputs as I
import oracle as O


def test_unpack_int4_known_answer(golden):
    packed, scales, zeros, bits, gs, n = I.unpack4()
    out = O.unpack_quant(packed, scales, zeros, bits, gs, n)
    assert out.view(np.uint32).tolist() == golden["unpack4_expected"].view(np.uint32).tolist()


def test_unpack_int8_known_answer(golden):
    packed, scales, zeros, bits, gs, n = I.unpack8()
    out = O.unpack_quant(packed, scales, zeros, bits, gs, n)
    assert np.array_equal(out.view(np.uint32), golden["unpack8_expected"].view(np.uint32))


def test_rmsnorm_matches_reference(golden):
    x, g = I.rmsnorm()
    np.testing.assert_allclose(O.rmsnorm(x, g, 1e-5), golden["rmsnorm_out"], rtol=1e-5, atol=1e-6)
    x, g = I.rmsnorm_small()
    np.testing.assert_allclose(O.rmsnorm(x, g, 1e-5), golden["rmsnorm2_out"], rtol=1e-5, atol=1e-6)


def test_rope_matches_reference(golden):
    # forge-py evaluates theta, cos and sin in fp32; the oracle rounds theta to fp32 then
    # takes cos/sin in double: agreement is at fp32 rounding level
    np.testing.assert_allclose(O.rope(I.rope(), 10000.0, 0), golden["rope_out"], atol=1e-5)
    # offset 2047: theta is ~2e3 rad, so one fp32 ulp of theta moves cos/sin by ~1e-4
    np.testing.assert_allclose(O.rope(I.rope_offset(), 10000.0, 2047), golden["rope_off_out"], atol=5e-4)


def test_swiglu_matches_reference(golden):
    gt, up = I.swiglu()
    np.testing.assert_allclose(O.swiglu(gt, up), golden["swiglu_out"], rtol=1e-6, atol=1e-6)


def test_attention_matches_reference(golden):
    q, k, v = I.mha()
    np.testing.assert_allclose(O.attention(q, k, v, causal=False), golden["mha_out"], atol=1e-5)
    q, k, v = I.gqa()
    np.testing.assert_allclose(O.attention(q, k, v, causal=True), golden["gqa_out"], atol=1e-5)


@pytest.mark.parametrize("shape", I.MATMUL_SHAPES)
def test_matmul_matches_reference(golden, shape):
    M, K, N = shape
    A, B = I.matmul(M, K, N)
    np.testing.assert_allclose(O.matmul(A, B), golden[f"matmul_{M}x{K}x{N}"], atol=1e-4, rtol=1e-4)


def test_greedy_pick():
    assert O.argmax(I.GREEDY_LOGITS) == I.GREEDY_INDEX
    assert O.argmax(np.array([3.0, 7.0, 7.0, 1.0], np.float32)) == 1  # first max wins


def test_llama_matches_reference_model(golden):
    """Oracle Llama (fp32 cache) vs the reference's LlamaForCausalLM on the
    same dequantised weights: prefill logits, then greedy decode steps."""
    w = O.synth_llama(O.LlamaShape(**I.LLAMA_SHAPE), seed=I.LLAMA_SEED)
    ref = O.LlamaRef(w, max_seq=32, kv_f16=False)
    lg = ref.forward(I.LLAMA_PROMPT)
    gl = golden["llama_prefill_logits"]
    assert np.abs(lg - gl).max() <= 1e-4 * np.abs(gl).max()
    toks = [O.argmax(lg[0, -1])]
    for step in range(1, I.LLAMA_STEPS):
        lg = ref.forward(np.array([[toks[-1]]], np.int32))
        sl = golden["llama_step_logits"][step]
        assert np.abs(lg[0, -1] - sl).max() <= 1e-4 * np.abs(sl).max()
        toks.append(O.argmax(lg[0, -1]))
    assert toks == golden["llama_tokens"].tolist()


def test_q4_0_gguf_mapping_is_exact():
    """GGUF dequant == reference unpack over the mapped operands, bit for bit."""
    w = O.normal(77, 0, 64 * 256, 0.0, 0.02).reshape(64, 256)
    for qt in (O.Q4_0, O.Q8_0):
        blocks = O.quantize(qt, w)
        packed, scales, zeros = O.gguf_to_ref(qt, blocks)
        ref = O.unpack_quant(packed, scales, zeros, 4 if qt == O.Q4_0 else 8, 32, w.size)
        deq = O.dequant(qt, blocks, 64, 256).reshape(-1)
        assert np.array_equal(ref.view(np.uint32), deq.view(np.uint32))
        assert np.abs(deq - w.reshape(-1)).max() <= np.abs(w).max() / (7 if qt == O.Q4_0 else 100)


def test_f16_conversion_matches_numpy():
    x = np.concatenate([O.normal(5, 0, 100000, 0, 3.0), O.normal(6, 0, 1000, 0, 1e-6),
                        np.array([65504, 65520, 1e5, -0.0, 6e-8, 3e-8, 2.98e-8], np.float32)])
    assert np.array_equal(O.f32_to_f16(x), x.astype(np.float16).view(np.uint16))
    h = np.arange(0, 65536, dtype=np.uint16)
    h = h[(h & 0x7C00) != 0x7C00]
    assert np.array_equal(O.f16_to_f32(h), h.view(np.float16).astype(np.float32))
