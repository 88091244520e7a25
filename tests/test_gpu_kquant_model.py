"""A k-quant Llama (the type mix of a llama.cpp Q4_K_M file: Q4_K Linears, Q6_K for attn_v, ffn_down and
the output matrix) through the model API against the oracle.

The prompt (20 tokens) runs every Linear as bit-exact dequantisation plus the fp32 matmul (tcgen05 tf32
with the three-term split where the product is large enough, the SIMT kernel below that); the decode
steps run the k-quant GEMVs, whose outputs then pass through the layered path's epilogues (RoPE + fp16
KV append, SwiGLU, residual add).  Logits within 2e-3 * ||ref||_inf, identical greedy tokens
(the decoder of packages/forge-py/src/forge/models/llama.py:86-188)."""
import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu

SHAPE = O.LlamaShape(512, 256, 512, 2, 4, 2)  # k-quant widths: multiples of 256


def _load(m, w):
    m.load("embed", w.embed_f16)
    m.load("norm", w.norm)
    m.load("lm_head", w.lm_head[1])
    for l, L in enumerate(w.layers):
        m.load("attn_norm", L["attn_norm"], l)
        m.load("ffn_norm", L["ffn_norm"], l)
        for name in ("q", "k", "v", "o", "gate", "up", "down"):
            m.load(name, L[name][1], l)


def test_kquant_model_prefill_and_decode_vs_oracle(ctx):
    import forge_b200
    cfg = forge_b200.LlamaConfig(max_position_embeddings=64, max_batch=1, qtype="Q4_K", **SHAPE.__dict__)
    m = forge_b200.LlamaForCausalLM(cfg, ctx)
    try:
        w = O.kquant_llama(SHAPE, 7)
        _load(m, w)
        assert m.decode_path(1) == "layered"
        ref = O.LlamaRef(w, max_seq=64)
        prompt = (np.arange(20, dtype=np.int32) * 37 % 512).reshape(1, 20)
        lg, nxt = m.forward(prompt)
        rl = ref.forward(prompt)[:, -1]
        assert max_rel_err(lg, rl) <= 2e-3
        assert int(nxt[0]) == O.argmax(rl[0])
        for _ in range(4):
            n2, lg2 = m.decode(nxt, return_logits=True)
            rl2 = ref.forward(nxt.reshape(1, 1))[:, -1]
            assert max_rel_err(lg2, rl2) <= 2e-3
            assert int(n2[0]) == O.argmax(rl2[0])
            nxt = n2
    finally:
        m.close()


def test_kquant_model_rejects_wrong_block_bytes(ctx):
    import forge_b200
    from forge_b200.errors import AMEVAForgeShapeError
    cfg = forge_b200.LlamaConfig(max_position_embeddings=16, max_batch=1, qtype="Q4_K", **SHAPE.__dict__)
    m = forge_b200.LlamaForCausalLM(cfg, ctx)
    try:
        with pytest.raises(AMEVAForgeShapeError, match="Q4_K"):
            m.load("q", np.zeros(1000, np.uint8), 0)  # neither Q4_K nor Q6_K bytes of [256, 256]
    finally:
        m.close()


def test_kquant_gguf_file_loads_as_kquant_model(ctx, tmp_path):
    """A Q4_K_M-style GGUF file: the config reports a k-quant model, every Q4_K / Q6_K Linear loads, and
    the model gives the oracle's logits."""
    import forge_b200
    from gguf_write import write_llama
    w = O.kquant_llama(SHAPE, 9)
    path = str(tmp_path / "kq.gguf")
    write_llama(path, w)
    m = forge_b200.LlamaForCausalLM.from_gguf(path, ctx, max_position_embeddings=64)
    try:
        assert m.config.qtype == "Q4_K"
        ref = O.LlamaRef(w, max_seq=64)
        prompt = (np.arange(7, dtype=np.int32) * 11 % 512).reshape(1, 7)
        lg, _ = m.forward(prompt)
        assert max_rel_err(lg, ref.forward(prompt)[:, -1]) <= 2e-3
    finally:
        m.close()
