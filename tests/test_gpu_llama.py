"""Llama decode path on the GPU vs the oracle's restatement of
LlamaForCausalLM (llama.py:69-248) on identical synthetic Q4_0 weights."""
import numpy as np
import pytest

import inputs as I
import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3  # relative to ||ref||_inf, after 2+ layers of fp32 GEMV + fp16 KV


def make(ctx, shape, seed, cap=256, max_batch=1, qtype="Q4_0", load_from_host=None):
    import forge_b200
    cfg = forge_b200.LlamaConfig(max_position_embeddings=cap, max_batch=max_batch, qtype=qtype, **shape)
    m = forge_b200.LlamaForCausalLM(cfg, ctx)
    if load_from_host is None:
        m.synthesize(seed)
    else:
        w = load_from_host
        m.load("embed", w.embed_f16)
        m.load("norm", w.norm)
        m.load("lm_head", w.lm_head)
        for li, L in enumerate(w.layers):
            for name, arr in L.items():
                m.load(name, arr, li)
    return m


def oracle_model(shape, seed, cap=256, qtype=O.Q4_0):
    return O.LlamaRef(O.synth_llama(O.LlamaShape(**shape), seed, qtype), max_seq=cap, kv_f16=True)


def test_tiny_matches_oracle_and_reference(ctx, golden):
    """The reference-model fixture: GPU (fp16 KV) vs oracle (fp16 KV) tightly,
    and vs the reference's own fp32-KV logits within the fp16-cache error."""
    m = make(ctx, I.LLAMA_SHAPE, I.LLAMA_SEED)
    ref = oracle_model(I.LLAMA_SHAPE, I.LLAMA_SEED)
    lg, nxt = m.forward(I.LLAMA_PROMPT)
    rl = ref.forward(I.LLAMA_PROMPT)[:, -1]
    assert max_rel_err(lg, rl) <= LOGIT_TOL
    assert max_rel_err(lg[0], golden["llama_prefill_logits"][0, -1]) <= 5e-3
    toks = [int(nxt[0])]
    for step in range(1, I.LLAMA_STEPS):
        n2, lg2 = m.decode(np.array([toks[-1]], np.int32), return_logits=True)
        rl2 = ref.forward(np.array([[toks[-1]]], np.int32))[:, -1]
        assert max_rel_err(lg2, rl2) <= LOGIT_TOL
        assert max_rel_err(lg2[0], golden["llama_step_logits"][step]) <= 5e-3
        toks.append(int(n2[0]))
    assert toks == golden["llama_tokens"].tolist()


def test_host_loaded_weights_equal_synthesized(ctx):
    shape = dict(I.LLAMA_SHAPE)
    w = O.synth_llama(O.LlamaShape(**shape), 77)
    a = make(ctx, shape, 77)
    b = make(ctx, shape, 0, load_from_host=w)
    la, _ = a.forward(I.LLAMA_PROMPT)
    lb, _ = b.forward(I.LLAMA_PROMPT)
    assert np.array_equal(la, lb)


@pytest.mark.parametrize("name,shape", [
    ("tinyllama_2layer", dict(O.LlamaShape(32000, 2048, 5632, 2, 32, 4).__dict__)),
    ("llama7b_1layer", dict(O.LlamaShape(32000, 4096, 11008, 1, 32, 32).__dict__)),
])
def test_full_width_layers_vs_oracle(ctx, name, shape):
    """Full TinyLlama / Llama-2-7B layer widths (head_dim 64 GQA 8:1 and
    head_dim 128 MHA), prefill of 40 tokens then 3 decode steps."""
    m = make(ctx, shape, 5, cap=128)
    ref = oracle_model(shape, 5, cap=128)
    prompt = (np.arange(40, dtype=np.int32) * 7919 % 32000).reshape(1, 40)
    lg, nxt = m.forward(prompt)
    rl = ref.forward(prompt)[:, -1]
    assert max_rel_err(lg, rl) <= LOGIT_TOL
    t = nxt
    for _ in range(3):
        t2, lg2 = m.decode(t, return_logits=True)
        rl2 = ref.forward(t.reshape(1, 1))[:, -1]
        assert max_rel_err(lg2, rl2) <= LOGIT_TOL
        t = t2


def test_q8_0_model_vs_oracle(ctx):
    m = make(ctx, I.LLAMA_SHAPE, 9, qtype="Q8_0")
    ref = oracle_model(I.LLAMA_SHAPE, 9, qtype=O.Q8_0)
    lg, _ = m.forward(I.LLAMA_PROMPT)
    assert max_rel_err(lg, ref.forward(I.LLAMA_PROMPT)[:, -1]) <= LOGIT_TOL


def test_chunked_prefill_equals_single_prefill(ctx):
    shape = dict(I.LLAMA_SHAPE)
    prompt = (np.arange(100, dtype=np.int32) * 13 % 96).reshape(1, 100)
    a = make(ctx, shape, 3)
    la, na = a.forward(prompt)
    b = make(ctx, shape, 3)
    b.forward(prompt[:, :37], return_logits=False)
    b.forward(prompt[:, 37:70], return_logits=False)
    lb, nb = b.forward(prompt[:, 70:])
    assert max_rel_err(lb, la) <= 1e-4 and nb[0] == na[0]


def test_graph_decode_equals_eager_forward(ctx):
    shape = dict(I.LLAMA_SHAPE)
    a, b = make(ctx, shape, 4), make(ctx, shape, 4)
    _, na = a.forward(I.LLAMA_PROMPT)
    _, nb = b.forward(I.LLAMA_PROMPT)
    for _ in range(4):
        la, na2 = a.forward(na.reshape(1, 1))          # eager, T == 1
        nb2, lb = b.decode(nb, return_logits=True)      # CUDA graph
        assert np.array_equal(la, lb) and na2[0] == nb2[0]
        na, nb = na2, nb2


def test_device_generation_equals_host_loop(ctx):
    shape = dict(I.LLAMA_SHAPE)
    a, b = make(ctx, shape, 6), make(ctx, shape, 6)
    _, n = a.forward(I.LLAMA_PROMPT)
    host = []
    for _ in range(12):
        n = a.decode(n)
        host.append(int(n[0]))
    b.forward(I.LLAMA_PROMPT)
    dev = b.generate_device(1, 12)
    assert dev[:, 0].tolist() == host


@pytest.mark.parametrize("B", [2, 5])
def test_batched_decode_matches_single_sequences(ctx, B):
    """B sequences decoded together (GEMV for B <= 4, GEMM beyond) equal the
    same sequences decoded alone."""
    shape = dict(I.LLAMA_SHAPE)
    prompts = (np.arange(B * 8, dtype=np.int32).reshape(B, 8) * 17 + 3) % 96
    mb = make(ctx, shape, 8, max_batch=B)
    _, nb = mb.forward(prompts)
    seqs_b = [nb.copy()]
    for _ in range(3):
        nb = mb.decode(nb)
        seqs_b.append(nb.copy())
    for s in range(B):
        m1 = make(ctx, shape, 8)
        _, n1 = m1.forward(prompts[s:s + 1])
        seq = [int(n1[0])]
        for _ in range(3):
            n1 = m1.decode(n1)
            seq.append(int(n1[0]))
        assert seq == [int(x[s]) for x in seqs_b]


def test_generate_api(ctx):
    m = make(ctx, I.LLAMA_SHAPE, I.LLAMA_SEED)
    out = m.generate(list(I.LLAMA_PROMPT[0]), max_new_tokens=I.LLAMA_STEPS)
    assert out[len(I.LLAMA_PROMPT[0]):] == [int(t) for t in np.asarray(O.LlamaRef(
        O.synth_llama(O.LlamaShape(**I.LLAMA_SHAPE), I.LLAMA_SEED), 64).generate(I.LLAMA_PROMPT, I.LLAMA_STEPS)[0][0])]
