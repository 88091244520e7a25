"""Persistent decode-step kernel (one launch per token, batch 1) against the
layered per-kernel decode path and the oracle.

The layered path is selected with FORGE_B200_DECODE=layered when a model is
created.  Both paths compute the same GEMVs with the same split; attention
is split over the KV cache differently, so logits agree to fp32 rounding
(1e-4 * ||ref||_inf here) and the greedy tokens are identical.
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu

TINY2 = dict(O.LlamaShape(32000, 2048, 5632, 2, 32, 4).__dict__)   # head_dim 64, GQA 8:1
L7B1 = dict(O.LlamaShape(32000, 4096, 11008, 1, 32, 32).__dict__)  # head_dim 128, MHA
GQA4 = dict(O.LlamaShape(32000, 4096, 11008, 1, 32, 8).__dict__)   # head_dim 128, GQA 4:1 (tensor-core tiles)
GQA2 = dict(O.LlamaShape(32000, 2048, 5632, 1, 32, 16).__dict__)   # head_dim 64, GQA 2:1 (CUDA-core tiles)
GQA8D128 = dict(O.LlamaShape(32000, 4096, 11008, 1, 32, 4).__dict__)  # head_dim 128, GQA 8:1 (tensor-core tiles)
GQA4D64 = dict(O.LlamaShape(32000, 2048, 5632, 1, 32, 8).__dict__)    # head_dim 64, GQA 4:1 (tensor-core tiles)


def make(ctx, shape, seed, cap, layered=False):
    import forge_b200
    old = os.environ.pop("FORGE_B200_DECODE", None)
    if layered:
        os.environ["FORGE_B200_DECODE"] = "layered"
    try:
        cfg = forge_b200.LlamaConfig(max_position_embeddings=cap, max_batch=1, **shape)
        m = forge_b200.LlamaForCausalLM(cfg, ctx)
        m.synthesize(seed)
    finally:
        os.environ.pop("FORGE_B200_DECODE", None)
        if old is not None:
            os.environ["FORGE_B200_DECODE"] = old
    return m


@pytest.mark.parametrize("name,shape,plen", [
    ("tinyllama_2layer", TINY2, 300),   # 10 tiles of keys: 5 splits of two tiles per KV head
    ("llama7b_1layer", L7B1, 340),      # 11 tiles: 5 splits, the last of three tiles; partial last tile
    ("llama7b_1layer_short", L7B1, 5),  # one partial tile, one split
    ("gqa4_d128_1layer", GQA4, 201),    # 7 tiles, the last partial
    ("gqa4_d128_short", GQA4, 3),       # one partial tile
    ("gqa2_d64_1layer", GQA2, 100),
    ("gqa8_d128_1layer", GQA8D128, 150),
    ("gqa4_d64_1layer", GQA4D64, 97),
])
def test_step_kernel_equals_layered_decode(ctx, name, shape, plen):
    prompt = (np.arange(plen, dtype=np.int32) * 7919 % 32000).reshape(1, plen)
    a = make(ctx, shape, 11, cap=512)
    b = make(ctx, shape, 11, cap=512, layered=True)
    _, na = a.forward(prompt)
    _, nb = b.forward(prompt)
    assert na[0] == nb[0]
    for _ in range(6):
        na2, la = a.decode(na, return_logits=True)
        nb2, lb = b.decode(nb, return_logits=True)
        assert max_rel_err(la, lb) <= 1e-4
        assert na2[0] == nb2[0]
        na, nb = na2, nb2


def test_step_kernel_vs_oracle_long_context(ctx):
    shape = dict(O.LlamaShape(32000, 2048, 5632, 1, 32, 4).__dict__)
    m = make(ctx, shape, 21, cap=256)
    ref = O.LlamaRef(O.synth_llama(O.LlamaShape(**shape), 21), max_seq=256, kv_f16=True)
    prompt = (np.arange(150, dtype=np.int32) * 31 % 32000).reshape(1, 150)
    _, t = m.forward(prompt)
    ref.forward(prompt)
    for _ in range(4):
        t2, lg = m.decode(t, return_logits=True)
        rl = ref.forward(t.reshape(1, 1))[:, -1]
        assert max_rel_err(lg, rl) <= 2e-3
        t = t2


def test_step_kernel_device_generation_equals_host_loop(ctx):
    shape = dict(O.LlamaShape(32000, 2048, 5632, 1, 32, 4).__dict__)
    prompt = (np.arange(40, dtype=np.int32) * 7 % 32000).reshape(1, 40)
    a, b = make(ctx, shape, 13, cap=128), make(ctx, shape, 13, cap=128)
    _, n = a.forward(prompt)
    host = []
    for _ in range(10):
        n = a.decode(n)
        host.append(int(n[0]))
    b.forward(prompt)
    dev = b.generate_device(1, 10)
    assert dev[:, 0].tolist() == host
