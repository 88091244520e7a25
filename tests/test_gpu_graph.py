"""Graph front-end on the GPU: fg_execute_graph against the executeGraph
oracle (oracle/graph_oracle.py) and against the reference's own results on
graphs built by the reference's GraphBuilder (tests/golden/graph_*.npz), the
lazy rewrites (x W^T from W, Q4_0 W on the fused kernels, GQA head maps),
and validateInstruction's errors with transaction rollback."""
import json
import os

import numpy as np
import pytest

import graph_oracle as G
import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
LAYOUT = {"slice_step", "slice_index", "cat_dim1", "cat_last", "permute", "transpose", "neg", "relu"}


def _load(name):
    z = np.load(os.path.join(HERE, "golden", name))
    return z, bytes(z["json"]).decode(), [z[f"input_{i}"] for i in range(int(z["n_inputs"]))]


def _run(ctx, js, inputs=()):
    import forge_b200
    return forge_b200.execute_graph(ctx, js, list(inputs))


def _dispose(ctx, out, keep=()):
    hs = [h for k, h in out.items() if k not in keep]
    ctx.dispose_batch(hs)


def test_reference_llama_graph_prefill_and_decode(ctx):
    """The reference model's own 255-node graph (prefill, KV cat-append, GQA repetition, decode step)."""
    z, js, inputs = _load("graph_llama.npz")
    nodes = json.loads(js)
    _dispose(ctx, _run(ctx, js, inputs))  # first run: the context caches its RoPE frequency table
    ctx.synchronize()
    before = ctx.quota()["active"]
    out = _run(ctx, js, inputs)
    assert len(out) == len(nodes)
    ctx.synchronize()
    # lazy nodes (transposes read only by matmul, GQA slices / cats) hold no memory until read
    total = sum(4 * int(np.prod(n["shape"])) for n in nodes)
    assert ctx.quota()["active"] - before < total
    r1, r2 = (str(int(v)) for v in z["roots"])
    assert max_rel_err(ctx.read(out[r1]), z["logits_prefill"]) <= 1e-3
    assert max_rel_err(ctx.read(out[r2]), z["logits_decode"]) <= 1e-3
    # every node (lazy ones materialised on read) against the oracle applied to the node's GPU inputs:
    # bit-exact for layout and gather ops, the float tolerance for the rest
    got = {n["id"]: ctx.read(out[str(n["id"])]) for n in nodes}
    k_in = 0
    for n in nodes:
        data = None
        if n["op"] == "upload":
            data = inputs[k_in]
            k_in += 1
        ref = G.eval_node(n, [got[i] for i in n.get("in", [])], data)
        assert got[n["id"]].shape == ref.shape, n
        if n["op"] in ("upload", "reshape", "transpose", "permute", "slice", "cat", "embedding"):
            assert np.array_equal(got[n["id"]], ref), n
        else:
            assert max_rel_err(got[n["id"]], ref) <= 1e-3, n
    # and the whole chain on the CPU
    val = G.run_graph(js, inputs, {})
    for r in (r1, r2):
        assert max_rel_err(got[int(r)], val[int(r)]) <= 1e-3
    _dispose(ctx, out)
    ctx.synchronize()
    assert ctx.quota()["active"] == before


def test_reference_op_graph(ctx):
    z, js, inputs = _load("graph_ops.npz")
    out = _run(ctx, js, inputs)
    for name, root in zip(z["names"], z["roots"]):
        got, ref = ctx.read(out[str(int(root))]), z["expect_" + str(name)]
        if str(name) in LAYOUT:
            assert np.array_equal(got, ref), name
        else:
            np.testing.assert_allclose(got, ref, rtol=2e-6, atol=1e-6, err_msg=str(name))
    _dispose(ctx, out)


def _linear_graph(M, N, K, w_handle=None):
    import forge_b200
    g = forge_b200.GraphBuilder()
    x = g.add_upload((M, K))
    w = g.add_load((N, K), w_handle) if w_handle else g.add_upload((N, K))
    t = g.add_op("transpose", (K, N), [w], [N, K])
    y = g.add_op("matmul", (M, N), [x, t], [M, N, K])
    return g.compile()[0], t, y


@pytest.mark.parametrize("M", [1, 3, 40])
def test_linear_f32_reads_w_directly(ctx, M):
    rng = np.random.default_rng(M)
    N, K = 96, 64
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((N, K)).astype(np.float32)
    js, t, y = _linear_graph(M, N, K)
    out = _run(ctx, js, [x, w])
    assert max_rel_err(ctx.read(out[str(y)]), O.matmul(x, np.ascontiguousarray(w.T))) <= 1e-5
    assert np.array_equal(ctx.read(out[str(t)]), w.T)  # materialised on read
    _dispose(ctx, out)


@pytest.mark.parametrize("qt,M", [("Q4_0", 1), ("Q4_0", 4), ("Q4_0", 40), ("Q8_0", 2)])
def test_linear_quantized_weight_runs_fused_kernels(ctx, qt, M):
    qtype = O.Q4_0 if qt == "Q4_0" else O.Q8_0
    rng = np.random.default_rng(7 + M)
    N, K = 256, 512
    blocks = O.quantize(qtype, rng.standard_normal((N, K)).astype(np.float32) * 0.05)
    wh = ctx.upload_quant(qt, blocks, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    js, t, y = _linear_graph(M, N, K, wh)
    out = _run(ctx, js, [x])
    assert max_rel_err(ctx.read(out[str(y)]), O.qmatmul(qtype, blocks, N, K, x)) <= 1e-3
    assert out["2"] == wh  # the load node names the existing tensor
    assert np.array_equal(ctx.read(out[str(t)]), O.dequant(qtype, blocks, N, K).T)
    _dispose(ctx, out, keep=("2",))
    ctx.dispose(wh)


def test_lazy_transpose_survives_source_dispose(ctx):
    rng = np.random.default_rng(3)
    w = rng.standard_normal((48, 32)).astype(np.float32)
    wh = ctx.upload(w)
    x = rng.standard_normal((2, 32)).astype(np.float32)
    js, t, y = _linear_graph(2, 48, 32, wh)
    out = _run(ctx, js, [x])
    ctx.dispose(wh)  # the unread transpose takes its value first
    assert np.array_equal(ctx.read(out[str(t)]), w.T)
    _dispose(ctx, out, keep=("2",))


def test_gqa_head_maps_feed_attention(ctx):
    """k[:, h:h+1] slices and dim-1 cats (llama.py's GQA loop) into flash_attention."""
    import forge_b200
    rng = np.random.default_rng(9)
    B, H, Hkv, S, d = 2, 8, 2, 37, 64
    q = rng.standard_normal((B, H, S, d)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, S, d)).astype(np.float32)
    v = rng.standard_normal((B, Hkv, S, d)).astype(np.float32)
    g = forge_b200.GraphBuilder()
    iq, ik, iv = g.add_upload(q.shape), g.add_upload(k.shape), g.add_upload(v.shape)

    def head(src, h):
        p = [4, 0, h, 0, 0] + [0] * 4 + [1, 1, 1, 1] + [0] * 4 + [Hkv * S * d, S * d, d, 1] + [0] * 4 + \
            [S * d, S * d, d, 1] + [0] * 4
        return g.add_op("slice", (B, 1, S, d), [src], p)

    def rep(src):
        cur, n = None, 0
        for h in range(Hkv):
            s = head(src, h)
            for _ in range(H // Hkv):
                cur = s if cur is None else g.add_op("cat", (B, n + 1, S, d), [cur, s], [n, 1, S * d])
                n += 1
        return cur

    kr, vr = rep(ik), rep(iv)
    o = g.add_op("flash_attention", (B, H, S, d), [iq, kr, vr], [float(H), 1.0 / np.sqrt(d), 1.0, float(S)])
    js = g.compile()[0]
    out = _run(ctx, js, [q, k, v])
    ref = O.attention(q, k, v, causal=True)
    assert max_rel_err(ctx.read(out[str(o)]), ref) <= 1e-3
    assert np.array_equal(ctx.read(out[str(kr)]), np.repeat(k, H // Hkv, axis=1))
    _dispose(ctx, out)


def _err(ctx, js, inputs=(), cls=None):
    from forge_b200 import errors as E
    ctx.synchronize()
    before = ctx.quota()["active"]
    with pytest.raises(cls or E.AMEVAForgeError) as ei:
        _run(ctx, js, inputs)
    ctx.synchronize()
    assert ctx.quota()["active"] == before  # rollback
    return ei.value


def test_validation_errors_and_rollback(ctx):
    from forge_b200 import errors as E
    one = np.ones(4, np.float32)
    up = {"op": "upload", "id": 1, "shape": [4]}
    _err(ctx, "[{", cls=E.AMEVAForgeSecurityError)
    _err(ctx, json.dumps({"op": "upload"}), cls=E.AMEVAForgeSecurityError)
    _err(ctx, '[{"op": "upload", "id": 1, "shape": [4], "__proto__": {}}]', [one], cls=E.AMEVAForgeSecurityError)
    _err(ctx, json.dumps([{"op": "nope", "id": 1, "shape": [1]}]), cls=E.AMEVAForgeUnsupportedOpError)
    _err(ctx, json.dumps([{"op": "upload", "id": 0, "shape": [4]}]), [one], cls=E.AMEVAForgeSecurityError)
    _err(ctx, json.dumps([{"op": "upload", "id": 1, "shape": [1] * 9}]), [one], cls=E.AMEVAForgeShapeError)
    _err(ctx, json.dumps([{"op": "upload", "id": 1, "shape": [-1]}]), [one], cls=E.AMEVAForgeShapeError)
    _err(ctx, json.dumps([up, {"op": "relu", "id": 2, "shape": [4], "in": [1], "params": ["x"]}]), [one],
         cls=E.AMEVAForgeSecurityError)
    _err(ctx, json.dumps([up, {"op": "matmul", "id": 2, "shape": [4], "in": [1, 1], "params": [2, 2]}]), [one],
         cls=E.AMEVAForgeSecurityError)
    _err(ctx, json.dumps([up, {"op": "relu", "id": 2, "shape": [4], "in": [7]}]), [one], cls=E.AMEVAForgeSecurityError)
    _err(ctx, json.dumps([up]), [], cls=E.AMEVAForgeSecurityError)  # no input for the upload
    bad = one.copy()
    bad[2] = np.nan
    _err(ctx, json.dumps([up]), [bad], cls=E.AMEVAForgeValidationError)
    _err(ctx, json.dumps([up, {"op": "axpy", "id": 2, "shape": [4], "in": [1, 1], "params": [1, 1]},
                          {"op": "relu", "id": 3, "shape": [4], "in": [1]}]), [one], cls=E.AMEVAForgeSecurityError)
    _err(ctx, json.dumps([{"op": "fill", "id": 1, "shape": [4], "params": [1, 0]}]), cls=E.AMEVAForgeUnsupportedOpError)
    _err(ctx, json.dumps([{"op": "flash_attention", "id": 1, "shape": [1, 1, 1, 512], "in": [1, 1, 1]}]),
         cls=E.AMEVAForgeSecurityError)
    # rollback after work was done: three uploads, then a matmul whose operands do not fit
    g = [up, {"op": "upload", "id": 2, "shape": [4]}, {"op": "add", "id": 3, "shape": [4], "in": [1, 2]},
         {"op": "matmul", "id": 4, "shape": [2, 2], "in": [3, 3], "params": [2, 2, 3]}]
    _err(ctx, json.dumps(g), [one, one], cls=E.AMEVAForgeShapeError)
    # load of a tensor under another shape
    h = ctx.upload(one)
    _err(ctx, json.dumps([{"op": "load", "id": 1, "shape": [2, 2], "handle": h}]), cls=E.AMEVAForgeShapeError)
    ctx.dispose(h)
    _err(ctx, json.dumps([{"op": "load", "id": 1, "shape": [4], "handle": h}]), cls=E.AMEVAForgeDisposedError)


def test_runtime_limits(ctx):
    import forge_b200
    from forge_b200 import errors as E
    one = np.ones(4, np.float32)
    g = json.dumps([{"op": "upload", "id": 1, "shape": [4]}, {"op": "relu", "id": 2, "shape": [4], "in": [1]},
                    {"op": "neg", "id": 3, "shape": [4], "in": [2]}])
    forge_b200.configure_graph(ctx, max_instructions=2)
    try:
        _err(ctx, g, [one], cls=E.AMEVAForgeSecurityError)
    finally:
        forge_b200.configure_graph(ctx)
    out = _run(ctx, g, [one])
    assert np.array_equal(ctx.read(out["3"]), -one)
    _dispose(ctx, out)
    ctx.configure_runtime(allow_non_finite=True)
    try:
        bad = one.copy()
        bad[0] = np.inf
        out = _run(ctx, g, [bad])
        assert ctx.read(out["3"])[0] == -np.inf
        _dispose(ctx, out)
    finally:
        ctx.configure_runtime(allow_non_finite=False)


def test_kv_append_in_place_across_calls(ctx):
    """cat(past, new, dim=2) graphs chained through load handles: in-place appends to the newest tensor,
    a copy for an older one, and every tensor keeps its own positions."""
    import forge_b200
    rng = np.random.default_rng(21)
    B, H, S, d = 1, 2, 5, 16
    past = rng.standard_normal((B, H, S, d)).astype(np.float32)
    news = [rng.standard_normal((B, H, 1, d)).astype(np.float32) for _ in range(3)]
    q = rng.standard_normal((B, H, 1, d)).astype(np.float32)

    def step(prev_handle, prev, new, with_attn):
        g = forge_b200.GraphBuilder()
        a = g.add_load(prev.shape, prev_handle) if prev_handle else g.add_upload(prev.shape)
        b = g.add_upload(new.shape)
        n = prev.shape[2] + 1
        c = g.add_op("cat", (B, H, n, d), [a, b], [prev.shape[2], 1, d])
        ins = ([] if prev_handle else [prev]) + [new]
        o = None
        if with_attn:
            iq = g.add_upload(q.shape)
            o = g.add_op("flash_attention", (B, H, 1, d), [iq, c, c], [float(H), 1.0 / np.sqrt(d), 1.0, float(n)])
            ins.append(q)
        out = _run(ctx, g.compile()[0], ins)
        return out, out[str(c)], (out[str(o)] if o else None), np.concatenate([prev, new], axis=2)

    o1, c1, a1, r1 = step(None, past, news[0], True)
    o2, c2, a2, r2 = step(c1, r1, news[1], True)     # c1 is the store's newest: in place
    o3, c3, _, r3 = step(c1, r1, news[2], False)     # c1 again: no longer the newest, copied
    assert np.array_equal(ctx.read(c1), r1)
    assert np.array_equal(ctx.read(c2), r2)
    assert np.array_equal(ctx.read(c3), r3)
    assert max_rel_err(ctx.read(a1), O.attention(q, r1, r1, causal=True)) <= 1e-3
    assert max_rel_err(ctx.read(a2), O.attention(q, r2, r2, causal=True)) <= 1e-3
    for o, keep in ((o3, ("1",)), (o2, ("1",)), (o1, ())):
        _dispose(ctx, o, keep)


@pytest.mark.parametrize("qt", ["Q4_0", "Q8_0"])
def test_graph_llama_generate_matches_oracle(ctx, qt):
    """forge-py's model graph (GraphLlama) with GGUF weights loaded by handle: greedy tokens and logits of
    a cached generation equal the oracle model's (fp32 cache, as the reference keeps)."""
    from forge_b200.graph_llama import GraphLlama
    shape = dict(vocab_size=96, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
                 num_key_value_heads=2)
    qtype = O.Q4_0 if qt == "Q4_0" else O.Q8_0
    w = O.synth_llama(O.LlamaShape(**shape), seed=31, qtype=qtype, std=0.2)
    m = GraphLlama(ctx, **shape)
    H, I, kvd = 64, 96, 2 * 16
    dims = {"q": (H, H), "k": (kvd, H), "v": (kvd, H), "o": (H, H), "gate": (I, H), "up": (I, H), "down": (H, I)}
    handles = {"embed": ctx.upload(w.embed_f16.view(np.float16)), "norm": ctx.upload(w.norm),
               "lm_head": ctx.upload_quant(qt, w.lm_head, 96, H)}
    for l, lw in enumerate(w.layers):
        for name, (r, c) in dims.items():
            handles[f"layers.{l}.{name}"] = ctx.upload_quant(qt, lw[name], r, c)
        handles[f"layers.{l}.attn_norm"] = ctx.upload(lw["attn_norm"])
        handles[f"layers.{l}.ffn_norm"] = ctx.upload(lw["ffn_norm"])
    m.weights = handles
    # four prompt tokens: every projection runs the GEMV path, whose x digits are exact (longer prompts
    # take the tensor-core GEMM with fp16 activations; its own tolerance tests are test_gpu_qmatmul's)
    prompt = [5, 17, 33, 2]
    m.generate(prompt, 1)  # the context caches its RoPE frequency table
    ctx.synchronize()
    before = ctx.quota()["active"]
    lg = []
    toks = m.generate(prompt, 4, lg)
    ctx.synchronize()
    assert ctx.quota()["active"] == before  # every graph tensor and cache store was released
    ref = O.LlamaRef(w, max_seq=16, kv_f16=False)
    ids = np.array([prompt], np.int32)
    want = []
    for step in range(4):
        logits = ref.forward(ids)[0, -1]
        assert max_rel_err(lg[step], logits) <= 1e-3, step
        want.append(O.argmax(logits))
        ids = np.array([[want[-1]]], np.int32)
    assert toks == prompt + want
    ctx.dispose_batch(list(handles.values()))
