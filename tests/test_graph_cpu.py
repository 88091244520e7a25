"""Graph front-end, CPU side: the executeGraph oracle is pinned to the
reference (graph fixtures built by forge-py's own GraphBuilder, expected
values from forge-py's CPU path), and forge_b200.GraphBuilder emits the
reference builder's JSON."""
import json
import os

import numpy as np
import pytest

import graph_oracle as G

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(name):
    z = np.load(os.path.join(HERE, "golden", name))
    js = bytes(z["json"]).decode()
    inputs = [z[f"input_{i}"] for i in range(int(z["n_inputs"]))]
    return z, js, inputs


def test_oracle_runs_reference_llama_graph():
    z, js, inputs = _load("graph_llama.npz")
    val = G.run_graph(js, inputs, {})
    r1, r2 = (int(v) for v in z["roots"])
    np.testing.assert_allclose(val[r1], z["logits_prefill"], rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(val[r2], z["logits_decode"], rtol=2e-5, atol=2e-5)


def test_oracle_runs_reference_op_graph():
    z, js, inputs = _load("graph_ops.npz")
    val = G.run_graph(js, inputs, {})
    for name, root in zip(z["names"], z["roots"]):
        np.testing.assert_allclose(val[int(root)], z["expect_" + str(name)], rtol=1e-6, atol=1e-6, err_msg=str(name))


def test_builder_matches_reference_json_contract():
    import forge_b200
    g = forge_b200.GraphBuilder()
    a = g.add_upload((2, 3), np.ones((2, 3), np.float32))
    w = g.add_load((4, 3), "tensor_0000010000000001")
    t = g.add_op("transpose", (3, 4), [w], [4, 3])
    m = g.add_op("matmul", (2, 4), [a, t], [2, 4, 3])
    js, inputs = g.compile()
    assert json.loads(js) == [
        {"op": "upload", "id": 1, "shape": [2, 3]},
        {"op": "load", "id": 2, "shape": [4, 3], "handle": "tensor_0000010000000001"},
        {"op": "transpose", "id": 3, "shape": [3, 4], "in": [2], "params": [4, 3]},
        {"op": "matmul", "id": 4, "shape": [2, 4], "in": [1, 3], "params": [2, 4, 3]}]
    assert len(inputs) == 1 and m == 4


def test_builder_rejects_like_reference():
    import forge_b200
    from forge_b200.errors import AMEVAForgeSecurityError, AMEVAForgeValidationError
    g = forge_b200.GraphBuilder()
    with pytest.raises(AMEVAForgeSecurityError):
        g.add_op("__proto__", (1,), [1])
    with pytest.raises(AMEVAForgeValidationError):
        g.add_op("", (1,), [1])
    with pytest.raises(ValueError):
        g.add_upload((1,) * 9)
    with pytest.raises(ValueError):
        g.add_op("relu", (2,), [0])


def test_graph_llama_emits_the_reference_graph():
    """forge_b200.graph_llama.GraphLlama reproduces forge-py's LlamaForCausalLM graph node for node
    (prefill of 3 tokens + one cached decode step, weights as uploads on first use)."""
    import make_graph_golden as M
    from forge_b200.graph import GraphBuilder
    from forge_b200.graph_llama import GraphLlama
    z, js, inputs = _load("graph_llama.npz")
    m = GraphLlama(None, **M.LLAMA_SHAPE)
    m.weights = {n: np.zeros(m.weight_shape(n), np.float32) for n in m.weight_names()}
    g = GraphBuilder()
    nodes = {}
    l1, _, present = m.forward(g, nodes, np.array(M.PROMPT), 0)
    l2, _, _ = m.forward(g, nodes, np.array(M.NEXT), 3, present)
    assert json.loads(g.compile()[0]) == json.loads(js)
    assert [l1, l2] == [int(v) for v in z["roots"]]
