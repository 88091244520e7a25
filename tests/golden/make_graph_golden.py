"""Regenerate tests/golden/graph_*.npz from the reference's own Python package.

Run in a container that holds the reference checkout:

    python tests/golden/make_graph_golden.py /path/to/ameva-forge

forge-py builds its GPU graphs lazily without a GPU: tensors on device
"gpu" record nodes, and GraphBuilder (packages/forge-py/src/forge/graph.py)
turns them into the executeGraph JSON.  This script records

  * graph_llama.npz: a 2-layer GQA LlamaForCausalLM (llama.py) prefill of 3
    tokens plus one cached decode step, as ONE instruction list (the decode
    step's KV cat-append and GQA slices included), its float32 upload inputs,
    the node ids of both logits, and the logits of the same model (same seed)
    run on the reference's CPU path;
  * graph_ops.npz: layout and elementwise ops (slice with steps, cat, permute,
    transpose, broadcasting add / mul / sub / div, unary ops) with their CPU
    results.

The GPU box never needs the reference: the tests read only the .npz files.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LLAMA_SHAPE = dict(vocab_size=64, hidden_size=32, intermediate_size=48, num_hidden_layers=2, num_attention_heads=4,
                   num_key_value_heads=2)
PROMPT = [[1, 5, 9]]
NEXT = [[7]]


def _inputs_f32(inputs):
    return [np.ascontiguousarray(np.asarray(x), dtype=np.float32) for x in inputs]


def llama(forge):
    from forge.graph import GraphBuilder
    from forge.models.llama import LlamaConfig, LlamaForCausalLM

    def build(dev):
        np.random.seed(5)
        return LlamaForCausalLM(LlamaConfig(**LLAMA_SHAPE, device=dev))

    mg, mc = build("gpu"), build("cpu")
    with forge.no_grad():
        ids = np.array(PROMPT, np.int32)
        nxt = np.array(NEXT, np.int32)
        lg, kv = mg.forward(forge.ops.tensor(ids, dtype="int32", device="gpu"), use_cache=True)
        lg2, _ = mg.forward(forge.ops.tensor(nxt, dtype="int32", device="gpu"), past_key_values=kv, offset_pos=3,
                            use_cache=True)
        lc, kvc = mc.forward(forge.ops.tensor(ids, dtype="int32", device="cpu"), use_cache=True)
        lc2, _ = mc.forward(forge.ops.tensor(nxt, dtype="int32", device="cpu"), past_key_values=kvc, offset_pos=3,
                            use_cache=True)
    g = GraphBuilder()
    r1, r2 = g.add_tensor(lg), g.add_tensor(lg2)
    js, inputs = g.compile()
    out = {"json": np.frombuffer(js.encode(), np.uint8), "roots": np.array([r1, r2], np.int64),
           "logits_prefill": lc.numpy().astype(np.float32), "logits_decode": lc2.numpy().astype(np.float32)}
    for i, a in enumerate(_inputs_f32(inputs)):
        out[f"input_{i}"] = a
    out["n_inputs"] = np.array(len(inputs))
    np.savez_compressed(os.path.join(HERE, "graph_llama.npz"), **out)


def ops(forge):
    from forge.graph import GraphBuilder
    rng = np.random.default_rng(11)
    a = rng.standard_normal((2, 3, 4, 5)).astype(np.float32)
    b = rng.standard_normal((4, 1)).astype(np.float32)
    c = (rng.random((3, 4)).astype(np.float32) + 0.5)
    d = rng.standard_normal((2, 6, 4, 5)).astype(np.float32)

    def exprs(dev):
        ta, tb = forge.tensor(a, device=dev), forge.tensor(b, device=dev)
        tc, td = forge.tensor(c, device=dev), forge.tensor(d, device=dev)
        return {
            "slice_step": ta[:, 1:, ::2, ::-2],
            "slice_index": ta[1, :, 2],
            "cat_dim1": forge.ops.cat([ta, td], dim=1),
            "cat_last": forge.ops.cat([ta, ta[:, :, :, :2]], dim=3),
            "permute": forge.ops.permute(ta, (3, 1, 0, 2)),
            "transpose": forge.ops.transpose(tc),
            "add_bcast": forge.ops.add(ta, tb.reshape((1, 1, 4, 1))),
            "mul_bcast": forge.ops.mul(tc, tb.reshape((1, 4))),
            "sub": forge.ops.sub(ta, ta[:, :, ::-1, :]),
            "div": forge.ops.div(tc, tc + tc),
            "relu": forge.ops.relu(ta),
            "exp": forge.exp(tb),
            "log": forge.log(tc),
            "sigmoid": forge.ops.sigmoid(ta),
            "tanh": forge.tanh(ta),
            "neg": forge.ops.neg(tc),
        }

    with forge.no_grad():
        eg, ec = exprs("gpu"), exprs("cpu")
    g = GraphBuilder()
    roots = {k: g.add_tensor(v) for k, v in eg.items()}
    js, inputs = g.compile()
    out = {"json": np.frombuffer(js.encode(), np.uint8), "names": np.array(list(roots)),
           "roots": np.array(list(roots.values()), np.int64), "n_inputs": np.array(len(inputs))}
    for k, v in ec.items():
        out["expect_" + k] = v.numpy().astype(np.float32)
    for i, x in enumerate(_inputs_f32(inputs)):
        out[f"input_{i}"] = x
    np.savez_compressed(os.path.join(HERE, "graph_ops.npz"), **out)


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "packages", "forge-py", "src"))
    import forge
    llama(forge)
    ops(forge)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AMEVA_FORGE_REFERENCE", "")
    if not root:
        sys.exit(f"usage: python {os.path.basename(__file__)} <reference checkout root> "
                 "(or set AMEVA_FORGE_REFERENCE)")
    main(root)
