"""TEST INFRASTRUCTURE ONLY -- CPU restatement of the reference's graph
executor (executeGraph, packages/forge/src/tensor/graphExecutor.ts:517-1979)
for the parity tests of fg_execute_graph.

``run_graph(instructions_json, inputs, loads)`` evaluates a GraphBuilder
instruction list (packages/forge-py/src/forge/graph.py:26-203) node by node
in numpy with each kernel's index arithmetic, calling the C primitives of
``oracle.py`` for the float kernels; ``eval_node`` evaluates one instruction
on given input arrays.  ``loads`` maps handle strings to
arrays (a quantized weight enters as its exact dequantised float32 matrix).
Only ``tests/`` may import this module.
"""
from __future__ import annotations

import json
from typing import Dict, Sequence

import numpy as np

import oracle as O


def _slice(x: np.ndarray, params, n: int) -> np.ndarray:
    """slice.wgsl.ts:77-92: coordinates from the output strides, in = sum (start + c step) in_stride."""
    rank = int(params[0])
    start = [int(v) for v in params[1:9]]
    step = [int(v) for v in params[9:17]]
    istr = [int(v) for v in params[17:25]]
    ostr = [int(v) for v in params[25:33]]
    t = np.arange(n, dtype=np.int64)
    off = np.zeros(n, dtype=np.int64)
    for i in range(rank):
        os_ = max(ostr[i], 1)
        c = t // os_
        t = t % os_
        off += (start[i] + c * step[i]) * istr[i]
    return x.reshape(-1)[off]


def _cat(a: np.ndarray, b: np.ndarray, params, n: int) -> np.ndarray:
    """cat.wgsl.ts: out[idx] from a or b along one dimension, chunk = (a_dim + b_dim) stride."""
    ad, bd, st = int(params[0]), int(params[1]), max(int(params[2]), 1)
    idx = np.arange(n, dtype=np.int64)
    chunk = (ad + bd) * st
    bi, rem = idx // chunk, idx % chunk
    di, si = rem // st, rem % st
    out = np.empty(n, dtype=np.float32)
    m = di < ad
    out[m] = a.reshape(-1)[(bi[m] * ad + di[m]) * st + si[m]]
    out[~m] = b.reshape(-1)[(bi[~m] * bd + di[~m] - ad) * st + si[~m]]
    return out


def run_graph(instructions_json: str, inputs: Sequence[np.ndarray], loads: Dict[str, np.ndarray]):
    """{id: float32 array of the node's shape} for every node."""
    nodes = json.loads(instructions_json)
    val: Dict[int, np.ndarray] = {}
    k_in = 0
    for nd in nodes:
        data = None
        if nd["op"] == "upload":
            data = inputs[k_in]
            k_in += 1
        val[nd["id"]] = eval_node(nd, [val[i] for i in nd.get("in", [])], data, loads)
    return val


def eval_node(nd, ins, upload=None, loads=None) -> np.ndarray:
    """One instruction on given input arrays (an upload takes `upload`, a load `loads[handle]`)."""
    op, shape, p = nd["op"], tuple(nd["shape"]), nd.get("params", [])
    n = int(np.prod(shape, dtype=np.int64)) if shape else 1
    if op == "upload":
        r = np.asarray(upload, dtype=np.float32).reshape(shape)
    elif op == "load":
        r = np.asarray(loads[nd["handle"]], dtype=np.float32).reshape(shape)
    elif op == "reshape":
        r = ins[0].reshape(shape)
    elif op == "transpose":  # transpose.wgsl.ts: [B][M][N] -> [B][N][M]
        M, N = int(p[0]), int(p[1])
        B = int(p[2]) if len(p) > 2 else 1
        r = ins[0].reshape(B, M, N).transpose(0, 2, 1).reshape(shape)
    elif op in ("matmul", "matmul_tiled"):
        M, N, K = int(p[0]), int(p[1]), int(p[2])
        r = O.matmul(ins[0].reshape(M, K), ins[1].reshape(K, N)).reshape(shape)
    elif op == "permute":
        r = np.ascontiguousarray(ins[0].transpose([int(d) for d in p])).reshape(shape)
    elif op == "slice":
        r = _slice(ins[0], p, n).reshape(shape)
    elif op == "cat":
        r = _cat(ins[0], ins[1], p, n).reshape(shape)
    elif op in ("add", "sub", "mul", "div"):  # broadcastParams.ts: right-aligned, size-1 dims repeat
        a, b = ins
        f = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide}[op]
        r = np.broadcast_to(f(a, b), shape).astype(np.float32)
    elif op in ("relu", "neg", "exp", "log", "sigmoid", "tanh"):
        x = ins[0].reshape(-1)[:n].astype(np.float32)
        with np.errstate(all="ignore"):
            r = {"relu": lambda v: np.maximum(v, np.float32(0)), "neg": np.negative, "exp": np.exp, "log": np.log,
                 "sigmoid": lambda v: np.float32(1) / (np.float32(1) + np.exp(-v)),
                 "tanh": np.tanh}[op](x).astype(np.float32).reshape(shape)
    elif op == "rope":
        base = float(p[0]) if len(p) > 0 else 10000.0
        off = (int(np.trunc(p[1])) % (1 << 32)) if len(p) > 1 else 0
        r = O.rope(ins[0].reshape(shape), base, off)
    elif op == "rmsnorm":
        eps = float(p[0]) if p else 1e-5
        gamma = ins[1].reshape(-1)[: shape[-1]] if len(ins) > 1 else None
        r = O.rmsnorm(ins[0].reshape(shape), gamma, eps)
    elif op == "swiglu":
        r = O.swiglu(ins[0].reshape(-1)[:n], ins[1].reshape(-1)[:n]).reshape(shape)
    elif op == "unpack_quant":
        bits = int(p[0]) if len(p) > 0 else 4
        gs = int(p[1]) if len(p) > 1 else 128
        packed = np.ascontiguousarray(ins[0], dtype=np.float32).view(np.uint32)
        r = O.unpack_quant(packed.reshape(-1), ins[1].reshape(-1), ins[2].reshape(-1), bits, gs, n).reshape(shape)
    elif op == "embedding":  # embedding.wgsl.ts:41-61: round the float index; NaN / out of range -> zero row
        vocab, dim = int(p[2]), shape[-1]
        raw = ins[1].reshape(-1)[: n // dim if dim else 0].astype(np.float32)
        rounded = np.rint(raw)
        ids = np.where(np.isnan(raw) | (rounded < 0) | (rounded >= vocab), -1, rounded).astype(np.int32)
        r = O.embedding(ins[0].reshape(-1)[: vocab * dim].reshape(vocab, dim), ids).reshape(shape)
    elif op == "flash_attention":
        B, H, Nq, d = shape
        Hkv = int(p[0]) if len(p) > 0 else H
        scale = float(p[1]) if len(p) > 1 else 1.0 / np.sqrt(d)
        causal = len(p) > 2 and p[2] == 1
        Nkv = int(p[3]) if len(p) > 3 else ins[1].shape[-2]
        r = O.attention(ins[0].reshape(shape), ins[1].reshape(B, Hkv, Nkv, d), ins[2].reshape(B, Hkv, Nkv, d),
                        scale=scale, causal=causal)
    else:
        raise NotImplementedError(op)
    return np.ascontiguousarray(r, dtype=np.float32).reshape(shape)
