"""Graph front-end: the JSON graph contract of forge-py's GraphBuilder
(packages/forge-py/src/forge/graph.py:26-203) and its executor
(executeGraph, packages/forge/src/tensor/graphExecutor.ts:487-1979), here
over libforge_b200's fg_execute_graph.

``GraphBuilder`` records nodes exactly as the reference's builder does (same
op allow-list, same shape and id checks, same JSON); ``execute_graph`` is the
bridge call (forge-py bridge.py:229-264): it returns ``{str(node_id):
"tensor_<hex>"}`` for every node, and raises the reference's typed errors.
Loaded tensors may be float32, float16 or GGUF Q4_0 / Q8_0 weights; a
``transpose`` of a quantized weight feeding ``matmul`` runs the fused
dequant GEMV / tensor-core GEMM.
"""
from __future__ import annotations

import ctypes
import json
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _capi as C
from .errors import AMEVAForgeSecurityError, AMEVAForgeValidationError

# forge-py graph.py:16-24
ALLOWED_OPS_WHITELIST = frozenset([
    'upload', 'load', 'matmul', 'matmul_tiled', 'batched_matmul', 'relu', 'add', 'mul', 'transpose',
    'relu_backward', 'sub', 'neg', 'div', 'exp', 'log', 'sigmoid', 'tanh', 'sigmoid_backward', 'tanh_backward',
    'fill', 'sum', 'max', 'sum_axis', 'max_axis', 'max_axis_backward', 'axpy', 'cat', 'where', 'pad', 'gather',
    'scatter', 'maxpool2d', 'avgpool2d', 'im2col', 'col2im', 'dropout', 'permute', 'matmul_bias_relu', 'reshape',
    'slice', 'slice_backward', 'reduce_axes', 'flash_attention', 'rope', 'rmsnorm', 'swiglu', 'unpack_quant',
    'embedding', 'embedding_backward', 'adam_step', 'sgd_momentum_step', 'sparse_cross_entropy',
    'sparse_cross_entropy_backward', 'mse_loss', 'mse_loss_backward'
])


def _clean_shape(shape) -> List[int]:
    if not isinstance(shape, (tuple, list)):
        raise TypeError(f"Shape must be a tuple or list of ints, got {type(shape)}")
    out = []
    for d in shape:
        if not isinstance(d, (int, np.integer)) or int(d) < 0:
            raise ValueError(f"Shape dimensions must be non-negative integers, got {d}")
        out.append(int(d))
    if len(out) > 8:
        raise ValueError(f"Shape dimensions cannot exceed 8, got {len(out)}")
    return out


class GraphBuilder:
    """Records graph nodes in order (forge-py graph.py:26-203)."""

    def __init__(self):
        self.nodes: List[Dict[str, Any]] = []
        self.inputs: List[Any] = []
        self.next_id = 1

    def alloc_id(self) -> int:
        idx = self.next_id
        self.next_id += 1
        return idx

    def add_upload(self, shape: Sequence[int], data: Any = None) -> int:
        clean = _clean_shape(shape)
        nid = self.alloc_id()
        self.nodes.append({"op": "upload", "id": nid, "shape": clean})
        if data is not None:
            self.inputs.append(data)
        return nid

    def add_load(self, shape: Sequence[int], handle: str) -> int:
        if not isinstance(handle, str) or not handle.strip():
            raise ValueError(f"Handle must be a non-empty string, got {handle}")
        if not isinstance(shape, (tuple, list)):
            raise TypeError(f"Shape must be a tuple or list of ints, got {type(shape)}")
        nid = self.alloc_id()
        self.nodes.append({"op": "load", "id": nid, "shape": [int(d) for d in shape], "handle": handle})
        return nid

    def add_op(self, op_name: str, shape: Sequence[int], in_ids: List[int], params: Optional[List[Any]] = None) -> int:
        if not isinstance(op_name, str) or not op_name.strip():
            raise AMEVAForgeValidationError(f"[AMEVA-Forge Error] op_name must be a valid non-empty string, got: {op_name}")
        if op_name not in ALLOWED_OPS_WHITELIST:
            raise AMEVAForgeSecurityError(
                f"[AMEVA-Forge Security Alert] Prohibited, unrecognized, or unregistered op '{op_name}' detected in "
                f"computation graph. Execution halted to protect runtime integrity.")
        clean = _clean_shape(shape)
        ins = []
        for i in in_ids:
            if not isinstance(i, (int, np.integer)) or int(i) <= 0:
                raise ValueError(f"in_ids must contain positive integers, got {i}")
            ins.append(int(i))
        nid = self.alloc_id()
        node: Dict[str, Any] = {"op": op_name, "id": nid, "shape": clean, "in": ins}
        if params is not None:
            cp = []
            for p in params:
                if isinstance(p, bool):
                    cp.append(p)
                elif isinstance(p, (float, np.floating)):
                    cp.append(float(p))
                elif isinstance(p, (int, np.integer)):
                    cp.append(int(p))
                else:
                    cp.append(p)
            node["params"] = cp
        self.nodes.append(node)
        return nid

    def add_trusted(self, op_name: str, shape, in_ids, params=None) -> int:
        """add_op for emitters whose arguments are already plain ints / floats of an allowed op
        (GraphLlama): the same node, without the per-element checks."""
        nid = self.next_id
        self.next_id += 1
        node: Dict[str, Any] = {"op": op_name, "id": nid, "shape": list(shape), "in": list(in_ids)}
        if params is not None:
            node["params"] = list(params)
        self.nodes.append(node)
        return nid

    def to_dict(self) -> Dict[str, Any]:
        return {"instructions": self.nodes, "inputs": self.inputs}

    def compile(self) -> Tuple[str, List[Any]]:
        return json.dumps(self.nodes), self.inputs


def execute_graph(ctx, instructions_json: str, inputs: Optional[Sequence[Any]] = None) -> Dict[str, str]:
    """executeGraph(json, inputs) -> {str(id): handle}; inputs are float32 arrays, one per upload node."""
    arrays = []
    for a in inputs or []:
        if hasattr(a, "dtype") and str(a.dtype) != "float32":
            raise TypeError(f"Expected float32, got {a.dtype}")  # bridge.py:236-239
        arrays.append(np.ascontiguousarray(a, dtype=np.float32))
    n_in = len(arrays)
    ptrs = (ctypes.c_void_p * max(1, n_in))(*[a.ctypes.data for a in arrays])
    sizes = (ctypes.c_uint64 * max(1, n_in))(*[a.nbytes for a in arrays])
    js = instructions_json.encode("utf-8") if isinstance(instructions_json, str) else instructions_json
    # every node has an "op" key: the count bounds the node count (the library reports the exact count
    # without running anything when the arrays are too small, and the call is repeated once)
    cap = max(1, js.count(b'"op"'))
    n_out = ctypes.c_int32(0)
    for _ in range(2):
        ids = (ctypes.c_int64 * cap)()
        hs = (ctypes.c_uint64 * cap)()
        st = C.lib().fg_execute_graph(ctx.ptr, js, ptrs, sizes, n_in, ids, hs, cap, ctypes.byref(n_out))
        if st == 0 or n_out.value <= cap:
            break
        cap = n_out.value
    C.check(st)
    return {str(ids[i]): "tensor_%016x" % hs[i] for i in range(n_out.value)}


executeGraph = execute_graph


def configure_graph(ctx, max_instructions: int = 10000, max_shape_dim: int = 8, max_elements: int = 256 * 1024 * 1024):
    """configureRuntime's graph limits (graphExecutor.ts:98-127)."""
    C.call("fg_configure_graph", ctx.ptr, max_instructions, max_shape_dim, max_elements)
