"""forge-py's LlamaForCausalLM (packages/forge-py/src/forge/models/llama.py:
45-248) as the executeGraph instruction lists its lazy tensors produce.

``GraphLlama`` emits, node for node and in the same order, the graph that
forge-py's GraphBuilder records for ``forward(input_ids, past_key_values,
offset_pos)``: embedding, per layer RMSNorm, the q/k/v ``nn.Linear``s as
reshape -> transpose(W) -> matmul -> reshape, head split by reshape +
permute, RoPE, the KV cat-append, the GQA head repetition (slices and a left
fold of dim-1 cats), flash_attention, the o/gate/up/down projections, SwiGLU,
the residual adds, the final norm and lm_head.  Weights enter as ``load``
nodes of library handles (Q4_0 / Q8_0 matrices run the fused kernels), or as
``upload`` nodes on their first use as forge-py does for fresh parameters.

``generate`` is llama.py's cached greedy loop (:211-248): one graph per
token, logits read back and arg-maxed on the host, the present keys/values
kept as handles that the next graph loads.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from .graph import GraphBuilder, execute_graph


class GraphLlama:
    LAYER_WEIGHTS = ("attn_norm", "q", "k", "v", "o", "ffn_norm", "gate", "up", "down")

    def __init__(self, ctx, vocab_size: int, hidden_size: int, intermediate_size: int, num_hidden_layers: int,
                 num_attention_heads: int, num_key_value_heads: int, rms_norm_eps: float = 1e-5,
                 rope_theta: float = 10000.0, weights: Optional[Dict[str, object]] = None, **_):
        self.ctx = ctx
        self.V, self.H, self.I = vocab_size, hidden_size, intermediate_size
        self.L, self.Hq, self.Hkv = num_hidden_layers, num_attention_heads, num_key_value_heads
        self.hd = hidden_size // num_attention_heads
        self.G = self.Hq // self.Hkv
        self.eps, self.theta = float(rms_norm_eps), float(rope_theta)
        # name -> handle string (load node) or float32 array (upload node on first use)
        self.weights: Dict[str, object] = dict(weights or {})

    # ------------------------------------------------------------ weight shapes
    def weight_shape(self, name: str) -> Tuple[int, ...]:
        H, I, V, kvd = self.H, self.I, self.V, self.Hkv * self.hd
        if name == "embed":
            return (V, H)
        if name == "norm":
            return (H,)
        if name == "lm_head":
            return (V, H)
        kind = name.split(".")[-1]
        return {"attn_norm": (H,), "ffn_norm": (H,), "q": (H, H), "k": (kvd, H), "v": (kvd, H), "o": (H, H),
                "gate": (I, H), "up": (I, H), "down": (H, I)}[kind]

    def weight_names(self) -> List[str]:
        names = ["embed"]
        for l in range(self.L):
            names += [f"layers.{l}.{k}" for k in self.LAYER_WEIGHTS]
        return names + ["norm", "lm_head"]

    # ------------------------------------------------------------ emitters
    def _w(self, g: GraphBuilder, nodes: Dict[str, int], name: str) -> int:
        if name not in nodes:
            w = self.weights[name]
            shape = self.weight_shape(name)
            if isinstance(w, str):
                nodes[name] = g.add_load(shape, w)
            else:
                nodes[name] = g.add_upload(shape, np.ascontiguousarray(w, dtype=np.float32))
        return nodes[name]

    def _linear(self, g, nodes, x: int, x_shape: Tuple[int, ...], wname: str) -> Tuple[int, Tuple[int, ...]]:
        """nn.Linear (nn.py:248-259) through forge matmul (ops.py:495-507): flatten, x @ W^T, restore."""
        N, K = self.weight_shape(wname)
        lead = tuple(x_shape[:-1])
        flat = int(np.prod(lead))
        a2 = g.add_trusted("reshape", (flat, K), [x], [flat, K])
        w = self._w(g, nodes, wname)
        t = g.add_trusted("transpose", (K, N), [w], [N, K])
        m = g.add_trusted("matmul", (flat, N), [a2, t], [flat, N, K])
        out_shape = lead + (N,)
        return g.add_trusted("reshape", out_shape, [m], list(out_shape)), out_shape

    def _heads(self, g, x: int, B: int, L: int, nh: int) -> int:
        r = g.add_trusted("reshape", (B, L, nh, self.hd), [x], [B, L, nh, self.hd])
        return g.add_trusted("permute", (B, nh, L, self.hd), [r], [0, 2, 1, 3])

    def _head_slice(self, g, src: int, B: int, S: int, h: int) -> int:
        """k[:, h:h+1, :, :] (ops.py:2340-2395 params: rank, starts, steps, in/out strides, each padded to 8)."""
        hd, Hkv = self.hd, self.Hkv
        pad = [0] * 4
        params = ([4] + [0, h, 0, 0] + pad + [1, 1, 1, 1] + pad + [Hkv * S * hd, S * hd, hd, 1] + pad +
                  [S * hd, S * hd, hd, 1] + pad)
        return g.add_trusted("slice", (B, 1, S, hd), [src], params)

    def _repeat(self, g, src: int, B: int, S: int) -> int:
        """llama.py:116-127: every KV head G times, concatenated on dim 1 (a left fold of binary cats)."""
        if self.G == 1:
            return src
        cur, n = None, 0
        for h in range(self.Hkv):
            s = self._head_slice(g, src, B, S, h)
            for _ in range(self.G):
                if cur is None:
                    cur, n = s, 1
                else:
                    cur = g.add_trusted("cat", (B, n + 1, S, self.hd), [cur, s], [n, 1, S * self.hd])
                    n += 1
        return cur

    def forward(self, g: GraphBuilder, nodes: Dict[str, int], ids: np.ndarray, offset: int,
                past: Optional[Sequence[Tuple[int, int, int]]] = None):
        """Emit one forward; past = [(k node, v node, cached length)] per layer.  Returns
        (logits node, logits shape, present [(k node, v node, length)])."""
        B, L = ids.shape
        H, hd = self.H, self.hd
        emb = self._w(g, nodes, "embed")
        idn = g.add_upload((B, L), np.ascontiguousarray(ids, dtype=np.float32))
        h = g.add_trusted("embedding", (B, L, H), [emb, idn], [B * L, H, self.V, 0])
        shp = (B, L, H)
        present = []
        for l in range(self.L):
            p = f"layers.{l}."
            normed = g.add_trusted("rmsnorm", shp, [h, self._w(g, nodes, p + "attn_norm")], [self.eps])
            q, _ = self._linear(g, nodes, normed, shp, p + "q")
            q = g.add_trusted("rope", (B, self.Hq, L, hd), [self._heads(g, q, B, L, self.Hq)], [self.theta, float(offset)])
            k, _ = self._linear(g, nodes, normed, shp, p + "k")
            k = g.add_trusted("rope", (B, self.Hkv, L, hd), [self._heads(g, k, B, L, self.Hkv)], [self.theta, float(offset)])
            if past is not None:
                pk, pv, ps = past[l]
                k = g.add_trusted("cat", (B, self.Hkv, ps + L, hd), [pk, k], [ps, L, hd])
            else:
                ps = 0
            S = ps + L
            kr = self._repeat(g, k, B, S)
            v, _ = self._linear(g, nodes, normed, shp, p + "v")
            v = self._heads(g, v, B, L, self.Hkv)
            if past is not None:
                v = g.add_trusted("cat", (B, self.Hkv, S, hd), [pv, v], [ps, L, hd])
            vr = self._repeat(g, v, B, S)
            present.append((k, v, S))
            att = g.add_trusted("flash_attention", (B, self.Hq, L, hd), [q, kr, vr],
                           [float(self.Hq), 1.0 / math.sqrt(hd), 1.0, float(S)])
            att = g.add_trusted("permute", (B, L, self.Hq, hd), [att], [0, 2, 1, 3])
            att = g.add_trusted("reshape", shp, [att], list(shp))
            o, _ = self._linear(g, nodes, att, shp, p + "o")
            h = g.add_trusted("add", shp, [h, o], [B * L * H, B * L * H])
            nm = g.add_trusted("rmsnorm", shp, [h, self._w(g, nodes, p + "ffn_norm")], [self.eps])
            gate, gshp = self._linear(g, nodes, nm, shp, p + "gate")
            up, _ = self._linear(g, nodes, nm, shp, p + "up")
            sw = g.add_trusted("swiglu", gshp, [gate, up])
            down, _ = self._linear(g, nodes, sw, gshp, p + "down")
            h = g.add_trusted("add", shp, [h, down], [B * L * H, B * L * H])
        h = g.add_trusted("rmsnorm", shp, [h, self._w(g, nodes, "norm")], [self.eps])
        logits, lshp = self._linear(g, nodes, h, shp, "lm_head")
        return logits, lshp, present

    # ------------------------------------------------------------ execution
    def generate(self, prompt: Sequence[int], max_new_tokens: int, logits_out: Optional[list] = None) -> List[int]:
        """Cached greedy generation (llama.py:211-248), one executeGraph call per token; the last-position
        logits of every step are appended to `logits_out` when given."""
        ctx = self.ctx
        out = list(prompt)
        past = None  # [(k handle, v handle, length)]
        for step in range(max_new_tokens):
            g = GraphBuilder()
            nodes: Dict[str, int] = {}
            ids = np.array([out] if step == 0 else [[out[-1]]], np.int32)
            offset = 0 if step == 0 else len(prompt) + step - 1
            past_nodes = None
            if past is not None:
                past_nodes = [(g.add_load((1, self.Hkv, s, self.hd), kh), g.add_load((1, self.Hkv, s, self.hd), vh), s)
                              for kh, vh, s in past]
            logits, lshp, present = self.forward(g, nodes, ids, offset, past_nodes)
            js, inputs = g.compile()
            res = execute_graph(ctx, js, inputs)
            lg = ctx.read(res[str(logits)]).reshape(lshp)
            if logits_out is not None:
                logits_out.append(lg[0, -1].copy())
            out.append(int(np.argmax(lg[0, -1])))
            keep = {str(logits)}
            new_past = []
            for k, v, s in present:
                new_past.append((res[str(k)], res[str(v)], s))
                keep |= {str(k), str(v)}
            # every other new tensor of this graph (loads name existing tensors: weights, the past cache)
            loaded = {str(n["id"]) for n in g.nodes if n["op"] == "load"}
            ctx.dispose_batch([h for i, h in res.items() if i not in keep and i not in loaded])
            ctx.dispose(res[str(logits)])
            if past is not None:
                ctx.dispose_batch([x for kh, vh, _ in past for x in (kh, vh)])
            past = new_past
        if past is not None:
            ctx.dispose_batch([x for kh, vh, _ in past for x in (kh, vh)])
        return out
