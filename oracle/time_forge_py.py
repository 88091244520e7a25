"""Time the reference's own CPU decode path beside the oracle port.

    python oracle/time_forge_py.py <reference checkout root> [--layers 2] [--steps 3]

(or set AMEVA_FORGE_REFERENCE).  Runs where the reference checkout is: its
Python package (packages/forge-py/src) is imported from there, so this
script cannot run on a host without the checkout, and bench.py only reads
the JSON it writes.

Workload: greedy decode at context 4096 of the Llama-2-7B-shaped model with
`layers` of its 32 layers, plus embedding, final norm and lm_head; the same
seeded weights (dequantised to fp32 for forge-py, which has no quantized
path) and the same seeded fp16 KV cache as the benchmark.  Both sides run
`steps` timed steps after one warm-up step, on this host's cores:

* forge-py `LlamaForCausalLM(device='cpu')` -- the model-forward API of
  packages/forge-py/src/forge/models/llama.py:199-248, numpy fp32, with its
  KV append by `cat` (llama.py:111-113);
* the oracle port (oracle/forge_oracle.c via LlamaRef), the same arithmetic
  the benchmark's reference arm times on the GPU host.

Writes oracle/forge_py_cpu_timing.json: seconds per step of each side, the
full-model tokens/s each implies (layer time scaled to 32 layers), the core
count and the CPU model.
"""
import json
import os
import platform
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import oracle as O  # noqa: E402

SHAPE = dict(vocab_size=32000, hidden_size=4096, intermediate_size=11008, num_attention_heads=32,
             num_key_value_heads=32, rms_norm_eps=1e-5, rope_theta=10000.0)
SEED, CONTEXT, FULL_LAYERS = 20240601, 4096, 32


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor()


def main(ref_root, layers, steps):
    sys.path.insert(0, os.path.join(ref_root, "packages", "forge-py", "src"))
    import forge
    from forge.models.llama import LlamaConfig, LlamaForCausalLM

    shp = O.LlamaShape(**SHAPE, num_hidden_layers=layers)
    w = O.synth_llama(shp, SEED)
    ref = O.LlamaRef(w, max_seq=CONTEXT + steps + 2, kv_f16=True)
    ref.synthesize_kv(SEED + 1, CONTEXT)

    cfg = LlamaConfig(**SHAPE, num_hidden_layers=layers, device="cpu")
    m = LlamaForCausalLM(cfg)
    H, d = shp.hidden_size, shp.head_dim

    def deq(blocks, r, c):
        return forge.tensor(O.dequant(O.Q4_0, blocks, r, c))

    m.model.embed_tokens.weight = forge.tensor(O.f16_to_f32(w.embed_f16))
    m.model.norm.weight = forge.tensor(w.norm)
    m.lm_head.weight = deq(w.lm_head, shp.vocab_size, H)
    kvd = shp.num_key_value_heads * d
    for li, L in enumerate(w.layers):
        layer = m.model.layers[li]
        layer.input_layernorm.weight = forge.tensor(L["attn_norm"])
        layer.post_attention_layernorm.weight = forge.tensor(L["ffn_norm"])
        a = layer.self_attn
        a.q_proj.weight = deq(L["q"], H, H)
        a.k_proj.weight = deq(L["k"], kvd, H)
        a.v_proj.weight = deq(L["v"], kvd, H)
        a.o_proj.weight = deq(L["o"], H, H)
        mlp = layer.mlp
        mlp.gate_proj.weight = deq(L["gate"], shp.intermediate_size, H)
        mlp.up_proj.weight = deq(L["up"], shp.intermediate_size, H)
        mlp.down_proj.weight = deq(L["down"], H, shp.intermediate_size)
    kvs = [(forge.tensor(np.ascontiguousarray(ref.k[li][:, :, :CONTEXT])),
            forge.tensor(np.ascontiguousarray(ref.v[li][:, :, :CONTEXT]))) for li in range(layers)]

    def forge_step(tok, pos):
        nonlocal kvs
        lg, kvs = m.forward(forge.tensor(np.array([[tok]], np.int32)), past_key_values=kvs, offset_pos=pos,
                            use_cache=True)
        return int(np.argmax(lg.numpy()[0, -1]))

    def timed(fn, n):
        out = []
        for _ in range(n):
            t0 = time.perf_counter()
            fn()
            out.append(time.perf_counter() - t0)
        return out

    state = {"tok": 1, "pos": CONTEXT}

    def fstep():
        state["tok"] = forge_step(state["tok"], state["pos"])
        state["pos"] += 1

    rtok = {"tok": np.array([[1]], np.int32)}

    def ostep():
        lg = ref.forward(rtok["tok"])
        rtok["tok"] = np.array([[O.argmax(lg[0, -1])]], np.int32)

    t_forge = timed(fstep, 1 + steps)[1:]
    t_port = timed(ostep, 1 + steps)[1:]
    # the head (final norm + lm_head) does not scale with the layer count
    x = O.normal(1, 0, H, 0.0, 1.0).reshape(1, H)
    t0 = time.perf_counter()
    O.qmatmul(O.Q4_0, w.lm_head, shp.vocab_size, H, O.rmsnorm(x, w.norm))
    t_head_port = time.perf_counter() - t0
    wl = m.lm_head.weight.numpy()
    t0 = time.perf_counter()
    _ = x @ wl.T
    t_head_forge = time.perf_counter() - t0

    def full(ts, th):
        per = float(np.median(ts))
        return per, 1.0 / ((per - th) * (FULL_LAYERS / layers) + th)

    pf, vf = full(t_forge, t_head_forge)
    pp, vp = full(t_port, t_head_port)
    out = {
        "what": "forge-py LlamaForCausalLM(device='cpu') decode beside the oracle port, same weights and KV",
        "workload": f"Llama-2-7B shape, {layers} of {FULL_LAYERS} layers + embedding + lm_head, batch 1, "
                    f"context {CONTEXT}, fp16-valued KV cache, greedy",
        "steps_timed": steps, "warmup": 1, "layers_timed": layers,
        "forge_py": {"s_per_step_sample": pf, "tokens_per_s_full_model_scaled": vf,
                     "code": "packages/forge-py/src/forge/models/llama.py:199-248 (numpy fp32)"},
        "oracle_port": {"s_per_step_sample": pp, "tokens_per_s_full_model_scaled": vp,
                        "threads": O.num_threads(), "code": "oracle/forge_oracle.c via oracle.LlamaRef"},
        "host": {"cores": os.cpu_count(), "cpu": cpu_model()},
        "measured_where": "the build container (the reference checkout is not on the GPU host)",
    }
    path = os.path.join(HERE, "forge_py_cpu_timing.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("root", nargs="?", default=os.environ.get("AMEVA_FORGE_REFERENCE", ""),
                    help="reference checkout root (or AMEVA_FORGE_REFERENCE)")
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--steps", type=int, default=3)
    a = ap.parse_args()
    if not a.root:
        ap.error("the reference checkout root is required")
    main(a.root, a.layers, a.steps)
