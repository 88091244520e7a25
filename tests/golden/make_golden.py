"""Regenerate the golden fixtures in this directory from the reference itself.

Run in a container that holds the reference checkout:

    python tests/golden/make_golden.py /path/to/ameva-forge

It imports the reference's Python package (packages/forge-py/src) and runs
its CPU code paths -- F.rms_norm, F.rope, F.swiglu,
F.scaled_dot_product_attention, forge matmul and LlamaForCausalLM -- on the
deterministic inputs that the reference's own tests use, and stores inputs
and outputs as .npz.  The unpack known-answer vectors follow the input
formulas of packages/forge/tests/quantization_unpack.test.ts:101-206 with
expected values from an independent vectorised restatement of
unpack_quant.wgsl.ts:25-62 (the TS suite only checks finiteness, and node is
not available to run it).  The GPU box never needs the reference: the tests
read only the .npz files written here.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "packages", "forge-py", "src"))
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import forge
    import forge.functional as F
    import oracle as O

    out = {}
    sys.path.insert(0, HERE)
    import inputs as I

    # -- unpack known answers: independent vectorised restatement of the WGSL
    for name, (packed, scales, zeros, bits, gs, n) in (("unpack4", I.unpack4()), ("unpack8", I.unpack8())):
        i = np.arange(n)
        per = 32 // bits
        raw = ((packed[i // per] >> (bits * (i % per)).astype(np.uint32)) & ((1 << bits) - 1)).astype(np.float32)
        out[name + "_expected"] = ((raw - zeros[i // gs]).astype(np.float32) * scales[i // gs]).astype(np.float32)

    x, g = I.rmsnorm()
    out["rmsnorm_out"] = F.rms_norm(forge.tensor(x), forge.tensor(g), eps=1e-5).numpy()
    x, g = I.rmsnorm_small()
    out["rmsnorm2_out"] = F.rms_norm(forge.tensor(x), forge.tensor(g), eps=1e-5).numpy()
    out["rope_out"] = F.rope(forge.tensor(I.rope()), base_freq=10000.0, offset_pos=0).numpy()
    out["rope_off_out"] = F.rope(forge.tensor(I.rope_offset()), base_freq=10000.0, offset_pos=2047).numpy()
    gt, up = I.swiglu()
    out["swiglu_out"] = F.swiglu(forge.tensor(gt), forge.tensor(up)).numpy()

    q, k, v = I.mha()
    out["mha_out"] = F.scaled_dot_product_attention(forge.tensor(q), forge.tensor(k), forge.tensor(v),
                                                    is_causal=False, scale=1.0 / np.sqrt(q.shape[-1])).numpy()
    q, k, v = I.gqa()
    rep = q.shape[1] // k.shape[1]  # GQA by head repetition, as llama.py:116-127 does
    out["gqa_out"] = F.scaled_dot_product_attention(
        forge.tensor(q), forge.tensor(np.repeat(k, rep, axis=1)), forge.tensor(np.repeat(v, rep, axis=1)),
        is_causal=True, scale=1.0 / np.sqrt(q.shape[-1])).numpy()

    for (M, K, Nn) in I.MATMUL_SHAPES:
        A, Bm = I.matmul(M, K, Nn)
        out[f"matmul_{M}x{K}x{Nn}"] = forge.matmul(forge.tensor(A), forge.tensor(Bm)).numpy()

    # -- tiny Llama through the reference's LlamaForCausalLM on CPU, weights =
    #    the dequantised synthetic Q4_0 model (fp16 embedding widened to fp32)
    from forge.models.llama import LlamaConfig, LlamaForCausalLM
    shp = O.LlamaShape(**I.LLAMA_SHAPE)
    w = O.synth_llama(shp, seed=I.LLAMA_SEED)
    cfg = LlamaConfig(**I.LLAMA_SHAPE, device="cpu")
    m = LlamaForCausalLM(cfg)
    Hd, d = shp.hidden_size, shp.head_dim

    def deq(blocks, r, c):
        return forge.tensor(O.dequant(O.Q4_0, blocks, r, c))

    m.model.embed_tokens.weight = forge.tensor(O.f16_to_f32(w.embed_f16))
    m.model.norm.weight = forge.tensor(w.norm)
    m.lm_head.weight = deq(w.lm_head, shp.vocab_size, Hd)
    kvd = shp.num_key_value_heads * d
    for li, L in enumerate(w.layers):
        layer = m.model.layers[li]
        layer.input_layernorm.weight = forge.tensor(L["attn_norm"])
        layer.post_attention_layernorm.weight = forge.tensor(L["ffn_norm"])
        a = layer.self_attn
        a.q_proj.weight = deq(L["q"], Hd, Hd)
        a.k_proj.weight = deq(L["k"], kvd, Hd)
        a.v_proj.weight = deq(L["v"], kvd, Hd)
        a.o_proj.weight = deq(L["o"], Hd, Hd)
        mlp = layer.mlp
        mlp.gate_proj.weight = deq(L["gate"], shp.intermediate_size, Hd)
        mlp.up_proj.weight = deq(L["up"], shp.intermediate_size, Hd)
        mlp.down_proj.weight = deq(L["down"], Hd, shp.intermediate_size)

    prompt = I.LLAMA_PROMPT
    logits, kvs = m.forward(forge.tensor(prompt), use_cache=True, offset_pos=0)
    lg = logits.numpy()
    toks, step_logits = [int(np.argmax(lg[0, -1]))], [lg[0, -1].copy()]
    for step in range(1, I.LLAMA_STEPS):
        inp = forge.tensor(np.array([[toks[-1]]], np.int32))
        lg2, kvs = m.forward(inp, past_key_values=kvs, offset_pos=prompt.shape[1] + step - 1, use_cache=True)
        lgn = lg2.numpy()
        step_logits.append(lgn[0, -1].copy())
        toks.append(int(np.argmax(lgn[0, -1])))
    out.update(llama_prefill_logits=lg, llama_tokens=np.array(toks, np.int32),
               llama_step_logits=np.stack(step_logits))

    path = os.path.join(HERE, "reference_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes,", len(out), "arrays")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AMEVA_FORGE_REFERENCE", "")
    if not root:
        sys.exit(f"usage: python {os.path.basename(__file__)} <reference checkout root> "
                 "(or set AMEVA_FORGE_REFERENCE)")
    main(root)
