"""GGUF container reader (fg_gguf_*, host code: runs without a GPU) and the
Llama loader (fg_llama_load_gguf) against the oracle on the same weights."""
import struct

import numpy as np
import pytest

import gguf_write as GW
import oracle as O
from conftest import max_rel_err

SHAPE = dict(vocab_size=96, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2)
SEED = 43


@pytest.fixture(scope="module")
def model_file(tmp_path_factory):
    w = O.synth_llama(O.LlamaShape(**SHAPE), SEED)
    path = tmp_path_factory.mktemp("gguf") / "tiny.gguf"
    GW.write_llama(str(path), w)
    return str(path), w


def test_table_metadata_and_bytes(model_file):
    import forge_b200
    path, w = model_file
    with forge_b200.GGUFFile(path) as g:
        ts = {t["name"]: t for t in g.tensors()}
        assert len(ts) == 3 + 9 * SHAPE["num_hidden_layers"]
        assert ts["token_embd.weight"]["dtype"] == "F16" and ts["token_embd.weight"]["dims"] == (64, 96)
        assert ts["blk.1.ffn_down.weight"]["dims"] == (128, 64) and ts["blk.1.ffn_down.weight"]["dtype"] == "Q4_0"
        assert np.array_equal(ts["blk.0.attn_q.weight"]["bytes"], w.layers[0]["q"].reshape(-1))
        assert np.array_equal(ts["output.weight"]["bytes"], w.lm_head.reshape(-1))
        assert g.string("general.architecture") == "llama"
        assert g.number("llama.block_count") == 2
        assert abs(g.number("llama.rope.freq_base") - 10000.0) < 1e-3
        cfg = g.llama_config(max_position_embeddings=80)
        assert (cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers,
                cfg.num_attention_heads, cfg.num_key_value_heads, cfg.qtype, cfg.max_position_embeddings) == \
               (96, 64, 128, 2, 4, 2, "Q4_0", 80)


def test_malformed_files_are_validation_errors(model_file, tmp_path):
    import forge_b200
    from forge_b200.errors import AMEVAForgeValidationError
    path, _ = model_file
    raw = open(path, "rb").read()
    cases = {"truncated.gguf": raw[:len(raw) // 2],      # tensor data past the end of the file
             "magic.gguf": b"GGUX" + raw[4:],
             "version.gguf": raw[:4] + struct.pack("<I", 9) + raw[8:],
             "header.gguf": raw[:30]}                      # cut inside the metadata
    for name, data in cases.items():
        p = tmp_path / name
        p.write_bytes(data)
        with pytest.raises(AMEVAForgeValidationError):
            forge_b200.GGUFFile(str(p))
    with pytest.raises(AMEVAForgeValidationError):
        forge_b200.GGUFFile(str(tmp_path / "missing.gguf"))


@pytest.mark.gpu
def test_from_gguf_matches_oracle(ctx, model_file):
    import forge_b200
    path, w = model_file
    m = forge_b200.LlamaForCausalLM.from_gguf(path, ctx, max_position_embeddings=64)
    ref = O.LlamaRef(w, max_seq=64, kv_f16=True)
    prompt = (np.arange(12, dtype=np.int32) * 5 + 3) % 96
    lg, nxt = m.forward(prompt[None, :])
    lr = ref.forward(prompt[None, :])[0, -1]
    assert max_rel_err(lg[0], lr) <= 2e-3
    assert int(nxt[0]) == O.argmax(lr)
    m.close()
