"""Tensor parallelism of the Llama decoder over 2 ranks (gloo, CPU).

The GPU path (ameva-forge_b200/csrc/llama.cu) splits the decoder Megatron
style:
- q/k/v and gate/up by output rows (whole heads, whole FFN columns);
- o_proj and down_proj by input columns, followed by a sum all-reduce;
- lm_head by vocabulary rows; the greedy pick all-reduces a (value, lowest
  index) key with MAX;
- the embedding and the norms are replicated.

Here each rank restates that split with the oracle's primitives on its
shard, and the ranks exchange partial sums over torch.distributed (gloo), the
process-group plumbing the multi-GPU bench uses.  The logits gathered from
the ranks and the greedy tokens must equal the unsharded oracle's.
"""
import os
import socket
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "oracle"))

SHAPE = dict(vocab_size=96, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2)
SEED, STEPS = 31, 3
PROMPT = (np.arange(10, dtype=np.int32) * 7 + 5) % 96


def _rows(blocks, r0, r1):
    return np.ascontiguousarray(blocks[r0:r1])


def _cols(blocks, K, c0, c1):
    b = blocks.reshape(blocks.shape[0], K // 32, -1)
    return np.ascontiguousarray(b[:, c0 // 32:c1 // 32]).reshape(blocks.shape[0], -1)


def _key(v, idx):
    """Greedy key of logit v at global index idx: ordered float bits, then the
    lowest index; shifted into the signed int64 range for the MAX reduction."""
    bits = int(np.float32(v).view(np.uint32))
    bits = (~bits & 0xFFFFFFFF) if bits & 0x80000000 else (bits | 0x80000000)
    return ((bits << 32) | (0xFFFFFFFF - idx)) - (1 << 63)


def _rank_main(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shape = O.LlamaShape(**SHAPE)
    w = O.synth_llama(shape, SEED)
    Hd, H, Hkv, d, I, V = (shape.hidden_size, shape.num_attention_heads, shape.num_key_value_heads,
                           shape.head_dim, shape.intermediate_size, shape.vocab_size)
    Hl, Hkvl, Il, Vl = H // world, Hkv // world, I // world, V // world
    qt = w.qtype
    layers = []
    for L in w.layers:
        layers.append(dict(
            q=_rows(L["q"], rank * Hl * d, (rank + 1) * Hl * d),
            k=_rows(L["k"], rank * Hkvl * d, (rank + 1) * Hkvl * d),
            v=_rows(L["v"], rank * Hkvl * d, (rank + 1) * Hkvl * d),
            o=_cols(L["o"], Hd, rank * Hl * d, (rank + 1) * Hl * d),
            gate=_rows(L["gate"], rank * Il, (rank + 1) * Il),
            up=_rows(L["up"], rank * Il, (rank + 1) * Il),
            down=_cols(L["down"], I, rank * Il, (rank + 1) * Il),
            attn_norm=L["attn_norm"], ffn_norm=L["ffn_norm"]))
    lm = _rows(w.lm_head, rank * Vl, (rank + 1) * Vl)
    embed = O.f16_to_f32(w.embed_f16)
    cap = len(PROMPT) + STEPS + 1
    kc = [np.zeros((1, Hkvl, cap, d), np.float32) for _ in layers]
    vc = [np.zeros_like(kc[0]) for _ in layers]

    def allreduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
        dist.all_reduce(t)
        return t.numpy()

    pos = 0
    ids = PROMPT[None, :]
    logits_seq, tokens = [], []
    for _ in range(STEPS + 1):
        B, T = ids.shape
        h = O.embedding(embed, ids)
        for li, L in enumerate(layers):
            x = O.rmsnorm(h, L["attn_norm"], shape.rms_norm_eps)
            q = O.qmatmul(qt, L["q"], Hl * d, Hd, x).reshape(B, T, Hl, d).transpose(0, 2, 1, 3)
            k = O.qmatmul(qt, L["k"], Hkvl * d, Hd, x).reshape(B, T, Hkvl, d).transpose(0, 2, 1, 3)
            v = O.qmatmul(qt, L["v"], Hkvl * d, Hd, x).reshape(B, T, Hkvl, d).transpose(0, 2, 1, 3)
            q = O.rope(q, shape.rope_theta, pos)
            k = O.round_f16(O.rope(k, shape.rope_theta, pos))
            kc[li][:, :, pos:pos + T] = k
            vc[li][:, :, pos:pos + T] = O.round_f16(v)
            a = O.attention(q, kc[li], vc[li], 1.0 / np.sqrt(d), True, n_kv=pos + T)
            a = np.ascontiguousarray(a.transpose(0, 2, 1, 3)).reshape(B, T, Hl * d)
            h = h + allreduce(O.qmatmul(qt, L["o"], Hd, Hl * d, a))          # row-parallel o_proj
            x = O.rmsnorm(h, L["ffn_norm"], shape.rms_norm_eps)
            g = O.qmatmul(qt, L["gate"], Il, Hd, x)
            u = O.qmatmul(qt, L["up"], Il, Hd, x)
            h = h + allreduce(O.qmatmul(qt, L["down"], Hd, Il, O.swiglu(g, u)))  # row-parallel down_proj
        pos += T
        hn = O.rmsnorm(h[:, -1], w.norm, shape.rms_norm_eps)
        local = O.qmatmul(qt, lm, Vl, Hd, hn)[0]                             # vocabulary shard
        j = int(np.argmax(local))                                            # first max of the shard
        key = torch.tensor([_key(local[j], rank * Vl + j)], dtype=torch.int64)
        dist.all_reduce(key, op=dist.ReduceOp.MAX)
        tok = 0xFFFFFFFF - ((int(key.item()) + (1 << 63)) & 0xFFFFFFFF)
        parts = [torch.zeros(Vl) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(local)))
        logits_seq.append(torch.cat(parts).numpy())
        tokens.append(tok)
        ids = np.array([[tok]], np.int32)
    if rank == 0:
        np.savez(os.path.join(out_dir, "tp.npz"), logits=np.stack(logits_seq), tokens=np.array(tokens))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_split_equals_unsharded(tmp_path):
    import torch.multiprocessing as mp
    import oracle as O

    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    got = np.load(tmp_path / "tp.npz")
    ref = O.LlamaRef(O.synth_llama(O.LlamaShape(**SHAPE), SEED), max_seq=len(PROMPT) + STEPS + 1, kv_f16=True)
    lg = ref.forward(PROMPT[None, :])[0, -1]
    for step in range(STEPS + 1):
        tok = O.argmax(lg)
        np.testing.assert_allclose(got["logits"][step], lg, rtol=0, atol=1e-5 * np.abs(lg).max())
        assert int(got["tokens"][step]) == tok
        lg = ref.forward(np.array([[tok]], np.int32))[0, -1]
