"""Tensor parallelism on two GPUs: the TP=2 model (two ranks, NCCL all-reduce
after o_proj and down_proj, vocabulary-sharded lm_head) must give the logits
and greedy tokens of the TP=1 model on the same synthesized weights.

Each rank synthesizes only its shard; shards are slices of the same global
tensors (counter-based generator with global row/column offsets), so the two
runs differ only in the order of the all-reduced partial sums.  The prompt
(40 tokens) takes the tensor-core GEMM and attention with NCCL all-reduces;
the batch-1 decode steps take the persistent step kernel on both sides: at
TP=2 its tensor-parallel instance, which exchanges the o_proj / down_proj
partial sums and the greedy keys over NVLink peer memory inside the kernel
(no NCCL).  Each run records the decode path it took, and the test asserts
it was the step kernel.
"""
import os
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# GQA 2:1 per rank (the step kernel's CUDA-core attention tile) and GQA 4:1 (its tensor-core tile)
SHAPES = {
    "gqa2": dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                 num_key_value_heads=2),
    "gqa4": dict(vocab_size=512, hidden_size=512, intermediate_size=512, num_hidden_layers=2, num_attention_heads=8,
                 num_key_value_heads=2),
}
SEED, STEPS = 97, 3
PROMPT = ((np.arange(40, dtype=np.int32) * 37 + 11) % 512).reshape(1, 40)


def _run(ctx, shape, out_path):
    import forge_b200
    cfg = forge_b200.LlamaConfig(max_position_embeddings=64, max_batch=1, qtype="Q4_0", **SHAPES[shape])
    m = forge_b200.LlamaForCausalLM(cfg, ctx)
    m.synthesize(SEED)
    path = m.decode_path(1)
    logits, nxt = m.forward(PROMPT)
    seq = [logits[0].copy()]
    toks = [int(nxt[0])]
    ids = np.asarray(nxt, np.int32)
    for _ in range(STEPS):
        ids, lg = m.decode(ids, return_logits=True)
        seq.append(lg[0].copy())
        toks.append(int(ids[0]))
    m.close()
    if out_path:
        np.savez(out_path, logits=np.stack(seq), tokens=np.array(toks), path=np.array(path))


def _rank(rank, world, nid, shape, out_dir):
    import forge_b200
    ctx = forge_b200.Context(device=rank, tp_rank=rank, tp_size=world, nccl_id=nid)
    _run(ctx, shape, os.path.join(out_dir, "tp2.npz") if rank == 0 else None)
    ctx.shutdown()
    if rank == 0:  # the unsharded model on the same device
        ctx1 = forge_b200.Context(device=0)
        _run(ctx1, shape, os.path.join(out_dir, "tp1.npz"))
        ctx1.shutdown()


@pytest.mark.parametrize("shape", sorted(SHAPES))
def test_two_gpu_tensor_parallel_matches_single_gpu(tmp_path, shape):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import forge_b200
    nid = forge_b200.nccl_unique_id()
    ctxs = mp.start_processes(_rank, args=(2, nid, shape, str(tmp_path)), nprocs=2, join=False, start_method="spawn")
    deadline = time.time() + 240
    while not ctxs.join(timeout=5):
        if time.time() > deadline:
            for p in ctxs.processes:
                p.kill()
            pytest.fail("tensor-parallel ranks did not finish within 240 s")
    a, b = np.load(tmp_path / "tp2.npz"), np.load(tmp_path / "tp1.npz")
    ref = b["logits"]
    err = np.abs(a["logits"] - ref).max() / np.abs(ref).max()
    assert err <= 1e-3, err
    assert list(a["tokens"]) == list(b["tokens"])
    assert str(a["path"]) == "step" and str(b["path"]) == "step"
