"""Deterministic inputs of the reference's own tests, restated as formulas so
the fixtures only store the reference's outputs.  Each function cites the
test whose inputs it reproduces (packages/forge/tests/...)."""
import numpy as np

MATMUL_SHAPES = [(16, 16, 16), (64, 64, 64), (128, 128, 128), (256, 256, 256), (32, 64, 128), (128, 32, 64),
                 (64, 128, 32), (1, 17, 1), (7, 13, 11), (17, 33, 19), (65, 127, 31), (100, 200, 150),
                 (128, 768, 768), (128, 768, 2304), (128, 3072, 768)]


def unpack4():
    """quantization_unpack.test.ts:101-152: 1024 INT4 values, group 32."""
    n, gs = 1024, 32
    words = np.arange(n // 8, dtype=np.uint64)
    packed = np.zeros(n // 8, dtype=np.uint64)
    for nib in range(8):
        packed |= ((words * 8 + nib) % 16) << np.uint64(4 * nib)
    scales = (0.05 + np.arange(n // gs) * 0.001).astype(np.float32)
    return packed.astype(np.uint32), scales, np.full(n // gs, 8.0, np.float32), 4, gs, n


def unpack8():
    """quantization_unpack.test.ts:155-206: 1024 INT8 values, group 64."""
    n, gs = 1024, 64
    words = np.arange(n // 4, dtype=np.uint64)
    packed = np.zeros(n // 4, dtype=np.uint64)
    for b in range(4):
        packed |= ((words * 4 + b) % 256) << np.uint64(8 * b)
    scales = (0.01 + np.arange(n // gs) * 0.0005).astype(np.float32)
    return packed.astype(np.uint32), scales, np.full(n // gs, 128.0, np.float32), 8, gs, n


def rmsnorm():
    """llm_generation_primitives.test.ts:184-216: 32 x 2048."""
    x = (np.sin(np.arange(32 * 2048) * 0.02) * 1.5).astype(np.float32).reshape(32, 2048)
    g = (1.0 + np.cos(np.arange(2048) * 0.02) * 0.1).astype(np.float32)
    return x, g


def rmsnorm_small():
    """packages/forge-py/tests/test_release2_llm_modules.py:13-25."""
    x = np.array([[-1.0, 2.0, 3.0, -4.0], [0.5, -0.5, 1.5, -1.5]], np.float32)
    g = np.array([1.0, 2.0, 0.5, 1.5], np.float32)
    return x, g


def rope():
    """llm_generation_primitives.test.ts:132-163: B2 H4 N128 d64, offset 0."""
    return (np.sin(np.arange(2 * 4 * 128 * 64) * 0.01) * 0.5).astype(np.float32).reshape(2, 4, 128, 64)


def rope_offset():
    """Long-context case (offset 2047, d 128) on the same kind of input."""
    return (np.cos(np.arange(1 * 2 * 4 * 128) * 0.013) * 0.7).astype(np.float32).reshape(1, 2, 4, 128)


def swiglu():
    """llm_generation_primitives.test.ts:237-266: 10 000 elements."""
    i = np.arange(10000)
    return (np.sin(i * 0.05) * 2.0).astype(np.float32), (np.cos(i * 0.05) * 2.0).astype(np.float32)


def mha():
    """flash_attention.test.ts:203-223: B2 H4 N64 d64, not causal."""
    B, H, N, d = 2, 4, 64, 64
    n = B * H * N * d
    q = (np.sin(np.arange(n) * 0.05) * 0.5).astype(np.float32).reshape(B, H, N, d)
    k = (np.cos(np.arange(n) * 0.05) * 0.5).astype(np.float32).reshape(B, H, N, d)
    v = (np.sin(np.arange(n) * 0.1) * 0.5).astype(np.float32).reshape(B, H, N, d)
    return q, k, v


def gqa():
    """flash_attention.test.ts:226-247: B1 H8 Hkv2 N128 d64, causal."""
    B, H, Hkv, N, d = 1, 8, 2, 128, 64
    q = (np.sin(np.arange(B * H * N * d) * 0.03) * 0.4).astype(np.float32).reshape(B, H, N, d)
    k = (np.cos(np.arange(B * Hkv * N * d) * 0.03) * 0.4).astype(np.float32).reshape(B, Hkv, N, d)
    v = (np.sin(np.arange(B * Hkv * N * d) * 0.07) * 0.4).astype(np.float32).reshape(B, Hkv, N, d)
    return q, k, v


def matmul(M, K, N):
    """matmul_tiled.test.ts:172-178: A = sin(i+1)*0.8, B = cos(i+1)*0.8."""
    A = (np.sin(np.arange(M * K) + 1.0) * 0.8).astype(np.float32).reshape(M, K)
    B = (np.cos(np.arange(K * N) + 1.0) * 0.8).astype(np.float32).reshape(K, N)
    return A, B


GREEDY_LOGITS = np.array([1.2, 5.8, -0.4, 3.1, 0.9], np.float32)  # llm_generation_primitives.test.ts:270-274
GREEDY_INDEX = 1

# Tiny Llama of the reference-model fixture (LlamaForCausalLM on CPU).
LLAMA_SEED = 1234
LLAMA_SHAPE = dict(vocab_size=96, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                   num_attention_heads=4, num_key_value_heads=2)
LLAMA_PROMPT = np.array([[5, 17, 33, 2, 90, 41, 7, 64]], np.int32)
LLAMA_STEPS = 6
