"""GGUF Q4_K: the oracle's restatement of the published block format against
hand-computed known answers (CPU), the GGUF reader listing Q4_K tensors
(CPU), and the device path -- upload round trip, bit-exact dequantisation,
the fused GEMV / GEMM, the graph front-end's transpose fold (GPU)."""
import os

import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err


def _block(d, dmin, scales12, nibble_byte):
    b = np.zeros(144, np.uint8)
    dh, mh = np.float16(d).view(np.uint16), np.float16(dmin).view(np.uint16)
    b[0], b[1], b[2], b[3] = dh & 255, dh >> 8, mh & 255, mh >> 8
    b[4:16] = scales12
    b[16:] = nibble_byte
    return b.reshape(1, 144)


def test_q4k_known_answers():
    # sub-blocks 0-3: scale s[j] & 63, min s[j+4] & 63; 4-7: low/high nibbles of s[j+4] (+ top bits of s[j-4], s[j])
    blk = _block(0.5, 0.25, [1, 2, 3, 4, 5, 6, 7, 8, 0x21, 0x43, 0x65, 0x87], 0x53)  # q = 3 (low), 5 (high)
    w = O.dequant_q4k(blk, 1, 256)[0]
    want = [0.5 * 1 * 3 - 0.25 * 5, 0.5 * 2 * 5 - 0.25 * 6, 0.5 * 3 * 3 - 0.25 * 7, 0.5 * 4 * 5 - 0.25 * 8,
            0.5 * 1 * 3 - 0.25 * 2, 0.5 * 3 * 5 - 0.25 * 4, 0.5 * 5 * 3 - 0.25 * 6, 0.5 * 7 * 5 - 0.25 * 8]
    for sb in range(8):
        assert np.all(w[32 * sb:32 * sb + 32] == np.float32(want[sb])), sb
    # the top two bits of s[0..7] extend the scales / mins of sub-blocks 4..7
    blk = _block(1.0, 1.0, [0xC1, 0x40, 0, 0, 0x80, 0, 0, 0xC0, 0x00, 0x00, 0x00, 0x00], 0x11)
    w = O.dequant_q4k(blk, 1, 256)[0]
    assert w[0] == np.float32(1 * 1 - 0)        # sub-block 0: scale 1, min 0 (0x80 & 63)
    assert w[128] == np.float32(48 * 1 - 32)    # sub-block 4: scale 0 | 3 << 4, min 0 | 2 << 4
    assert w[160] == np.float32(16 * 1 - 0)     # sub-block 5: scale 0 | 1 << 4, min 0
    assert w[224] == np.float32(0 * 1 - 48)     # sub-block 7: scale 0, min 0 | 3 << 4


def test_gguf_lists_q4k_tensors(tmp_path):
    import forge_b200
    import gguf_write as GW
    blocks = O.random_q4k(4, 512, 3)
    path = os.path.join(tmp_path, "q4k.gguf")
    GW.write(path, [("general.architecture", GW.V_STR, "llama")], [("blk.0.ffn_down.weight", 12, [512, 4], blocks)])
    with forge_b200.GGUFFile(path) as g:
        t = {t["name"]: t for t in g.tensors()}["blk.0.ffn_down.weight"]
        assert t["dtype"] == "Q4_K" and t["dims"] == (512, 4)
        assert np.array_equal(t["bytes"], blocks.reshape(-1))


@pytest.mark.gpu
def test_q4k_upload_roundtrip_and_exact_dequant(ctx):
    blocks = O.random_q4k(96, 1024, 5)
    h = ctx.upload_quant("Q4_K", blocks, 96, 1024)
    assert np.array_equal(ctx.read_quant_gguf(h), blocks)
    d = ctx.dequant(h)
    assert np.array_equal(ctx.read(d).view(np.uint32), O.dequant_q4k(blocks, 96, 1024).view(np.uint32))
    ctx.dispose_batch([h, d])


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 200, 2048), (3, 200, 2048), (8, 200, 2048), (12, 200, 2048),
                                   # 43 super-blocks per row: the cp.async ring wraps five times and its last
                                   # stage is partial (43 = 5 x 8 + 3)
                                   (1, 136, 11008), (4, 136, 11008), (1, 72, 8448),
                                   (64, 512, 4096)])  # dequant + the tensor-core matmul (transposed B)
def test_q4k_qmatmul(ctx, M, N, K):
    blocks = O.random_q4k(N, K, 7 + M)
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    h = ctx.upload_quant("Q4_K", blocks, N, K)
    xh = ctx.upload(x)
    y = ctx.qmatmul(xh, h)
    assert max_rel_err(ctx.read(y), O.qmatmul_q4k(blocks, N, K, x)) <= 1e-3
    ctx.dispose_batch([h, xh, y])


@pytest.mark.gpu
def test_q4k_graph_linear(ctx):
    import forge_b200
    N, K, M = 64, 512, 2
    blocks = O.random_q4k(N, K, 11)
    h = ctx.upload_quant("Q4_K", blocks, N, K)
    x = np.random.default_rng(1).standard_normal((M, K)).astype(np.float32)
    g = forge_b200.GraphBuilder()
    ix, iw = g.add_upload((M, K)), g.add_load((N, K), h)
    t = g.add_op("transpose", (K, N), [iw], [N, K])
    y = g.add_op("matmul", (M, N), [ix, t], [M, N, K])
    out = forge_b200.execute_graph(ctx, g.compile()[0], [x])
    assert max_rel_err(ctx.read(out[str(y)]), O.qmatmul_q4k(blocks, N, K, x)) <= 1e-3
    assert np.array_equal(ctx.read(out[str(t)]), O.dequant_q4k(blocks, N, K).T)
    ctx.dispose_batch([out[str(ix)], out[str(t)], out[str(y)], h])


# ---------------------------------------------------------------- Q6_K
def test_q6k_known_answers():
    b = np.zeros(210, np.uint8)
    b[0:128] = 0x21      # ql: low nibble 1, high nibble 2
    b[128:192] = 0xE4    # qh: bits 0-1 = 0, 2-3 = 1, 4-5 = 2, 6-7 = 3
    sc = np.array([1, -2, 3, -4, 5, -6, 7, -8, 9, -10, 11, -12, 13, -14, 15, -16], np.int8)
    b[192:208] = sc.view(np.uint8)
    dh = np.float16(0.5).view(np.uint16)
    b[208], b[209] = dh & 255, dh >> 8
    w = O.dequant_q6k(b.reshape(1, 210), 1, 256)[0]
    q = [-31, -15, 2, 18]  # (1 | 0 << 4), (1 | 1 << 4), (2 | 2 << 4), (2 | 3 << 4), each minus 32
    for h in range(2):
        for quarter in range(4):
            for l in (0, 15, 16, 31):
                want = np.float32(np.float32(0.5) * np.float32(sc[8 * h + l // 16 + 2 * quarter])) * np.float32(q[quarter])
                assert w[128 * h + 32 * quarter + l] == want, (h, quarter, l)


def test_gguf_lists_q6k_tensors(tmp_path):
    import forge_b200
    import gguf_write as GW
    blocks = O.random_q6k(3, 512, 4)
    path = os.path.join(tmp_path, "q6k.gguf")
    GW.write(path, [("general.architecture", GW.V_STR, "llama")], [("output.weight", 14, [512, 3], blocks)])
    with forge_b200.GGUFFile(path) as g:
        t = {t["name"]: t for t in g.tensors()}["output.weight"]
        assert t["dtype"] == "Q6_K" and t["dims"] == (512, 3)
        assert np.array_equal(t["bytes"], blocks.reshape(-1))


@pytest.mark.gpu
def test_q6k_upload_roundtrip_and_exact_dequant(ctx):
    blocks = O.random_q6k(96, 1024, 15)
    h = ctx.upload_quant("Q6_K", blocks, 96, 1024)
    assert np.array_equal(ctx.read_quant_gguf(h), blocks)
    d = ctx.dequant(h)
    assert np.array_equal(ctx.read(d).view(np.uint32), O.dequant_q6k(blocks, 96, 1024).view(np.uint32))
    ctx.dispose_batch([h, d])


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 200, 2048), (3, 200, 2048), (8, 200, 2048), (12, 200, 2048),
                                   # >= 32 super-blocks per row take the 8-in-flight loop; 43 and 33 leave
                                   # tails of 3 and 1 super-blocks
                                   (1, 136, 11008), (4, 136, 11008), (1, 72, 8448),
                                   (64, 512, 4096)])
def test_q6k_qmatmul(ctx, M, N, K):
    blocks = O.random_q6k(N, K, 17 + M)
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    h = ctx.upload_quant("Q6_K", blocks, N, K)
    xh = ctx.upload(x)
    y = ctx.qmatmul(xh, h)
    assert max_rel_err(ctx.read(y), O.qmatmul_q6k(blocks, N, K, x)) <= 1e-3
    ctx.dispose_batch([h, xh, y])
