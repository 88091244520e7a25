"""Quant path on the GPU vs the oracle: bit-exact unpack / dequant / repack,
and the seeded generator + quantizer bit-identical to the CPU recipe."""
import numpy as np
import pytest

import inputs as I
import oracle as O
from forge_b200.errors import AMEVAForgeShapeError, AMEVAForgeValidationError

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("case", ["unpack4", "unpack8"])
def test_unpack_known_answers(ctx, golden, case):
    packed, scales, zeros, b, gs, n = getattr(I, case)()
    h = ctx.unpackQuant(ctx.upload(packed), ctx.upload(scales), ctx.upload(zeros), b, gs, n)
    assert np.array_equal(bits(ctx.read(h)), bits(golden[case + "_expected"]))


@pytest.mark.parametrize("bitw,gs,n", [(4, 32, 1000), (8, 64, 4097), (4, 128, 7), (8, 1, 33), (4, 3, 0)])
def test_unpack_ragged_matches_oracle(ctx, bitw, gs, n):
    rng = np.random.default_rng(n)
    words = max(1, -(-n // (8 if bitw == 4 else 4)))
    groups = max(1, -(-n // gs))
    packed = rng.integers(0, 2**32, words, dtype=np.uint64).astype(np.uint32)
    scales = rng.normal(size=groups).astype(np.float32)
    zeros = rng.integers(0, 16 if bitw == 4 else 256, groups).astype(np.float32)
    h = ctx.unpackQuant(ctx.upload(packed), ctx.upload(scales), ctx.upload(zeros), bitw, gs, n)
    out = ctx.read(h)
    assert out.shape == (n,)
    assert np.array_equal(bits(out), bits(O.unpack_quant(packed, scales, zeros, bitw, gs, n)))


def test_unpack_rejects_bad_arguments(ctx):
    p, s, z = ctx.upload(np.zeros(4, np.uint32)), ctx.upload(np.ones(1, np.float32)), ctx.upload(np.zeros(1, np.float32))
    with pytest.raises(AMEVAForgeValidationError):
        ctx.unpackQuant(p, s, z, 3, 32, 32)
    with pytest.raises(AMEVAForgeShapeError):
        ctx.unpackQuant(p, s, z, 4, 32, 64)  # needs 8 words, 2 groups


@pytest.mark.parametrize("qt,name", [(O.Q4_0, "Q4_0"), (O.Q8_0, "Q8_0")])
@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 96), (64, 4096), (4096, 11008)])
def test_upload_roundtrip_and_dequant_exact(ctx, qt, name, rows, cols):
    w = O.normal(rows * 7 + cols, 0, rows * cols, 0.0, 0.02).reshape(rows, cols)
    blocks = O.quantize(qt, w)
    h = ctx.upload_quant(name, blocks, rows, cols)
    assert np.array_equal(ctx.read_quant_gguf(h), blocks)
    deq = ctx.read(ctx.dequant(h))
    assert np.array_equal(bits(deq), bits(O.dequant(qt, blocks, rows, cols)))
    # and equal to the reference unpack over the mapped operands
    if rows * cols <= 1 << 20:
        packed, scales, zeros = O.gguf_to_ref(qt, blocks)
        ref = O.unpack_quant(packed, scales, zeros, 4 if qt == O.Q4_0 else 8, 32, rows * cols)
        assert np.array_equal(bits(deq).reshape(-1), bits(ref))


def test_upload_quant_validates(ctx):
    with pytest.raises(AMEVAForgeShapeError):
        ctx.upload_quant("Q4_0", np.zeros(18, np.uint8), 1, 48)
    with pytest.raises(AMEVAForgeShapeError):
        ctx.upload_quant("Q4_0", np.zeros(17, np.uint8), 1, 32)


@pytest.mark.parametrize("qt,name", [(O.Q4_0, "Q4_0"), (O.Q8_0, "Q8_0")])
def test_device_synthesis_matches_oracle_recipe(ctx, qt, name):
    rows, cols, seed, row0 = 96, 4096, 0xC0FFEE, 33
    h = ctx.synth_quant(name, rows, cols, seed, row0=row0, std=0.02)
    ref = O.quantize(qt, O.normal(seed, row0 * cols, rows * cols, 0.0, 0.02).reshape(rows, cols))
    assert np.array_equal(ctx.read_quant_gguf(h), ref)


def test_synth_normal_matches_oracle(ctx):
    h = ctx.synth_normal((1000, 37), np.float32, seed=99, offset=5, mean=1.0, std=0.1)
    assert np.array_equal(bits(ctx.read(h)).reshape(-1), bits(O.normal(99, 5, 37000, 1.0, 0.1)))
    h16 = ctx.synth_normal((4096,), np.float16, seed=7, std=0.02)
    assert np.array_equal(ctx.read(h16).view(np.uint16), O.f32_to_f16(O.normal(7, 0, 4096, 0.0, 0.02)))
