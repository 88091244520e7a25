"""Fused dequant-GEMV / GEMM vs the oracle (dequant + double-accumulated
x W^T).  Bar: max |err| <= 1e-3 * ||ref||_inf (fp32 accumulation)."""
import numpy as np
import pytest

import oracle as O
from conftest import max_rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


def run(ctx, qt, name, N, K, M, seed):
    w = O.normal(seed, 0, N * K, 0.0, 0.02).reshape(N, K)
    blocks = O.quantize(qt, w)
    x = O.normal(seed + 1, 0, M * K, 0.0, 1.0).reshape(M, K)
    y = ctx.read(ctx.qmatmul(ctx.upload(x), ctx.upload_quant(name, blocks, N, K)))
    ref = O.qmatmul(qt, blocks, N, K, x)
    return y, ref


def test_q8_0_gemv_4096(ctx):
    """Q8_0 4096x4096 dequant-GEMV, batch 1, fp32 activations ~N(0,1)."""
    y, ref = run(ctx, O.Q8_0, "Q8_0", 4096, 4096, 1, 11)
    assert max_rel_err(y, ref) <= TOL


@pytest.mark.parametrize("N,K", [(11008, 4096), (4096, 11008)])
@pytest.mark.parametrize("M", [1, 8, 32, 128])
def test_q4_0_llama_shapes(ctx, N, K, M):
    """Q4_0 4096x11008 / 11008x4096 at batch 1, 8, 32, 128."""
    y, ref = run(ctx, O.Q4_0, "Q4_0", N, K, M, 1000 + M)
    assert max_rel_err(y, ref) <= TOL


@pytest.mark.parametrize("N,K", [(11008, 4096), (4096, 11008)])
@pytest.mark.parametrize("M", [8, 32, 128, 200])
def test_q8_0_gemm_llama_shapes(ctx, N, K, M):
    """Q8_0 on the tensor-core GEMM (fp16 q * d in shared memory, fp32 accumulation in TMEM): batch 8, 32,
    128 and 200 (two 128-token tiles)."""
    y, ref = run(ctx, O.Q8_0, "Q8_0", N, K, M, 2000 + M)
    assert max_rel_err(y, ref) <= TOL


@pytest.mark.parametrize("N,K,M", [(66, 1056, 9), (300, 160, 40), (130, 2080, 130), (1, 32, 5)])
def test_q8_0_gemm_ragged(ctx, N, K, M):
    """Q8_0 GEMM with K not a multiple of 128 (the last quad's codes and scales read as zero past K),
    N not a multiple of 128 and token tiles cut short."""
    y, ref = run(ctx, O.Q8_0, "Q8_0", N, K, M, 3 * N + K + M)
    assert y.shape == (M, N)
    assert max_rel_err(y, ref) <= TOL


@pytest.mark.parametrize("qt,name", [(O.Q4_0, "Q4_0"), (O.Q8_0, "Q8_0")])
@pytest.mark.parametrize("N,K,M", [(1, 32, 1), (3, 64, 2), (5, 96, 3), (66, 1056, 4), (130, 2048, 5),
                                   (2, 32, 17), (1000, 512, 1), (32000, 2048, 1)])
def test_ragged_shapes(ctx, qt, name, N, K, M):
    y, ref = run(ctx, qt, name, N, K, M, N * 31 + K + M)
    assert y.shape == (M, N)
    assert max_rel_err(y, ref) <= TOL


def test_leading_dims_kept(ctx):
    w = O.quantize(O.Q4_0, O.normal(3, 0, 64 * 128, 0.0, 0.02).reshape(64, 128))
    x = O.normal(4, 0, 2 * 3 * 128, 0.0, 1.0).reshape(2, 3, 128)
    y = ctx.read(ctx.qmatmul(ctx.upload(x), ctx.upload_quant("Q4_0", w, 64, 128)))
    assert y.shape == (2, 3, 64)
    assert max_rel_err(y, O.qmatmul(O.Q4_0, w, 64, 128, x)) <= TOL
