"""LLMSampler.sample on the device (fg_sample) vs the oracle's statement-by-
statement restatement, and the reference's own known answers
(packages/forge/tests/llm_generation_primitives.test.ts:269-292)."""
import numpy as np
import pytest

import oracle as O


def test_oracle_known_answers():
    """The reference's sampler tests, on the oracle (CPU)."""
    assert O.sample([1.2, 5.8, -0.4, 3.1, 0.9], temperature=0.0) == 1
    for s in range(20):
        assert O.sample([0.1, 10.0, 9.0, 1.0, 0.5], temperature=1.0, top_k=2, seed=s + 1) in (1, 2)
    assert O.sample([100.0, 0.0, -10.0, -20.0], temperature=1.0, top_p=0.95, seed=7) == 0
    # Xorshift32 (s ^= s << 13; s ^= s >>> 17; s ^= s << 5) from seed 1: 270369
    assert O.xorshift32_first(1) == 270369 / 4294967296.0
    assert O.xorshift32_first(0) == O.xorshift32_first(1)  # (seed >>> 0) || 1


def test_oracle_selection_sort_tie_order():
    """The partial selection sort's swaps order ties differently from a stable
    sort: [3, 3, 5] with k = 2 keeps candidates (2, 1), not (2, 0)."""
    lg = [3.0, 3.0, 5.0]
    # spread 32-bit seeds (the first Xorshift32 draw of a small seed is small)
    picks = {O.sample(lg, 1.0, 2, 1.0, (s * 2654435761) & 0xFFFFFFFF) for s in range(1, 200)}
    assert picks == {2, 1}


CASES = [  # (V, temperature, top_k, top_p)
    (5, 0.0, 0, 1.0),
    (1000, 0.8, 0, 1.0),      # full stable sort path
    (1000, 1.0, 40, 1.0),     # selection-sort path
    (1000, 0.7, 40, 0.9),
    (1000, 1.3, 0, 0.8),
    (777, 1.0, 200, 0.95),    # k > 128: stable sort path with a top-k cut
    (4096, 0.9, 128, 1.0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("V,temp,top_k,top_p", CASES)
def test_device_sampler_matches_oracle(ctx, V, temp, top_k, top_p):
    rng = np.random.default_rng(V + top_k)
    rows = 6
    logits = (rng.standard_normal((rows, V)) * 3).astype(np.float32)
    logits[1, :min(8, V - 1)] = logits[1, V - 1]  # ties
    for seed in (1, 12345, 0xDEADBEEF, 0x9E3779B9, 0x7FFFFFFF):
        got = ctx.read(ctx.sample(ctx.upload(logits), temperature=temp, top_k=top_k, top_p=top_p, seed=seed))
        want = [O.sample(logits[r], temp, top_k, top_p, seed) for r in range(rows)]
        assert list(got) == want


@pytest.mark.gpu
def test_device_sampler_reference_cases(ctx):
    assert ctx.read(ctx.sample(ctx.upload(np.array([[1.2, 5.8, -0.4, 3.1, 0.9]], np.float32)), 0.0))[0] == 1
    assert ctx.read(ctx.sample(ctx.upload(np.array([[100.0, 0.0, -10.0, -20.0]], np.float32)), 1.0,
                               top_p=0.95))[0] == 0
    for s in range(10):
        assert ctx.read(ctx.sample(ctx.upload(np.array([[0.1, 10.0, 9.0, 1.0, 0.5]], np.float32)), 1.0,
                                   top_k=2, seed=s + 1))[0] in (1, 2)
