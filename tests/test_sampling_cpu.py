"""CPU: the sampling rule's restatement (oracle/sampling.py) and its binding.

The reference has no sampling (src/kernels/argmax.cu is its only next-token rule), so the oracle is pinned
where the two rules meet: top_k = 1 (any temperature) and a vanishing nucleus give the reference's argmax,
lowest index on ties. Beyond that the tests check the rule's own properties: draws follow the softmax of the
top-k logits, the nucleus cut, and the draw depends only on (seed, position)."""
from __future__ import annotations

import numpy as np
import pytest

from cudallm_b200 import abi
from oracle import sampling as S


def test_top1_and_tiny_nucleus_are_the_reference_argmax():
    rng = np.random.default_rng(1)
    for trial in range(50):
        logits = rng.normal(size=4096).astype(np.float32)
        if trial % 5 == 0:  # ties: the lowest index wins
            logits[[7, 300, 2000]] = logits.max() + 1.0
        for seed in (0, 17):
            assert S.draw(logits, 0.7, 1, 1.0, seed, trial)[0] == S.greedy(logits)
            assert S.draw(logits, 1.3, 64, 1e-6, seed, trial)[0] == S.greedy(logits)


def test_uniform_draw_is_a_function_of_seed_and_position():
    u = [S.sample_uniform(5, p) for p in range(1000)]
    assert all(0.0 <= x < 1.0 for x in u)
    assert u == [S.sample_uniform(5, p) for p in range(1000)]
    assert u != [S.sample_uniform(6, p) for p in range(1000)]
    assert abs(float(np.mean(u)) - 0.5) < 0.03


def test_draws_follow_the_top_k_softmax():
    logits = np.full(1000, -30.0, dtype=np.float32)
    logits[[3, 10, 500, 999]] = [2.0, 1.0, 0.5, 0.0]
    t = 0.8
    expect = np.exp(np.array([2.0, 1.0, 0.5, 0.0]) / t)
    expect /= expect.sum()
    n = 20000
    counts = {3: 0, 10: 0, 500: 0, 999: 0}
    for pos in range(n):
        tok, _ = S.draw(logits, t, 4, 1.0, 123, pos)
        counts[tok] += 1
    got = np.array([counts[i] for i in (3, 10, 500, 999)]) / n
    assert np.abs(got - expect).max() < 0.015


def test_nucleus_cut():
    logits = np.zeros(100, dtype=np.float32)
    logits[:4] = [3.0, 2.0, 1.0, 0.0]
    w = np.exp(np.array([3.0, 2.0, 1.0, 0.0]))
    p_two = float(w[:2].sum() / w.sum())
    seen = {S.draw(logits, 1.0, 4, p_two - 1e-3, 9, pos)[0] for pos in range(2000)}
    assert seen == {0, 1}


def test_binding_declares_set_sampling():
    args, ret = abi.declarations()[1]["cudallm_set_sampling"]
    assert len(args) == 5


@pytest.mark.parametrize("v", [-3.5, -0.0, 0.0, 1e-30, 2.0, 7e30])
def test_order_key_is_monotonic(v):
    # the candidate key of the kernel (kernels/sampling.cuh), restated: larger value -> larger key
    def key(x):
        u = int(np.float32(x).view(np.uint32))
        return (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)
    assert key(v) < key(np.nextafter(np.float32(v), np.float32(np.inf)))
