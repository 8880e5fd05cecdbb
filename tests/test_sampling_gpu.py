"""GPU: top-k / top-p sampling fused into the persistent step (cudallm_set_sampling).

Each step returns the unchanged logits and the drawn token; the oracle's rule (oracle/sampling.py) applied
to those logits must pick the same token, except where float32 rounding of exp could move the draw across
a cumulative boundary (oracle margin below MARGIN: skipped, and counted so that most steps are checked).
top_k = 1 must give the greedy ids; a rerun with the same seed reproduces the tokens."""
from __future__ import annotations

import numpy as np
import pytest

from cudallm_b200 import synth
from cudallm_b200.engine import CudaLLMError, Engine
from oracle import sampling as S

pytestmark = pytest.mark.gpu

MARGIN = 1e-4
PROMPT = 16


def _run(path, dtype_kv, temperature, top_k, top_p, seed, n, path_kind="persistent"):
    toks = synth.prompt_ids(PROMPT, seed=3)
    out = []
    with Engine(path, kv_dtype=dtype_kv, path_kind=path_kind) as eng:
        eng.set_sampling(temperature, top_k, top_p, seed)
        for t in toks[:-1]:
            eng.step(t)
        nxt, lg = eng.step(toks[-1], want_logits=True)
        pos = PROMPT - 1
        for _ in range(n):
            out.append((pos, nxt, lg))
            nxt, lg = eng.step(None, want_logits=True)
            pos += 1
    return out


@pytest.mark.parametrize("dtype", ["bf16", "int4"])
@pytest.mark.parametrize("temperature,top_k,top_p,seed", [(1.0, 0, 1.0, 1), (0.7, 40, 0.9, 2), (1.5, 8, 0.5, 3)])
def test_sampled_tokens_match_the_rule(model_path, dtype, temperature, top_k, top_p, seed):
    path, _ = model_path(dtype)
    steps = _run(path, "bf16", temperature, top_k, top_p, seed, 24)
    checked = 0
    for pos, tok, lg in steps:
        want, margin = S.draw(lg, temperature, top_k, top_p, seed, pos)
        if margin < MARGIN:
            continue
        assert tok == want, f"position {pos}"
        checked += 1
    assert checked >= 20


def test_top1_is_greedy(model_path):
    path, _ = model_path("bf16")
    sampled = _run(path, "bf16", 0.9, 1, 1.0, 7, 16)
    greedy = _run(path, "bf16", 0.0, 0, 1.0, 0, 16)
    assert [t for _, t, _ in sampled] == [t for _, t, _ in greedy]
    for _, tok, lg in sampled:
        assert tok == S.greedy(lg)


def test_rerun_reproduces_and_seed_matters(model_path):
    path, _ = model_path("bf16")
    a = [t for _, t, _ in _run(path, "bf16", 1.2, 0, 1.0, 11, 16)]
    b = [t for _, t, _ in _run(path, "bf16", 1.2, 0, 1.0, 11, 16)]
    c = [t for _, t, _ in _run(path, "bf16", 1.2, 0, 1.0, 12, 16)]
    assert a == b
    assert a != c


def test_sampling_validation(model_path):
    path, _ = model_path("bf16")
    with Engine(path, kv_dtype="bf16") as eng:
        for args in [(-1.0, 0, 1.0), (1.0, 65, 1.0), (1.0, -1, 1.0), (1.0, 0, 0.0), (1.0, 0, 1.5), (float("nan"), 0, 1.0)]:
            with pytest.raises(CudaLLMError) as ei:
                eng.set_sampling(*args)
            assert ei.value.code == 1
    with Engine(path, kv_dtype="bf16", path_kind="per_op") as eng:
        eng.set_sampling(0.0)  # greedy is every path's rule
        with pytest.raises(CudaLLMError) as ei:
            eng.set_sampling(1.0)
        assert ei.value.code == 1
