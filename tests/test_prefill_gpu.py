"""GPU: prompt prefill (cudallm_prefill, cudallm_batch_prefill): 64 prompt tokens per batched tensor-core step,
every row of the step one position of the same sequence.

The reference has no prefill: it feeds a prompt one cudallm_step at a time (src/tools/cudallm_bench.cpp:70,
src/engine/engine.cpp:117). So prefill must give what stepping gives:
  * the seeded golden prompt (32 tokens) prefilled, then 64 greedy tokens, reproduces the reference's
    ReferenceModel ids (golden_full_*) and its logits after the prompt within 2e-2 (its own tolerance), for
    bf16, int8 (which steps the prompt through the decode path) and int4 weights;
  * against the engine stepping the same tokens, the logits after the prompt are within 2e-3 (fp32 on both
    paths; the batched GEMMs carry activations as bf16 hi + lo planes), across chunk boundaries and when a
    prefill continues a sequence that earlier steps or prefills started;
  * in a batch engine, prefilling one sequence leaves every other row bitwise as it would have been.
"""
from __future__ import annotations

import numpy as np
import pytest

from cudallm_b200.engine import BatchEngine, CudaLLMError, Engine

pytestmark = pytest.mark.gpu

REF_TOL = 2e-2
PATH_TOL = 2e-3


@pytest.mark.parametrize("dtype", ["bf16", "int8", "int4"])
def test_prefill_golden_prompt_matches_reference(model_path, golden, dtype):
    g = golden(f"full_{dtype}_fp16")
    path, digest = model_path(dtype)
    assert digest == str(g["digest"])
    prompt = [int(t) for t in g["prompt"]]
    with Engine(path) as eng:
        nxt, lg = eng.prefill(prompt, want_logits=True)
        assert eng.pos == len(prompt)
        assert np.abs(lg - g[f"logits_{len(prompt) - 1}"]).max() < REF_TOL
        ids = [nxt]
        while len(ids) < len(g["ids"]):
            ids.append(eng.step(None)[0])
    assert ids == [int(t) for t in g["ids"]]


@pytest.mark.parametrize("dtype", ["bf16", "int4"])
@pytest.mark.parametrize("path_kind", ["persistent", "per_op"])
def test_prefill_matches_stepping_across_chunks(model_path, dtype, path_kind):
    """Prefills of 100 tokens (a full 64-token chunk and a partial one), then 3 fed steps, then a prefill of
    61 more: logits after each prefill against an engine that stepped the same 100 / 164 tokens."""
    path, _ = model_path(dtype)
    rng = np.random.default_rng(31)
    a = [int(t) for t in rng.integers(0, 128256, 100)]
    c = [int(t) for t in rng.integers(0, 128256, 3)]
    b = [int(t) for t in rng.integers(0, 128256, 61)]
    with Engine(path, path_kind=path_kind) as pre, Engine(path, path_kind=path_kind) as ref:
        _, lg1 = pre.prefill(a, want_logits=True)
        for t in a[:-1]:
            ref.step_async(t)
        _, r1 = ref.step(a[-1], want_logits=True)
        assert np.abs(lg1 - r1).max() < PATH_TOL
        for t in c:
            _, x = pre.step(t, want_logits=True)
            _, y = ref.step(t, want_logits=True)
            assert np.abs(x - y).max() < PATH_TOL
        n2, lg2 = pre.prefill(b, want_logits=True)
        assert pre.pos == 164
        for t in b[:-1]:
            ref.step_async(t)
        _, r2 = ref.step(b[-1], want_logits=True)
        assert np.abs(lg2 - r2).max() < PATH_TOL
        assert n2 == int(np.argmax(lg2))


def test_prefill_rejects_what_does_not_fit(model_path):
    path, _ = model_path("bf16")
    with Engine(path, max_seq_len=128) as eng:
        with pytest.raises(CudaLLMError) as e:
            eng.prefill(np.zeros(129, dtype=np.int32))
        assert e.value.code == 5
        with pytest.raises(CudaLLMError) as e:
            eng.prefill([1, 2, 128256])
        assert e.value.code == 1
        assert eng.pos == 0
        eng.prefill(np.ones(128, dtype=np.int32))
        assert eng.pos == 128


@pytest.mark.parametrize("dtype", ["bf16", "int4"])
def test_batch_prefill_leaves_other_rows_untouched(model_path, dtype):
    """Run A: 64 rows step 10 tokens each. Run B: the same rows step 5, sequence 7 is prefilled with 70 more
    tokens, then every row steps its next 5 tokens. Rows other than 7 end bitwise equal to run A; row 7 agrees
    with a batch-1 engine fed its 5 + 70 + 5 tokens."""
    path, _ = model_path(dtype)
    rng = np.random.default_rng(8)
    toks = rng.integers(0, 128256, (10, 64)).astype(np.int32)
    extra = [int(t) for t in rng.integers(0, 128256, 70)]
    with BatchEngine(path, n_seq=64, max_seq_len=256) as eng:
        for i in range(9):
            eng.step_async(toks[i])
        _, la = eng.step(toks[9], want_logits=True)
    with BatchEngine(path, n_seq=64, max_seq_len=256) as eng:
        for i in range(5):
            eng.step_async(toks[i])
        eng.prefill(7, extra)
        assert eng.pos(7) == 75 and eng.pos(6) == 5
        for i in range(5, 9):
            eng.step_async(toks[i])
        _, lb = eng.step(toks[9], want_logits=True)
    others = [r for r in range(64) if r != 7]
    assert np.array_equal(la[others], lb[others])
    with Engine(path, max_seq_len=256) as one:
        for t in [int(x) for x in toks[:5, 7]] + extra + [int(x) for x in toks[5:9, 7]]:
            one.step_async(t)
        _, ref = one.step(int(toks[9, 7]), want_logits=True)
    assert np.abs(lb[7] - ref).max() < PATH_TOL
