"""GPU: long-context decode (4096 and 32768 cached tokens) on the seeded bf16 weights in a
max_seq_len 32896 file, bf16 KV cache.

  * 4096-token prompt against wasiqnauman/cudallm's own ReferenceModel (golden_long_bf16_bf16.npz: the same
    file, the same seeded prompt, bf16 KV): after the prompt the logits are within 2e-2 (the reference test's
    tolerance) and the per-layer residuals of the last prompt step within rel-L2 3e-3 (the bf16-KV residual
    tolerance of the engine tests), and the 8 greedy ids equal the reference's wherever the reference's top-2
    margin is at least 2e-3. Persistent and per-op decode paths, prompt fed by the chunked prefill.
  * 32768 cached tokens (no CPU reference can run that far): the persistent step's split attention (513
    tiles per KV head cut into ranges over many CTAs, merged in range order) against the per-op path's split-K
    kernels, which the kernel tests pin to float64 at 32896 tokens: 4 teacher-forced steps, logits within
    2e-2 and the same argmax; and a reset + rerun of the persistent engine is bit-identical.
  * The two attention forms of the persistent step (one CTA per KV head, or ranges over many CTAs) agree on
    the same tokens at contexts on either side of the switch.
"""
from __future__ import annotations

import numpy as np
import pytest

from cudallm_b200 import synth
from cudallm_b200.engine import Engine

pytestmark = pytest.mark.gpu

LONG_MAX_SEQ = 32896
REF_TOL = 2e-2
RES_TOL = 3e-3
MARGIN = 2e-3


@pytest.fixture(scope="module")
def long_path():
    path, digest = synth.ensure_model("bf16", seed=0, max_seq_len=LONG_MAX_SEQ)
    return path, digest


def _rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("path_kind", ["persistent", "per_op"])
def test_4096_prompt_matches_reference(long_path, golden, path_kind):
    g = golden("long_bf16_bf16")
    path, digest = long_path
    assert digest == str(g["digest"]), "synthetic weights differ from the ones the golden run used"
    prompt = [int(t) for t in g["prompt"]]
    n = len(prompt)
    with Engine(path, kv_dtype="bf16", path_kind=path_kind, max_seq_len=LONG_MAX_SEQ) as eng:
        assert eng.decode_path == path_kind
        eng.prefill(prompt[:-1])
        nxt, lg, res = eng.step_debug(prompt[-1])
        assert eng.pos == n
        ids = [nxt]
        while len(ids) < len(g["ids"]):
            ids.append(eng.step(None)[0])
    ref = g[f"logits_{n - 1}"]
    assert np.abs(lg - ref).max() < REF_TOL
    assert int(np.argmax(lg)) == int(np.argmax(ref))
    ref_res = g[f"res_{n - 1}"]
    for layer in range(ref_res.shape[0]):
        assert _rel_l2(res[layer], ref_res[layer]) < RES_TOL, f"residual {layer}"
    # margins of the generated steps: the last len(ids) entries of the per-step statistics
    margins = g["margin"][-len(g["ids"]):]
    n_cmp = next((i for i, m in enumerate(margins) if m < MARGIN), len(ids))
    assert ids[:n_cmp] == [int(t) for t in g["ids"][:n_cmp]]


@pytest.fixture(scope="module")
def context_32k(long_path):
    """32768 seeded random tokens through the prefill, then 4 fed steps, on both decode paths; and a second
    persistent run after a reset."""
    path, _ = long_path
    toks = synth.prompt_ids(32768 + 4, seed=7)
    out = {}
    for kind, runs in (("persistent", 2), ("per_op", 1)):
        with Engine(path, kv_dtype="bf16", path_kind=kind, max_seq_len=LONG_MAX_SEQ) as eng:
            for r in range(runs):
                eng.reset()
                eng.prefill(toks[:32768])
                assert eng.pos == 32768
                out[(kind, r)] = [eng.step(t, want_logits=True)[1] for t in toks[32768:]]
    return out


def test_32k_persistent_split_attention_matches_per_op(context_32k):
    for a, b in zip(context_32k[("persistent", 0)], context_32k[("per_op", 0)]):
        assert np.abs(a - b).max() < REF_TOL
        assert int(np.argmax(a)) == int(np.argmax(b))


def test_32k_rerun_bit_identical(context_32k):
    for a, b in zip(context_32k[("persistent", 0)], context_32k[("persistent", 1)]):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("dtype", ["bf16", "int4"])
@pytest.mark.parametrize("ctx", [300, 700, 2100])
def test_attention_forms_agree(model_path, dtype, ctx):
    """Knob whole_head_max_tiles forces one CTA per KV head (the largest value) or ranges over many CTAs
    (0) on the same tokens: logits of 3 fed steps within 2e-3 (different summation order of the softmax
    states), the same argmax."""
    path, _ = model_path(dtype)
    toks = synth.prompt_ids(ctx + 3, seed=ctx)
    got = {}
    for form, knob in (("whole", 4096 // 64), ("split", 0)):
        with Engine(path, kv_dtype="bf16") as eng:
            eng.set_knob("whole_head_max_tiles", knob)
            eng.prefill(toks[:ctx])
            got[form] = [eng.step(t, want_logits=True)[1] for t in toks[ctx:]]
    for a, b in zip(got["whole"], got["split"]):
        assert np.abs(a - b).max() < 2e-3
        assert int(np.argmax(a)) == int(np.argmax(b))
