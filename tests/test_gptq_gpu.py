"""GPU: the engine-side quality evaluation of cudallm_b200/gptq.py (evaluate_engine), which runs .cudallm files
through this library's decode engine and compares their teacher-forced logits with a reference file's.

  * a file compared with itself gives zero error, full top-1 agreement and zero KL (the engine is
    deterministic, so the measure has no noise floor of its own);
  * the reference quantiser's int4 file against the bf16 one gives finite, positive error figures.
"""
from __future__ import annotations

import numpy as np
import pytest

from cudallm_b200 import synth
from cudallm_b200.gptq import evaluate_engine

pytestmark = pytest.mark.gpu


def test_self_comparison_is_exact(native_lib):
    bf16, _ = synth.ensure_model("bf16")
    r = evaluate_engine(bf16, [bf16], n_tokens=6)["results"][str(bf16)]
    assert r["logits_rel_l2"] == 0.0 and r["top1_agreement"] == 1.0 and r["mean_kl"] == 0.0


def test_int4_against_bf16(native_lib):
    bf16, _ = synth.ensure_model("bf16")
    int4, _ = synth.ensure_model("int4")
    r = evaluate_engine(bf16, [int4], n_tokens=6)["results"][str(int4)]
    assert np.isfinite(r["logits_rel_l2"]) and r["logits_rel_l2"] > 0.0
    assert 0.0 <= r["top1_agreement"] <= 1.0 and r["mean_kl"] > 0.0
