"""CPU: pins the oracle, the format writer, the quantiser and the synthetic-weight generator against
outputs of wasiqnauman/cudallm's own code (tests/golden/make_golden.py)."""
from __future__ import annotations

import hashlib
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

import tiny_spec
from cudallm_b200 import format as fmt
from cudallm_b200 import synth
from cudallm_b200.quantize import quantize_int4_groups, quantize_int8_rows
from oracle.refmodel import RefModel


def test_quantizers_bit_exact_vs_reference(golden):
    g = golden("quant")
    for k in ("a", "b"):
        w = g[f"{k}_in"]
        q8, s8 = quantize_int8_rows(w)
        np.testing.assert_array_equal(q8, g[f"{k}_q8"])
        np.testing.assert_array_equal(s8.view(np.uint32), g[f"{k}_s8"].view(np.uint32))
        q4, s4 = quantize_int4_groups(w, 128)
        np.testing.assert_array_equal(q4, g[f"{k}_q4"])
        np.testing.assert_array_equal(s4.view(np.uint16), g[f"{k}_s4"].view(np.uint16))


def test_format_writer_bytes_vs_reference(golden, tmp_path):
    p = tmp_path / "f.cudallm"
    fmt.write_cudallm(p, tiny_spec.FORMAT_HEADER, tiny_spec.format_tensors())
    raw = p.read_bytes()
    g = golden("format")
    assert len(raw) == int(g["size"])
    assert hashlib.sha256(raw).hexdigest() == str(g["sha256"])


@pytest.fixture(scope="module")
def tiny_files():
    d = Path(tempfile.mkdtemp(prefix="cllm_tiny_"))
    out = {}
    for dtype, code in (("bf16", 1), ("int8", 3), ("int4", 4)):
        p = d / f"tiny_{dtype}.cudallm"
        fmt.write_cudallm(p, tiny_spec.header(code),
                          tiny_spec.build_tensor_list(dtype, fmt, quantize_int8_rows, quantize_int4_groups))
        out[dtype] = p
    return out


@pytest.mark.parametrize("dtype", ["bf16", "int8", "int4"])
def test_tiny_file_bytes_match_reference_writer(dtype, tiny_files, golden):
    g = golden("tiny")
    assert hashlib.sha256(tiny_files[dtype].read_bytes()).hexdigest() == str(g[f"{dtype}_sha256"])


@pytest.mark.parametrize("dtype,kv", [("bf16", "fp16"), ("int8", "fp16"), ("int4", "fp16"), ("bf16", "bf16")])
@pytest.mark.parametrize("cache_dense", [False, True])
def test_oracle_bit_exact_vs_reference_model(dtype, kv, cache_dense, tiny_files, golden):
    """The restated CPU model reproduces ReferenceModel's logits, residuals and greedy ids exactly."""
    g = golden("tiny")
    ref = RefModel(tiny_files[dtype], kv_dtype=torch.float16 if kv == "fp16" else torch.bfloat16,
                   cache_dense=cache_dense)
    ids = list(tiny_spec.PROMPT)
    got_logits, got_res, got_ids = [], [], []
    step = 0
    while True:
        lg, res = ref.step(ids[step])
        got_logits.append(lg.numpy())
        got_res.append(torch.stack(res).numpy())
        nxt = int(torch.argmax(lg))
        step += 1
        if step >= len(tiny_spec.PROMPT):
            got_ids.append(nxt)
            if len(got_ids) >= tiny_spec.N_NEW:
                break
            ids.append(nxt)
    np.testing.assert_array_equal(np.stack(got_logits), g[f"{dtype}_{kv}_logits_all"])
    np.testing.assert_array_equal(np.stack(got_res), g[f"{dtype}_{kv}_res_all"])
    assert got_ids == g[f"{dtype}_{kv}_ids"].tolist()
    assert ref.greedy(tiny_spec.PROMPT, tiny_spec.N_NEW) == got_ids


def test_synth_generator_reproduces_golden_digest(golden):
    """The seeded Llama-3.2-1B bf16 file regenerates to the digest the reference runs were made on."""
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "m.cudallm"
        digest = synth.write_model(path, "bf16", seed=0, max_seq_len=4096)
        assert digest == str(golden("full_bf16_fp16")["digest"])
        hdr = fmt.read_header(path)
        assert hdr["max_seq_len"] == 4096 and hdr["n_tensors"] == 99
        table = fmt.read_table(path)
        assert [e["name"] for e in table] == fmt.expected_names(16, False)
        w = fmt.load_tensor(path, table[1], mmap=True)[:2048]
        np.testing.assert_array_equal(fmt.bf16_bits_to_f32(w), synth.block_values(0, "tok_embeddings.weight", 0))


@pytest.mark.parametrize("dtype", ["int8", "int4"])
def test_synth_quantized_digest(dtype, golden):
    with tempfile.TemporaryDirectory() as d:
        digest = synth.write_model(Path(d) / "m.cudallm", dtype, seed=0, max_seq_len=4096)
    g = golden(f"full_{dtype}_fp16")
    assert digest == str(g["digest"])
    assert g["quant_blocks_equal"].all()


def test_full_golden_sanity(golden):
    """Internal consistency of the reference runs on the full model (what the GPU tests compare to)."""
    for cfg in ("bf16_fp16", "int8_fp16", "int4_fp16", "bf16_bf16"):
        g = golden(f"full_{cfg}")
        assert g["ids"].shape == (64,)
        assert g["prompt"].tolist() == synth.prompt_ids(32, seed=0)
        lg = g["logits_31"]
        assert int(np.argmax(lg)) == int(g["ids"][0])
        assert g["res_0"].shape == (17, 2048) and g["res_31"].shape == (17, 2048)
        assert np.all(g["margin"] >= 0)
