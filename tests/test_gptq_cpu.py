"""CPU: the GPTQ calibrated-int4 quantiser (cudallm_b200/gptq.py).

  * with an isotropic Hessian (H = c I) error feedback has nowhere to go, so GPTQ must give exactly the
    reference quantiser's RTN codes and scales (quantize.py, pinned by test_oracle_golden against the
    reference's own outputs): this pins the layout, the rounding and the scale rule;
  * on correlated inputs GPTQ lowers the calibration objective ||(W - Q) X||^2 well below RTN's;
  * inputs that never vary (zero Hessian diagonal) give zero weights;
  * a whole calibration on a small Llama-shaped file writes a valid int4 .cudallm (tensor order, dtypes,
    header) with a lower calibration error than RTN, and the evaluation runs on it.
"""
from __future__ import annotations

import numpy as np
import pytest

from cudallm_b200 import format as fmt
from cudallm_b200.gptq import calibrate, evaluate, gptq_int4
from cudallm_b200.quantize import dequantize_int4_groups, quantize_int4_groups, unpack_int4


def _weights(rows: int, cols: int, seed: int) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal((rows, cols)) * 0.02).astype(np.float32)


def test_isotropic_hessian_gives_rtn_exactly():
    w = _weights(40, 384, 1)
    packed, scales = gptq_int4(w, 3.0 * np.eye(384))
    rp, rs = quantize_int4_groups(w)
    assert packed.dtype == np.uint8 and scales.dtype == np.float16
    np.testing.assert_array_equal(packed, rp)
    np.testing.assert_array_equal(scales, rs)


def test_correlated_inputs_lower_the_weighted_error():
    rng = np.random.default_rng(2)
    rows, cols, T = 64, 512, 1024
    w = _weights(rows, cols, 3)
    mix = rng.standard_normal((cols, cols)) / np.sqrt(cols)
    x = rng.standard_normal((T, cols)) @ mix + 0.3 * rng.standard_normal((T, cols))
    packed, scales = gptq_int4(w, x.T @ x)
    q = unpack_int4(packed)
    assert q.min() >= -8 and q.max() <= 7
    wq = dequantize_int4_groups(packed, scales)
    wr = dequantize_int4_groups(*quantize_int4_groups(w))
    err = lambda a: float(np.sum(((w - a) @ x.T) ** 2))  # noqa: E731
    assert err(wq) < 0.7 * err(wr)


def test_constant_inputs_give_zero_weights():
    w = _weights(8, 256, 4)
    h = np.eye(256)
    h[5, 5] = 0.0
    h[200, 200] = 0.0
    q = unpack_int4(gptq_int4(w, h)[0])
    assert np.all(q[:, 5] == 0) and np.all(q[:, 200] == 0)


def test_rejects_bad_shapes():
    with pytest.raises(ValueError):
        gptq_int4(_weights(4, 200, 5), np.eye(200))
    with pytest.raises(ValueError):
        gptq_int4(_weights(4, 256, 5), np.eye(128))


def _tiny_bf16(path, layers=2, hidden=256, inter=512, heads=4, kv=2, hd=64, vocab=512):
    rng = np.random.default_rng(9)
    header = {"weight_dtype": fmt.WEIGHT_BF16, "hidden_size": hidden, "intermediate_size": inter, "n_layers": layers,
              "n_heads": heads, "n_kv_heads": kv, "head_dim": hd, "vocab_size": vocab, "max_seq_len": 256,
              "rms_eps": 1e-5, "rope_theta": 500000.0, "group_size": 0}
    shapes = {"wqkv": ((heads + 2 * kv) * hd, hidden), "wo": (hidden, heads * hd), "w_gate_up": (2 * inter, hidden),
              "w_down": (hidden, inter)}
    bf = lambda r, c: fmt.f32_to_bf16_bits((rng.standard_normal((r, c)) * 0.02).astype(np.float32)).tobytes()  # noqa: E731
    inv = (1.0 / 500000.0 ** (np.arange(hd // 2) * 2.0 / hd)).astype(np.float32)
    tensors = []
    for name in fmt.expected_names(layers, False):
        if name == "rope.inv_freq":
            tensors.append((name, fmt.F32, hd // 2, 1, inv.tobytes()))
        elif name == "tok_embeddings.weight":
            tensors.append((name, fmt.BF16, vocab, hidden, bf(vocab, hidden)))
        elif name.endswith("norm.weight"):
            tensors.append((name, fmt.F32, hidden, 1, np.ones(hidden, np.float32).tobytes()))
        else:
            r, c = shapes[name.split(".")[2]]
            tensors.append((name, fmt.BF16, r, c, bf(r, c)))
    fmt.write_cudallm(path, header, tensors)


def test_calibrate_small_model(tmp_path):
    src, dst = tmp_path / "tiny_bf16.cudallm", tmp_path / "tiny_gptq.cudallm"
    _tiny_bf16(src)
    summary = calibrate(src, dst, n_tokens=256, seq_len=64, seed=7, log=lambda m: None)
    assert summary["calibration_tokens"] == 256
    assert 0.0 < summary["weighted_error_gptq_over_rtn"] < 1.0
    hdr = fmt.read_header(dst)
    assert hdr["weight_dtype"] == fmt.WEIGHT_INT4 and hdr["group_size"] == 128
    table = fmt.read_table(dst)
    assert [e["name"] for e in table] == fmt.expected_names(2, True)
    for e in table:
        if e["name"].endswith(".weight") and "norm" not in e["name"]:
            assert e["dtype"] == fmt.I4X2
        if e["name"].endswith(".scales"):
            assert e["dtype"] == fmt.F16 and e["cols"] == (512 if "w_down" in e["name"] else 256) // 128
        assert e["nbytes"] == fmt.expected_nbytes(e["dtype"], e["rows"], e["cols"])
    res = evaluate(src, [dst], n_tokens=16)["results"][str(dst)]
    assert np.isfinite(res["logits_rel_l2"]) and 0.0 <= res["top1_agreement"] <= 1.0 and res["mean_kl"] >= 0.0
