"""GPU: every single-kernel hook through the C ABI against float64 references, with the tolerances of
wasiqnauman/cudallm tests/test_kernels.py (matvec / attention rtol = atol = 1e-4, rmsnorm 1e-5,
RoPE q atol 1e-5 and K within 1 fp16 ulp, V bit-exact, argmax exact)."""
from __future__ import annotations

import numpy as np
import pytest

from cudallm_b200 import engine as E
from cudallm_b200.synth import llama3_inv_freq
from oracle import kernels64 as K

pytestmark = pytest.mark.gpu

NH, NKV, HD, MAX_SEQ = 32, 8, 64, 4096


@pytest.fixture(autouse=True)
def _lib(native_lib):
    return native_lib


def test_matvec_naive_bf16_store():
    rows, cols = 1024, 2048
    bits, _, w64 = K.matvec_operands("bf16", rows, cols, seed=10)
    x = np.random.default_rng(10).standard_normal(cols).astype(np.float32)
    y = E.kernel_matvec("naive", "bf16", "store", 0, 0, bits, None, x, None, 1e-5, None, rows, cols)
    assert np.allclose(y, w64 @ x.astype(np.float64), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("shape", [(1024, 2048), (2048, 8192)], ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("rpb", [1, 2, 4, 8])
@pytest.mark.parametrize("fuse_norm", [0, 1])
@pytest.mark.parametrize("epilogue", ["store", "add", "swiglu"])
@pytest.mark.parametrize("wtype", ["bf16", "int8", "int4"])
def test_matvec_opt(wtype, epilogue, fuse_norm, rpb, shape):
    rows, cols = shape
    eps = 1e-5
    w, scales, w64 = K.matvec_operands(wtype, rows, cols, seed=20 + rows + cols)
    rng = np.random.default_rng(21 + rows)
    x = rng.standard_normal(cols).astype(np.float32)
    norm_w = rng.uniform(0.5, 1.5, cols).astype(np.float32)
    out_rows = rows // 2 if epilogue == "swiglu" else rows
    y_init = rng.standard_normal(out_rows).astype(np.float32) if epilogue == "add" else None
    y = E.kernel_matvec("opt", wtype, epilogue, fuse_norm, rpb, w, scales, x, norm_w if fuse_norm else None, eps, y_init,
                        rows, cols)
    ref = K.matvec64(w64, x, epilogue, norm_w if fuse_norm else None, eps, y_init)
    assert np.allclose(y, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("wtype", ["bf16", "int8", "int4"])
@pytest.mark.parametrize("shape", [(3072, 2048), (16384, 2048), (2048, 8192), (1000, 1024), (37, 4096)],
                         ids=lambda s: f"{s[0]}x{s[1]}")
def test_matvec_opt_engine_shapes_default_rpb(wtype, shape):
    """The engine's shapes (and ragged ones) with the default tile size; rows not a multiple of anything."""
    rows, cols = shape
    ep = "swiglu" if rows == 16384 else "store"
    w, scales, w64 = K.matvec_operands(wtype, rows, cols, seed=rows + 3 * cols)
    x = np.random.default_rng(5).standard_normal(cols).astype(np.float32)
    nw = np.random.default_rng(6).uniform(0.5, 1.5, cols).astype(np.float32)
    y = E.kernel_matvec("opt", wtype, ep, 1, 0, w, scales, x, nw, 1e-5, None, rows, cols)
    assert np.allclose(y, K.matvec64(w64, x, ep, nw, 1e-5, None), rtol=1e-4, atol=1e-4)


def test_matvec_opt_deterministic():
    w, scales, _ = K.matvec_operands("int4", 2048, 8192, seed=3)
    x = np.random.default_rng(4).standard_normal(8192).astype(np.float32)
    a = E.kernel_matvec("opt", "int4", "store", 0, 0, w, scales, x, None, 1e-5, None, 2048, 8192)
    for rpb in (1, 8):
        b = E.kernel_matvec("opt", "int4", "store", 0, rpb, w, scales, x, None, 1e-5, None, 2048, 8192)
        np.testing.assert_array_equal(a, b)  # tile shape does not change any result bit


def test_rmsnorm():
    n, eps = 2048, 1e-5
    rng = np.random.default_rng(11)
    x = rng.standard_normal(n).astype(np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    assert np.allclose(E.kernel_rmsnorm(x, w, eps), K.rmsnorm64(x, w, eps), rtol=1e-5, atol=1e-5)


SENTINEL = np.float16(-7.25)


@pytest.mark.parametrize("pos", [0, 1, 777, 4095])
@pytest.mark.parametrize("fused", [0, 1])
def test_rope_kv(fused, pos):
    rng = np.random.default_rng(12 + pos)
    inv_freq = llama3_inv_freq()
    qkv = rng.standard_normal((NH + 2 * NKV) * HD).astype(np.float32)
    k_cache = np.full((NKV, MAX_SEQ, HD), SENTINEL, dtype=np.float16)
    v_cache = np.full((NKV, MAX_SEQ, HD), SENTINEL, dtype=np.float16)
    out_qkv, k_out, v_out = E.kernel_rope_kv(fused, qkv, inv_freq, pos, k_cache, v_cache, NH, NKV, HD, MAX_SEQ)
    k_out = k_out.reshape(NKV, MAX_SEQ, HD)
    v_out = v_out.reshape(NKV, MAX_SEQ, HD)
    q_ref = K.rope64(qkv[:NH * HD].astype(np.float64).reshape(NH, HD), inv_freq, pos)
    k_ref = K.rope64(qkv[NH * HD:(NH + NKV) * HD].astype(np.float64).reshape(NKV, HD), inv_freq, pos)
    v32 = qkv[(NH + NKV) * HD:].reshape(NKV, HD)
    assert np.allclose(out_qkv[:NH * HD].reshape(NH, HD), q_ref, rtol=0, atol=1e-5)
    if not fused:
        assert np.allclose(out_qkv[NH * HD:(NH + NKV) * HD].reshape(NKV, HD), k_ref, rtol=0, atol=1e-5)
        np.testing.assert_array_equal(out_qkv[(NH + NKV) * HD:], qkv[(NH + NKV) * HD:])
    assert np.all(K.fp16_ulp_diff(k_out[:, pos, :], k_ref.astype(np.float16)) <= 1)
    np.testing.assert_array_equal(v_out[:, pos, :], v32.astype(np.float16))
    others = np.ones(MAX_SEQ, dtype=bool)
    others[pos] = False
    assert np.all(k_out[:, others, :] == SENTINEL)
    assert np.all(v_out[:, others, :] == SENTINEL)


@pytest.fixture(scope="module")
def attn_data():
    rng = np.random.default_rng(13)
    q = rng.standard_normal(NH * HD).astype(np.float32)
    k = rng.standard_normal((NKV, MAX_SEQ, HD)).astype(np.float16)
    v = rng.standard_normal((NKV, MAX_SEQ, HD)).astype(np.float16)
    return q, k, v


@pytest.mark.parametrize("ctx", [1, 7, 63, 64, 65, 128, 129, 1000, 4096])
@pytest.mark.parametrize("impl", ["naive", "opt"])
def test_attention(impl, ctx, attn_data):
    q, k, v = attn_data
    out = E.kernel_attention(impl, q, k, v, ctx, NH, NKV, HD, MAX_SEQ)
    assert np.allclose(out, K.attention64(q, k, v, ctx, NH, NKV), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("ctx", [32768, 32896])
def test_attention_long_context(ctx):
    """The 32K-token configuration (split into 514 tiles; max_seq = 32768 + 128)."""
    max_seq = 32896
    rng = np.random.default_rng(ctx)
    q = rng.standard_normal(NH * HD).astype(np.float32)
    k = rng.standard_normal((NKV, max_seq, HD)).astype(np.float16)
    v = rng.standard_normal((NKV, max_seq, HD)).astype(np.float16)
    ref = K.attention64(q, k, v, ctx, NH, NKV)
    for impl in ("opt", "naive"):
        out = E.kernel_attention(impl, q, k, v, ctx, NH, NKV, HD, max_seq)
        assert np.allclose(out, ref, rtol=1e-4, atol=1e-4), impl


def test_attention_peaked_scores():
    """One dominant key per head: exercises the max-subtraction and the split merge."""
    q = np.full(NH * HD, 0.5, dtype=np.float32)
    k = np.zeros((NKV, MAX_SEQ, HD), dtype=np.float16)
    v = np.random.default_rng(2).standard_normal((NKV, MAX_SEQ, HD)).astype(np.float16)
    k[:, 700, :] = 8.0
    out = E.kernel_attention("opt", q, k, v, 1000, NH, NKV, HD, MAX_SEQ)
    assert np.allclose(out, K.attention64(q, k, v, 1000, NH, NKV), rtol=1e-4, atol=1e-4)


def test_silu_mul():
    inter = 8192
    gu = (np.random.default_rng(14).standard_normal(2 * inter) * 2).astype(np.float32)
    assert np.allclose(E.kernel_silu_mul(gu), K.silu_mul64(gu), rtol=1e-5)


VOCAB = 128256


def test_argmax_random():
    logits = np.random.default_rng(15).standard_normal(VOCAB).astype(np.float32)
    assert E.kernel_argmax(logits) == int(np.argmax(logits))


def test_argmax_tie_lowest_index():
    logits = np.random.default_rng(16).standard_normal(VOCAB).astype(np.float32)
    logits[5] = logits[100000] = 50.0
    assert E.kernel_argmax(logits) == 5


def test_argmax_last_index():
    logits = np.random.default_rng(17).standard_normal(VOCAB).astype(np.float32)
    logits[-1] = 50.0
    assert E.kernel_argmax(logits) == VOCAB - 1


@pytest.mark.parametrize("n", [1, 255, 257, 75776, VOCAB])
def test_argmax_all_equal_and_sizes(n):
    assert E.kernel_argmax(np.zeros(n, np.float32)) == 0
    x = np.full(n, -np.inf, dtype=np.float32)
    x[n // 2] = -1e30
    assert E.kernel_argmax(x) == n // 2
