"""GPU: the batched path's tensor-core GEMM (tcgen05, bf16 operands, fp32 accumulation) through its C-ABI
hook, against float64 products of the same bf16 values. Shapes cover full and partial 128-row tiles,
partial batches, K split evenly and unevenly over several CTA rows, the hi + lo activation planes that
carry an fp32 activation, and the three epilogues."""
from __future__ import annotations

import numpy as np
import pytest

from cudallm_b200 import engine as E
from cudallm_b200.format import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib(native_lib):
    return native_lib


def _operands(n, k, batch, seed):
    rng = np.random.default_rng(seed)
    w = f32_to_bf16_bits((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    x = f32_to_bf16_bits(rng.standard_normal((batch, k)).astype(np.float32))
    return w, x, bf16_bits_to_f32(w).astype(np.float64), bf16_bits_to_f32(x).astype(np.float64)


def _close(y, ref):
    scale = max(1.0, float(np.abs(ref).max()))
    np.testing.assert_allclose(y, ref, rtol=1e-4, atol=2e-4 * scale)


@pytest.mark.parametrize("n,k,batch,ksplit", [
    (128, 64, 64, 1),       # one tile, one K chunk
    (256, 2048, 64, 1),
    (3072, 2048, 64, 8),    # QKV shape, split K
    (3072, 2048, 64, 6),    # uneven split: 32 chunks over 6 rows
    (2048, 2048, 64, 9),    # o_proj shape, uneven split
    (2048, 8192, 64, 9),    # down shape, uneven split
    (200, 256, 5, 2),       # ragged rows and batch
    (1000, 2048, 17, 4),
    (128256 // 32, 2048, 64, 1),  # a slice of the lm_head shape
], ids=lambda v: str(v))
def test_gemm_store(n, k, batch, ksplit):
    w, x, w64, x64 = _operands(n, k, batch, seed=n + k + batch)
    y = E.kernel_gemm(w, x, ksplit=ksplit)
    _close(y, x64 @ w64.T)


def test_gemm_hi_lo_planes_carry_fp32_activations():
    n, k, batch = 512, 2048, 64
    rng = np.random.default_rng(11)
    w = f32_to_bf16_bits((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    x32 = rng.standard_normal((batch, k)).astype(np.float32)
    hi = f32_to_bf16_bits(x32)
    lo = f32_to_bf16_bits(x32 - bf16_bits_to_f32(hi))
    y = E.kernel_gemm(w, hi, x_lo_bits=lo, ksplit=4)
    ref = x32.astype(np.float64) @ bf16_bits_to_f32(w).astype(np.float64).T
    # hi + lo keeps ~16 mantissa bits of x: far closer to the fp32 product than the bf16 rounding alone.
    np.testing.assert_allclose(y, ref, rtol=1e-4, atol=1e-4)
    y_hi = E.kernel_gemm(w, hi, ksplit=4)
    assert np.abs(y - ref).max() * 20 < np.abs(y_hi - ref).max()


def test_gemm_add_accumulates_into_y():
    n, k, batch = 384, 1024, 33
    w, x, w64, x64 = _operands(n, k, batch, seed=5)
    y0 = np.random.default_rng(6).standard_normal((batch, n)).astype(np.float32)
    y = E.kernel_gemm(w, x, ksplit=2, epilogue="add", y=y0)
    _close(y, y0.astype(np.float64) + x64 @ w64.T)


def test_gemm_swiglu():
    n, k, batch = 2 * 512, 2048, 64
    w, x, w64, x64 = _operands(n, k, batch, seed=7)
    y = E.kernel_gemm(w, x, ksplit=4, epilogue="swiglu")
    s = x64 @ w64.T
    g, u = s[:, : n // 2], s[:, n // 2:]
    _close(y, g / (1.0 + np.exp(-g)) * u)


def test_gemm_rejects_bad_shapes():
    w = np.zeros((128, 100), dtype=np.uint16)
    x = np.zeros((4, 100), dtype=np.uint16)
    with pytest.raises(E.CudaLLMError):
        E.kernel_gemm(w, x)  # k not a multiple of 64
    w = np.zeros((128, 128), dtype=np.uint16)
    x = np.zeros((65, 128), dtype=np.uint16)
    with pytest.raises(E.CudaLLMError):
        E.kernel_gemm(w, x)  # batch above 64
    x = np.zeros((4, 128), dtype=np.uint16)
    with pytest.raises(E.CudaLLMError):
        E.kernel_gemm(w, x, ksplit=3)  # more K rows than 64-column chunks
