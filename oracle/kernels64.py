"""float64 references for the single-kernel hooks. TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Each function states the same quantity wasiqnauman/cudallm tests/test_kernels.py checks its kernels
against (cited per function); the tolerances live in the tests.
"""
from __future__ import annotations

import numpy as np

from cudallm_b200 import format as fmt
from cudallm_b200.quantize import (dequantize_int4_groups, dequantize_int8_rows, quantize_int4_groups,
                                   quantize_int8_rows)


def bf16_bits_to_f64(bits: np.ndarray) -> np.ndarray:
    return fmt.bf16_bits_to_f32(bits).astype(np.float64)


def matvec_operands(wtype: str, rows: int, cols: int, seed: int):
    """(stored weight, scales or None, exact dequantised weight as float64); test_kernels.py:51-62."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32)
    if wtype == "bf16":
        bits = fmt.f32_to_bf16_bits(w)
        return bits, None, bf16_bits_to_f64(bits)
    if wtype == "int8":
        q, scales = quantize_int8_rows(w)
        return q, scales, dequantize_int8_rows(q, scales).astype(np.float64)
    packed, scales = quantize_int4_groups(w, 128)
    return packed, scales, dequantize_int4_groups(packed, scales).astype(np.float64)


def rmsnorm64(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """test_kernels.py:101-109."""
    x64 = np.asarray(x, dtype=np.float64)
    return x64 / np.sqrt(np.mean(x64 * x64) + eps) * np.asarray(w, dtype=np.float64)


def matvec64(w64: np.ndarray, x: np.ndarray, epilogue: str, norm_w: np.ndarray | None, eps: float,
             y_init: np.ndarray | None) -> np.ndarray:
    """test_kernels.py:82-94: optional RMSNorm prologue, then STORE / ADD / SWIGLU."""
    x64 = np.asarray(x, dtype=np.float64)
    if norm_w is not None:
        x64 = rmsnorm64(x64, norm_w, eps)
    d = w64 @ x64
    if epilogue == "swiglu":
        half = d.size // 2
        g, u = d[:half], d[half:]
        return g / (1 + np.exp(-g)) * u
    if epilogue == "add":
        return np.asarray(y_init, dtype=np.float64) + d
    return d


def rope64(v: np.ndarray, inv_freq: np.ndarray, pos: int) -> np.ndarray:
    """test_kernels.py:117-122: angle formed in fp32 exactly like the kernel, rotation in float64."""
    hd = v.shape[1]
    ang = (np.float32(pos) * inv_freq).astype(np.float64)
    c, s = np.cos(ang), np.sin(ang)
    a, b = v[:, :hd // 2], v[:, hd // 2:]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=1)


def fp16_ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in fp16 ulps (test_kernels.py:125-130)."""
    def ordered(x):
        u = np.asarray(x).astype(np.float16).view(np.uint16).astype(np.int32)
        return np.where(u & 0x8000, 0x8000 - u, u)
    return np.abs(ordered(a) - ordered(b))


def attention64(q: np.ndarray, k: np.ndarray, v: np.ndarray, ctx: int, nh: int, nkv: int) -> np.ndarray:
    """test_kernels.py:168-179: per query head softmax(K q / 8) V over the first ctx tokens."""
    hd = k.shape[-1]
    q64 = np.asarray(q, dtype=np.float64).reshape(nh, hd)
    k64 = np.asarray(k[:, :ctx], dtype=np.float64)
    v64 = np.asarray(v[:, :ctx], dtype=np.float64)
    out = np.empty((nh, hd))
    for h in range(nh):
        kvh = h // (nh // nkv)
        s = (k64[kvh] @ q64[h]) / 8.0
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h] = p @ v64[kvh]
    return out.reshape(-1)


def silu_mul64(gu: np.ndarray) -> np.ndarray:
    gu = np.asarray(gu, dtype=np.float64)
    inter = gu.size // 2
    g, u = gu[:inter], gu[inter:]
    return g / (1 + np.exp(-g)) * u
