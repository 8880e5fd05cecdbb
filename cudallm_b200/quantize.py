"""Weight-only quantisers that produce the .cudallm int8 / int4 layouts.

The layouts and rounding are those of wasiqnauman/cudallm python/cudallm/quantize.py:5-29, and the
output must be bit-identical to it (the parity tests pin this against vectors that quantiser produced):
  int8: symmetric per row, scale = max|w| / 127 in fp32 (1.0 for an all-zero row),
        q = clip(round_half_even(w / scale), -127, 127).
  int4: groups of 128 columns, scale = max|w| / 7 in fp32 (1.0 for an all-zero group), stored as fp16,
        and q = clip(round_half_even(w / float32(fp16 scale)), -8, 7) so dequantisation uses the stored
        value; q + 8 is packed two per byte, even column in the low nibble.
Row blocks are processed independently (every step is per row or per group), which bounds memory and
lets callers parallelise.
"""
from __future__ import annotations

import numpy as np

INT4_GROUP = 128
_ROW_BLOCK = 1024


def quantize_int8_rows(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    q = np.empty((rows, cols), dtype=np.int8)
    scales = np.empty(rows, dtype=np.float32)
    for r0 in range(0, rows, _ROW_BLOCK):
        blk = w[r0:r0 + _ROW_BLOCK]
        s = np.max(np.abs(blk), axis=1) / np.float32(127)
        s = np.where(s == 0, np.float32(1.0), s).astype(np.float32)
        scales[r0:r0 + _ROW_BLOCK] = s
        q[r0:r0 + _ROW_BLOCK] = np.clip(np.rint(blk / s[:, None]), -127, 127).astype(np.int8)
    return q, scales


def dequantize_int8_rows(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    return q.astype(np.float32) * np.asarray(scales, dtype=np.float32)[:, None]


def quantize_int4_groups(w: np.ndarray, group: int = INT4_GROUP) -> tuple[np.ndarray, np.ndarray]:
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    if cols % group or cols % 2:
        raise ValueError("int4 needs cols divisible by the group size and by 2")
    packed = np.empty((rows, cols // 2), dtype=np.uint8)
    scales = np.empty((rows, cols // group), dtype=np.float16)
    for r0 in range(0, rows, _ROW_BLOCK):
        blk = w[r0:r0 + _ROW_BLOCK].reshape(-1, cols // group, group)
        s = np.max(np.abs(blk), axis=2) / np.float32(7)
        s = np.where(s == 0, np.float32(1.0), s)
        s16 = s.astype(np.float16)
        q = np.clip(np.rint(blk / s16.astype(np.float32)[:, :, None]), -8, 7).astype(np.int8)
        u = (q.reshape(-1, cols) + 8).astype(np.uint8)
        packed[r0:r0 + _ROW_BLOCK] = u[:, 0::2] | (u[:, 1::2] << 4)
        scales[r0:r0 + _ROW_BLOCK] = s16
    return packed, scales


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    out = np.empty((packed.shape[0], packed.shape[1] * 2), dtype=np.int8)
    out[:, 0::2] = (packed & 0x0F).astype(np.int8) - 8
    out[:, 1::2] = (packed >> 4).astype(np.int8) - 8
    return out


def dequantize_int4_groups(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    q = unpack_int4(packed).astype(np.float32)
    rows, cols = q.shape
    n_groups = scales.shape[1]
    s = np.asarray(scales).astype(np.float32)
    return (q.reshape(rows, n_groups, cols // n_groups) * s[:, :, None]).reshape(rows, cols)
