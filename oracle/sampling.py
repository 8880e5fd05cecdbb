"""Test infrastructure only (never part of the product path): CPU restatement of the persistent decode
step's next-token sampling (cudallm_b200/csrc/kernels/sampling.cuh, cudallm_set_sampling in
include/cudallm.h), used by the tests as the checker of the GPU's choice.

Parity unpinned for temperature > 0: wasiqnauman/cudallm decodes greedily only (src/kernels/argmax.cu:35-85,
lowest index on ties) and has no sampling to compare with. top_k = 1 reduces to that argmax rule, which the
tests pin. The rule restated here, in float32 with the GPU's order of operations:
  * candidates: the top_k logits ranked by (logit descending, index ascending);
  * w_i = exp((v_i - v_0) / temperature), S_i = w_0 + ... + w_i accumulated in that order;
  * nucleus: candidates 0..m, m the first index with S_m >= top_p * S_{k-1};
  * u = SplitMix64(seed + (pos + 1) * 0x9E3779B97F4A7C15) >> 40, divided by 2^24 (Steele, Lea and Flood,
    OOPSLA 2014); the token is the first candidate i <= m with S_i > u * S_m.
"""
from __future__ import annotations

import numpy as np

MASK64 = (1 << 64) - 1
MAX_TOP_K = 64


def sample_uniform(seed: int, pos: int) -> np.float32:
    z = (seed + (pos + 1) * 0x9E3779B97F4A7C15) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    z ^= z >> 31
    return np.float32(z >> 40) * np.float32(1.0 / 16777216.0)


def top_k_indices(logits: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest logits, by logit descending then index ascending."""
    logits = np.asarray(logits, dtype=np.float32)
    return np.lexsort((np.arange(logits.size), -logits))[:k]


def draw(logits: np.ndarray, temperature: float, top_k: int, top_p: float, seed: int, pos: int) -> tuple[int, float]:
    """(token, margin): the token the rule picks, and the distance of the draw u * S_m to the nearest
    cumulative boundary relative to S_m (a small margin means float32 rounding could change the pick)."""
    k = MAX_TOP_K if top_k == 0 else top_k
    idx = top_k_indices(logits, k)
    v = np.asarray(logits, dtype=np.float32)[idx]
    w = np.exp((v - v[0]) / np.float32(temperature)).astype(np.float32)
    s = np.cumsum(w, dtype=np.float32)
    cut = np.float32(top_p) * s[-1]
    m = int(np.argmax(s >= cut))
    target = sample_uniform(seed, pos) * s[m]
    pick = int(np.argmax(s[: m + 1] > target)) if (s[: m + 1] > target).any() else m
    # how firmly m is determined (with top_p = 1 the nucleus is every candidate of nonzero weight, and a
    # trailing weight that rounds differently moves m without changing any pick outside its own sliver)
    margin_cut = 1.0 if top_p >= 1.0 else float(np.min(np.abs(s - cut)) / s[-1])
    margin_pick = float(np.min(np.abs(s[: m + 1] - target)) / s[m])
    return int(idx[pick]), min(margin_cut, margin_pick)


def greedy(logits: np.ndarray) -> int:
    """The reference's argmax rule: the largest logit, lowest index on ties."""
    logits = np.asarray(logits, dtype=np.float32)
    return int(np.flatnonzero(logits == logits.max())[0])
