"""A tiny Llama-shaped model (same structure, small dimensions) used to pin the CPU oracle.

The values come from numpy's seeded generator only, so both the fixture generator (which writes the
file with wasiqnauman/cudallm's own format writer and quantiser) and the tests (which write it with
this package's) start from identical fp32 weights; equal file digests then prove the writer and the
quantiser produce the reference's bytes.
"""
from __future__ import annotations

import numpy as np

DIMS = {"hidden_size": 256, "intermediate_size": 512, "n_layers": 2, "n_heads": 4, "n_kv_heads": 1, "head_dim": 64,
        "vocab_size": 1000, "max_seq_len": 128, "rms_eps": 1e-5, "rope_theta": 500000.0}
SEED = 7
PROMPT = [3, 997, 42, 500, 1, 777, 256, 0]
N_NEW = 8


def llama3_inv_freq(head_dim: int = 64) -> np.ndarray:
    i = np.arange(head_dim // 2, dtype=np.float64)
    base = 1.0 / 500000.0 ** (2 * i / head_dim)
    lam = 2 * np.pi / base
    out = np.where(lam < 8192 / 4, base, np.where(lam > 8192, base / 32, 0.0))
    mid = (lam >= 8192 / 4) & (lam <= 8192)
    s = (8192 / lam - 1) / 3
    return np.where(mid, (1 - s) * base / 32 + s * base, out).astype(np.float32)


def bf16_round(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    bits = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    return bits


def tensors_f32() -> list[tuple[str, str, np.ndarray]]:
    """(name, kind, values) in file order; kind is "vec" (fp32 vector) or "mat" (bf16-exact matrix as fp32)."""
    d = DIMS
    H, I, V, L = d["hidden_size"], d["intermediate_size"], d["vocab_size"], d["n_layers"]
    qkv_rows = (d["n_heads"] + 2 * d["n_kv_heads"]) * d["head_dim"]
    rng = np.random.default_rng(SEED)

    def mat(rows, cols):
        w = rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32)
        return (bf16_round(w).astype(np.uint32) << 16).view(np.float32)

    def gain(n):
        return rng.uniform(0.8, 1.2, n).astype(np.float32)

    out = [("rope.inv_freq", "vec", llama3_inv_freq(d["head_dim"])), ("tok_embeddings", "mat", mat(V, H)),
           ("norm.weight", "vec", gain(H))]
    for i in range(L):
        p = f"layers.{i}."
        out += [(p + "attn_norm.weight", "vec", gain(H)), (p + "wqkv", "mat", mat(qkv_rows, H)),
                (p + "wo", "mat", mat(H, H)), (p + "ffn_norm.weight", "vec", gain(H)),
                (p + "w_gate_up", "mat", mat(2 * I, H)), (p + "w_down", "mat", mat(H, I))]
    return out


def header(weight_dtype_code: int) -> dict:
    h = dict(DIMS)
    h["weight_dtype"] = weight_dtype_code
    h["group_size"] = 128 if weight_dtype_code == 4 else 0
    return h


def build_tensor_list(dtype: str, fmt, quantize_int8_rows, quantize_int4_groups) -> list:
    """Tensor list for a `write_cudallm(path, header, tensors)` of either project."""
    tensors = []
    for name, kind, v in tensors_f32():
        if kind == "vec":
            tensors.append((name, fmt.F32, v.shape[0], 1, v.tobytes()))
            continue
        rows, cols = v.shape
        if dtype == "bf16":
            tensors.append((name + ".weight", fmt.BF16, rows, cols, bf16_round(v).tobytes()))
        elif dtype == "int8":
            q, s = quantize_int8_rows(v)
            tensors += [(name + ".weight", fmt.I8, rows, cols, q.tobytes()),
                        (name + ".scales", fmt.F32, rows, 1, s.astype(np.float32).tobytes())]
        else:
            q, s = quantize_int4_groups(v, 128)
            tensors += [(name + ".weight", fmt.I4X2, rows, cols, q.tobytes()),
                        (name + ".scales", fmt.F16, rows, cols // 128, s.astype(np.float16).tobytes())]
    return tensors


# Small mixed-dtype tensor set for the byte-level writer check (the reference's tests/test_format.py
# uses the same kind of set).
FORMAT_HEADER = {"weight_dtype": 1, "hidden_size": 2048, "intermediate_size": 8192, "n_layers": 16, "n_heads": 32,
                 "n_kv_heads": 8, "head_dim": 64, "vocab_size": 128256, "max_seq_len": 4096, "rms_eps": 1e-5,
                 "rope_theta": 500000.0, "group_size": 0}


def format_tensors() -> list:
    rng = np.random.default_rng(0)
    return [("a.f32", 0, 5, 1, rng.standard_normal((5, 1)).astype(np.float32).tobytes()),
            ("b.bf16", 1, 3, 7, rng.integers(0, 2**16, size=(3, 7), dtype=np.uint16).tobytes()),
            ("c.f16", 2, 2, 3, rng.standard_normal((2, 3)).astype(np.float16).tobytes()),
            ("d.i8", 3, 4, 9, rng.integers(-127, 128, size=(4, 9), dtype=np.int8).tobytes()),
            ("e.i4", 4, 3, 8, rng.integers(0, 256, size=(3, 4), dtype=np.uint8).tobytes())]
