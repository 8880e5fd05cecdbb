"""Seeded synthetic Llama-3.2-1B weight files and prompts (there is no checkpoint on this machine).

Procedure (fixed here; the reference does not define one):
  * Tensors follow the .cudallm order (format.expected_names). Every matrix is generated in blocks of
    2048 rows; block b of tensor k (k = position of its ".weight" name in the bf16 order) draws
    `np.random.default_rng([seed, k, b]).standard_normal((rows_in_block, cols), dtype=float32)`,
    multiplies by float32(0.02) and rounds to bf16 (round to nearest even).
  * RMSNorm gains are 1.0. rope.inv_freq is the llama3-scaled inverse frequency (theta 500000,
    factor 32, low 1, high 4, original context 8192), computed in float64 and stored as fp32.
  * int8 / int4 files quantise exactly those bf16 values (as fp32) with quantize.py, the reference's
    quantiser restated, block by block.
  * Prompts: `np.random.default_rng(seed).integers(0, 128256, n)` (batched: seed [seed, sequence]).
Blocks are generated in parallel worker processes (spawn start method, safe after CUDA is in use)
and written straight into a pre-sized file. Because spawned workers re-import the caller's main
module, a script that calls ensure_model/write_model must do so under `if __name__ == "__main__":`; a content digest (sha256 over per-block sha256s, in file
order) identifies the result and is kept in a side file next to the model.
"""
from __future__ import annotations

import fcntl
import hashlib
import json
import multiprocessing as mp
import os
from pathlib import Path

import numpy as np

from . import format as fmt
from .paths import MODEL_DIR
from .quantize import INT4_GROUP, quantize_int4_groups, quantize_int8_rows

HIDDEN, INTER, LAYERS, HEADS, KV_HEADS, HEAD_DIM, VOCAB = 2048, 8192, 16, 32, 8, 64, 128256
RMS_EPS, ROPE_THETA = 1e-5, 500000.0
BLOCK_ROWS = 2048
INIT_STD = 0.02
SYNTH_VERSION = 1

_LINEARS = {"tok_embeddings": (VOCAB, HIDDEN), "wqkv": ((HEADS + 2 * KV_HEADS) * HEAD_DIM, HIDDEN),
            "wo": (HIDDEN, HIDDEN), "w_gate_up": (2 * INTER, HIDDEN), "w_down": (HIDDEN, INTER)}


def llama3_inv_freq() -> np.ndarray:
    i = np.arange(HEAD_DIM // 2, dtype=np.float64)
    base = 1.0 / ROPE_THETA ** (2.0 * i / HEAD_DIM)
    wavelen = 2.0 * np.pi / base
    factor, low, high, orig = 32.0, 1.0, 4.0, 8192.0
    smooth = (orig / wavelen - low) / (high - low)
    scaled = np.where(wavelen < orig / high, base, np.where(wavelen > orig / low, base / factor,
                                                            (1.0 - smooth) * base / factor + smooth * base))
    return scaled.astype(np.float32)


def prompt_ids(n: int, seed: int = 0, sequence: int | None = None) -> list[int]:
    rng = np.random.default_rng(seed if sequence is None else [seed, sequence])
    return [int(t) for t in rng.integers(0, VOCAB, n)]


def header(dtype: str, max_seq_len: int) -> dict:
    return {"weight_dtype": {"bf16": fmt.WEIGHT_BF16, "int8": fmt.WEIGHT_INT8, "int4": fmt.WEIGHT_INT4}[dtype],
            "hidden_size": HIDDEN, "intermediate_size": INTER, "n_layers": LAYERS, "n_heads": HEADS,
            "n_kv_heads": KV_HEADS, "head_dim": HEAD_DIM, "vocab_size": VOCAB, "max_seq_len": max_seq_len,
            "rms_eps": RMS_EPS, "rope_theta": ROPE_THETA, "group_size": INT4_GROUP if dtype == "int4" else 0}


def _linear_shape(name: str) -> tuple[int, int] | None:
    for key, shape in _LINEARS.items():
        if name.endswith(key + ".weight"):
            return shape
    return None


def _specs(dtype: str) -> list[tuple[str, int, int, int]]:
    """(name, dtype code, rows, cols) in file order."""
    quant = dtype != "bf16"
    specs = []
    for name in fmt.expected_names(LAYERS, quant):
        if name == "rope.inv_freq":
            specs.append((name, fmt.F32, HEAD_DIM // 2, 1))
        elif name.endswith("norm.weight"):
            specs.append((name, fmt.F32, HIDDEN, 1))
        elif name.endswith(".weight"):
            rows, cols = _linear_shape(name)
            code = {"bf16": fmt.BF16, "int8": fmt.I8, "int4": fmt.I4X2}[dtype]
            specs.append((name, code, rows, cols))
        else:  # scales
            rows, cols = _linear_shape(name[:-len(".scales")] + ".weight")
            specs.append((name, fmt.F32, rows, 1) if dtype == "int8" else (name, fmt.F16, rows, cols // INT4_GROUP))
    return specs


def _weight_index(name: str) -> int:
    return fmt.expected_names(LAYERS, False).index(name)


def block_values(seed: int, name: str, block: int) -> np.ndarray:
    """bf16-rounded fp32 values of rows [block*2048, ...) of matrix `name`."""
    rows, cols = _linear_shape(name)
    r0 = block * BLOCK_ROWS
    n = min(BLOCK_ROWS, rows - r0)
    rng = np.random.default_rng([seed, _weight_index(name), block])
    v = rng.standard_normal((n, cols), dtype=np.float32)
    v *= np.float32(INIT_STD)
    return fmt.bf16_bits_to_f32(fmt.f32_to_bf16_bits(v))


def matrix_values(seed: int, name: str) -> np.ndarray:
    """Whole matrix (fp32, bf16-exact); for tests and the oracle on small shapes."""
    rows, _ = _linear_shape(name)
    return np.concatenate([block_values(seed, name, b) for b in range((rows + BLOCK_ROWS - 1) // BLOCK_ROWS)])


def _job_list(dtype: str, entries: list[dict]) -> list[tuple]:
    by_name = {e["name"]: e for e in entries}
    jobs = []
    for e in entries:
        name = e["name"]
        if not name.endswith(".weight") or name.endswith("norm.weight"):
            continue
        rows, cols = _linear_shape(name)
        scale_e = by_name.get(name[:-len(".weight")] + ".scales")
        for b in range((rows + BLOCK_ROWS - 1) // BLOCK_ROWS):
            jobs.append((name, b, e["offset"], scale_e["offset"] if scale_e else None, cols))
    return jobs


def _run_block(args) -> tuple[str, int, str, str | None]:
    path, seed, dtype, name, block, w_off, s_off, cols = args
    v = block_values(seed, name, block)
    r0 = block * BLOCK_ROWS
    fd = os.open(path, os.O_WRONLY)
    try:
        if dtype == "bf16":
            data = fmt.f32_to_bf16_bits(v).tobytes()
            os.pwrite(fd, data, w_off + r0 * cols * 2)
            sdata = None
        elif dtype == "int8":
            q, s = quantize_int8_rows(v)
            data = q.tobytes()
            sdata = s.astype(np.float32).tobytes()
            os.pwrite(fd, data, w_off + r0 * cols)
            os.pwrite(fd, sdata, s_off + r0 * 4)
        else:
            q, s = quantize_int4_groups(v, INT4_GROUP)
            data = q.tobytes()
            sdata = s.astype(np.float16).tobytes()
            os.pwrite(fd, data, w_off + r0 * cols // 2)
            os.pwrite(fd, sdata, s_off + r0 * (cols // INT4_GROUP) * 2)
    finally:
        os.close(fd)
    return name, block, hashlib.sha256(data).hexdigest(), hashlib.sha256(sdata).hexdigest() if sdata else None


def model_path(dtype: str, seed: int = 0, max_seq_len: int = 4096, directory: Path | None = None) -> Path:
    d = Path(directory) if directory else MODEL_DIR
    return d / f"llama3.2-1b-synth-v{SYNTH_VERSION}-seed{seed}-{dtype}-s{max_seq_len}.cudallm"


def write_model(path: Path, dtype: str, seed: int = 0, max_seq_len: int = 4096, workers: int | None = None) -> str:
    """Writes the file; returns its content digest."""
    entries, size = fmt.plan_layout(_specs(dtype))
    tmp = path.with_suffix(".partial")
    with open(tmp, "wb") as f:
        f.truncate(size)
        f.seek(0)
        f.write(fmt.pack_header(header(dtype, max_seq_len), len(entries)))
        f.write(fmt.pack_table(entries))
        by_name = {e["name"]: e for e in entries}
        f.seek(by_name["rope.inv_freq"]["offset"])
        f.write(llama3_inv_freq().tobytes())
        ones = np.ones(HIDDEN, dtype=np.float32).tobytes()
        for e in entries:
            if e["name"].endswith("norm.weight"):
                f.seek(e["offset"])
                f.write(ones)
    jobs = [(str(tmp), seed, dtype, *j) for j in _job_list(dtype, entries)]
    workers = workers or max(1, min(len(jobs), os.cpu_count() or 1, 32))
    with mp.get_context("spawn").Pool(workers) as pool:
        results = pool.map(_run_block, jobs, chunksize=1)
    h = hashlib.sha256()
    h.update(f"{dtype}|{seed}|{max_seq_len}|v{SYNTH_VERSION}".encode())
    h.update(llama3_inv_freq().tobytes())
    for name, block, dh, sh in results:  # pool.map keeps job (file) order
        h.update(f"{name}:{block}:{dh}:{sh}".encode())
    digest = h.hexdigest()
    os.replace(tmp, path)
    return digest


def ensure_model(dtype: str, seed: int = 0, max_seq_len: int = 4096, directory: Path | None = None) -> tuple[Path, str]:
    """Path of the cached synthetic model (generated on first use, process- and rank-safe) and its digest."""
    path = model_path(dtype, seed, max_seq_len, directory)
    meta = path.with_suffix(".json")
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path.with_suffix(".lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if path.exists() and meta.exists():
            return path, json.loads(meta.read_text())["digest"]
        digest = write_model(path, dtype, seed, max_seq_len)
        meta.write_text(json.dumps({"digest": digest, "dtype": dtype, "seed": seed, "max_seq_len": max_seq_len,
                                    "version": SYNTH_VERSION}))
        return path, digest


def main(argv: list[str] | None = None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description="write seeded synthetic Llama-3.2-1B .cudallm files")
    ap.add_argument("--dtype", choices=("bf16", "int8", "int4"), nargs="+", default=["bf16"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--max-seq-len", type=int, default=4096)
    args = ap.parse_args(argv)
    for d in args.dtype:
        p, digest = ensure_model(d, args.seed, args.max_seq_len)
        print(f"{p} {digest}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
