"""Reader / writer of the .cudallm weight file format.

The format is shared with wasiqnauman/cudallm (python/cudallm/format.py:1-147,
src/model/cudallm_format.h:12-46), so the byte layout is fixed by it: a 256-byte little-endian
header (`HEADER_FMT`, zero padded), a table of 80-byte tensor entries at byte 256, and every tensor's
data at a 256-byte aligned offset in table order. Function names follow that module so code written
against it reads the same; the implementation is this package's own (streamed writes from numpy
arrays, offsets planned up front so blocks can be written in parallel with os.pwrite).
"""
from __future__ import annotations

import struct
from pathlib import Path
from typing import Iterable

import numpy as np

MAGIC = b"CLLM"
VERSION = 1

# Tensor dtype codes (part of the format).
F32, BF16, F16, I8, I4X2 = 0, 1, 2, 3, 4
# File-level weight_dtype codes.
WEIGHT_BF16, WEIGHT_INT8, WEIGHT_INT4 = 1, 3, 4

HEADER_FMT = "<4s10I2f3IQ"
HEADER_SIZE = 256
ENTRY_FMT = "<48s4I2Q"
ENTRY_SIZE = 80
ALIGN = 256

HEADER_FIELDS = ("magic", "version", "weight_dtype", "hidden_size", "intermediate_size", "n_layers", "n_heads",
                 "n_kv_heads", "head_dim", "vocab_size", "max_seq_len", "rms_eps", "rope_theta", "group_size",
                 "n_tensors", "reserved0", "table_offset")

assert struct.calcsize(HEADER_FMT) == 72
assert struct.calcsize(ENTRY_FMT) == ENTRY_SIZE


def align_up(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def expected_nbytes(dtype: int, rows: int, cols: int) -> int:
    if dtype == F32:
        return rows * cols * 4
    if dtype in (BF16, F16):
        return rows * cols * 2
    if dtype == I8:
        return rows * cols
    if dtype == I4X2:
        if cols % 2:
            raise ValueError("I4X2 tensors need an even column count")
        return rows * cols // 2
    raise ValueError(f"unknown dtype code {dtype}")


def expected_names(n_layers: int, quant: bool) -> list[str]:
    """Tensor order of a Llama file: 99 names for bf16, 164 for int8/int4 (16 layers)."""
    names = ["rope.inv_freq", "tok_embeddings.weight"] + (["tok_embeddings.scales"] if quant else []) + ["norm.weight"]
    for i in range(n_layers):
        p = f"layers.{i}."
        names.append(p + "attn_norm.weight")
        for lin in ("wqkv", "wo"):
            names += [p + lin + ".weight"] + ([p + lin + ".scales"] if quant else [])
        names.append(p + "ffn_norm.weight")
        for lin in ("w_gate_up", "w_down"):
            names += [p + lin + ".weight"] + ([p + lin + ".scales"] if quant else [])
    return names


def pack_header(header: dict, n_tensors: int) -> bytes:
    raw = struct.pack(HEADER_FMT, MAGIC, VERSION, header["weight_dtype"], header["hidden_size"],
                      header["intermediate_size"], header["n_layers"], header["n_heads"], header["n_kv_heads"],
                      header["head_dim"], header["vocab_size"], header["max_seq_len"], header["rms_eps"],
                      header["rope_theta"], header["group_size"], n_tensors, 0, HEADER_SIZE)
    return raw + b"\0" * (HEADER_SIZE - len(raw))


def plan_layout(specs: Iterable[tuple[str, int, int, int]]) -> tuple[list[dict], int]:
    """specs: (name, dtype, rows, cols) in file order -> (entries with offset/nbytes, file size)."""
    specs = list(specs)
    offset = align_up(HEADER_SIZE + ENTRY_SIZE * len(specs))
    entries = []
    end = offset
    for name, dtype, rows, cols in specs:
        nbytes = expected_nbytes(dtype, rows, cols)
        entries.append({"name": name, "dtype": dtype, "rows": rows, "cols": cols, "offset": offset, "nbytes": nbytes})
        end = offset + nbytes
        offset = align_up(end)
    return entries, end


def pack_table(entries: list[dict]) -> bytes:
    out = bytearray()
    for e in entries:
        name = e["name"].encode("ascii")
        if len(name) >= 48:
            raise ValueError(f"tensor name too long: {e['name']}")
        out += struct.pack(ENTRY_FMT, name, e["dtype"], e["rows"], e["cols"], 0, e["offset"], e["nbytes"])
    return bytes(out)


def write_cudallm(path: Path | str, header: dict, tensors: list[tuple[str, int, int, int, bytes]]) -> None:
    """Writes a complete file from in-memory tensors (name, dtype, rows, cols, data)."""
    entries, size = plan_layout((n, d, r, c) for n, d, r, c, _ in tensors)
    with open(path, "wb") as f:
        f.write(pack_header(header, len(entries)))
        f.write(pack_table(entries))
        for e, (_, _, _, _, data) in zip(entries, tensors):
            data = memoryview(data).cast("B")
            if len(data) != e["nbytes"]:
                raise ValueError(f"{e['name']}: {len(data)} bytes, expected {e['nbytes']}")
            f.write(b"\0" * (e["offset"] - f.tell()))
            f.write(data)
        assert f.tell() == size


def read_header(path: Path | str) -> dict:
    with open(path, "rb") as f:
        raw = f.read(HEADER_SIZE)
    if len(raw) != HEADER_SIZE:
        raise ValueError(f"{path}: truncated header")
    return dict(zip(HEADER_FIELDS, struct.unpack(HEADER_FMT, raw[:struct.calcsize(HEADER_FMT)])))


def read_table(path: Path | str) -> list[dict]:
    hdr = read_header(path)
    n = hdr["n_tensors"]
    with open(path, "rb") as f:
        f.seek(hdr["table_offset"])
        raw = f.read(ENTRY_SIZE * n)
    out = []
    for k in range(n):
        name, dtype, rows, cols, reserved, offset, nbytes = struct.unpack_from(ENTRY_FMT, raw, k * ENTRY_SIZE)
        out.append({"name": name.rstrip(b"\0").decode("ascii"), "dtype": dtype, "rows": rows, "cols": cols,
                    "reserved": reserved, "offset": offset, "nbytes": nbytes})
    return out


_NP = {F32: np.float32, BF16: np.uint16, F16: np.float16, I8: np.int8, I4X2: np.uint8}


def load_tensor(path: Path | str, entry: dict, mmap: bool = False) -> np.ndarray:
    """Tensor data as stored: f32 vectors [rows], bf16 as uint16 bits, I4X2 as packed uint8 [rows][cols/2]."""
    rows, cols, dtype = entry["rows"], entry["cols"], entry["dtype"]
    shape = (rows, cols // 2) if dtype == I4X2 else (rows, cols)
    count = shape[0] * shape[1]
    if mmap:
        arr = np.memmap(path, dtype=_NP[dtype], mode="r", offset=entry["offset"], shape=(count,))
    else:
        arr = np.fromfile(path, dtype=_NP[dtype], count=count, offset=entry["offset"])
    if arr.size != count:
        raise ValueError(f"{path}: truncated tensor {entry['name']}")
    arr = arr.reshape(shape)
    if dtype == F32 and cols == 1:
        arr = arr.reshape(rows)
    return arr


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
