"""Generates the golden fixtures in tests/golden/ by running wasiqnauman/cudallm's own Python code.

Run in a container where the reference checkout is available (it is never needed at test time):
    CUDALLM_REFERENCE_PYTHON=/path/to/cudallm/python python tests/golden/make_golden.py --parts quant format tiny full

Parts (each writes one .npz):
  quant   reference quantize_int8_rows / quantize_int4_groups on seeded matrices with edge cases
          (all-zero rows/groups, exact half-way values, signed extremes) -> golden_quant.npz
  format  reference write_cudallm on a small tensor set -> sha256 of the file bytes -> golden_format.npz
  tiny    a tiny Llama-shaped model (tiny_spec.py) written with the reference's writer and quantiser;
          reference ReferenceModel logits / residuals / greedy ids -> golden_tiny.npz
  full    the seeded Llama-3.2-1B files this package generates (cudallm_b200.synth); the reference's
          quantiser re-applied to sampled blocks; ReferenceModel on the 32-token seeded prompt for
          32 + 63 steps: greedy ids, per-step top-2 margin and logit statistics, full logits at the last
          prompt step and residuals at two steps -> golden_full_<config>.npz
  long    the seeded bf16 weights in a max_seq_len 32896 file; ReferenceModel (bf16 KV) on a 4096-token
          seeded prompt + 8 greedy tokens -> golden_long_bf16_bf16.npz (about half an hour of CPU)
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))
sys.path.insert(0, os.environ.get("CUDALLM_REFERENCE_PYTHON", "/root/reference/python"))

import torch  # noqa: E402
from cudallm import format as ref_fmt  # noqa: E402  (the reference package)
from cudallm.quantize import quantize_int4_groups as ref_q4  # noqa: E402
from cudallm.quantize import quantize_int8_rows as ref_q8  # noqa: E402
from cudallm.reference import ReferenceModel  # noqa: E402

import tiny_spec  # noqa: E402
from cudallm_b200 import synth  # noqa: E402

FULL_PROMPT_LEN = 32
FULL_NEW = 64


def quant_inputs() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(11)
    a = rng.normal(0, 0.02, size=(64, 512)).astype(np.float32)
    a[3] = 0.0                      # zero row (int8 scale 1.0) and zero groups (int4)
    a[5, :128] = 0.0                # one zero int4 group
    a[7, :4] = [0.07, -0.07, 0.035, -0.035]   # exact half-way values after scaling
    a[7, 4] = 0.0875
    a[9] = np.linspace(-1, 1, 512, dtype=np.float32)
    a[10, 17] = -3.0                # negative extreme sets the scale
    b = rng.standard_normal((8, 1024)).astype(np.float32) * 10
    return {"a": a, "b": b}


def part_quant() -> None:
    out = {}
    for k, w in quant_inputs().items():
        q8, s8 = ref_q8(w)
        q4, s4 = ref_q4(w, 128)
        out.update({f"{k}_in": w, f"{k}_q8": q8, f"{k}_s8": s8, f"{k}_q4": q4, f"{k}_s4": s4})
    np.savez_compressed(HERE / "golden_quant.npz", **out)


def part_format() -> None:
    with tempfile.TemporaryDirectory() as d:
        p = Path(d) / "f.cudallm"
        ref_fmt.write_cudallm(p, tiny_spec.FORMAT_HEADER, tiny_spec.format_tensors())
        raw = p.read_bytes()
    np.savez_compressed(HERE / "golden_format.npz", sha256=np.array(hashlib.sha256(raw).hexdigest()),
                        size=np.array(len(raw)))


def run_reference(path: Path, prompt: list[int], n_new: int, kv: torch.dtype, keep_logits_at=(), keep_res_at=(),
                  store_all=False) -> dict:
    ref = ReferenceModel(path, kv_dtype=kv)
    out = {"ids": [], "margin": [], "lsum": [], "lsq": [], "top8_i": [], "top8_v": []}
    logits_keep, res_keep, all_logits, all_res = {}, {}, [], []
    ids = list(prompt)
    logits = None
    step = 0
    t0 = time.time()
    while True:
        tok = ids[step]
        logits, res = ref.step(tok)
        lg = logits.numpy().astype(np.float32)
        top = np.argsort(-lg, kind="stable")[:8]
        out["top8_i"].append(top.astype(np.int32))
        out["top8_v"].append(lg[top])
        out["margin"].append(float(lg[top[0]] - lg[top[1]]))
        out["lsum"].append(float(lg.astype(np.float64).sum()))
        out["lsq"].append(float((lg.astype(np.float64) ** 2).sum()))
        if step in keep_logits_at:
            logits_keep[step] = lg
        if step in keep_res_at:
            res_keep[step] = torch.stack(res).numpy()
        if store_all:
            all_logits.append(lg)
            all_res.append(torch.stack(res).numpy())
        nxt = int(torch.argmax(logits))
        step += 1
        if step >= len(prompt):
            out["ids"].append(nxt)
            if len(out["ids"]) >= n_new:
                break
            ids.append(nxt)
        print(f"  step {step} ({time.time() - t0:.0f}s)", flush=True)
    res = {k: np.array(v) for k, v in out.items()}
    for s, v in logits_keep.items():
        res[f"logits_{s}"] = v
    for s, v in res_keep.items():
        res[f"res_{s}"] = v
    if store_all:
        res["logits_all"] = np.stack(all_logits)
        res["res_all"] = np.stack(all_res)
    return res


def part_tiny() -> None:
    out = {}
    with tempfile.TemporaryDirectory() as d:
        for dtype, code in (("bf16", 1), ("int8", 3), ("int4", 4)):
            p = Path(d) / f"tiny_{dtype}.cudallm"
            ref_fmt.write_cudallm(p, tiny_spec.header(code), tiny_spec.build_tensor_list(dtype, ref_fmt, ref_q8, ref_q4))
            out[f"{dtype}_sha256"] = np.array(hashlib.sha256(p.read_bytes()).hexdigest())
            kvs = (("fp16", torch.float16), ("bf16", torch.bfloat16)) if dtype == "bf16" else (("fp16", torch.float16),)
            for kvn, kv in kvs:
                r = run_reference(p, tiny_spec.PROMPT, tiny_spec.N_NEW, kv, store_all=True)
                for k in ("ids", "logits_all", "res_all"):
                    out[f"{dtype}_{kvn}_{k}"] = r[k]
    np.savez_compressed(HERE / "golden_tiny.npz", **out)


def part_full(configs: list[str]) -> None:
    prompt = synth.prompt_ids(FULL_PROMPT_LEN, seed=0)
    for cfg in configs:
        dtype, kvn = cfg.split("_")
        path, digest = synth.ensure_model(dtype, seed=0, max_seq_len=4096)
        out = {"digest": np.array(digest), "prompt": np.array(prompt, dtype=np.int32)}
        if dtype != "bf16":
            # The reference quantiser on sampled blocks of the same bf16 values must give the file's bytes.
            table = {e["name"]: e for e in ref_fmt.read_table(path)}
            checks = []
            for name, block in (("layers.0.wqkv.weight", 0), ("layers.7.w_gate_up.weight", 5),
                                ("layers.15.w_down.weight", 0), ("tok_embeddings.weight", 62)):
                v = synth.block_values(0, name, block)
                q, s = ref_q8(v) if dtype == "int8" else ref_q4(v, 128)
                e = table[name]
                row_bytes = e["cols"] if dtype == "int8" else e["cols"] // 2
                stored = np.fromfile(path, dtype=np.uint8, count=q.nbytes,
                                     offset=e["offset"] + block * synth.BLOCK_ROWS * row_bytes)
                checks.append(bool(np.array_equal(stored, q.view(np.uint8).reshape(-1))))
            assert all(checks), f"{dtype}: reference quantiser disagrees with the generated file"
            out["quant_blocks_equal"] = np.array(checks)
        kv = torch.float16 if kvn == "fp16" else torch.bfloat16
        print(f"full {cfg}: running the reference", flush=True)
        r = run_reference(path, prompt, FULL_NEW, kv, keep_logits_at=(FULL_PROMPT_LEN - 1,),
                          keep_res_at=(0, FULL_PROMPT_LEN - 1))
        out.update(r)
        np.savez_compressed(HERE / f"golden_full_{cfg}.npz", **out)


LONG_PROMPT_LEN = 4096
LONG_NEW = 8
LONG_MAX_SEQ = 32896  # 32768 + 128: the long-context file serves both the 4096 and the 32768 contexts


def part_long() -> None:
    """ReferenceModel (bf16 KV) on the seeded bf16 weights in a max_seq_len 32896 file, prompted with 4096
    seeded random tokens, then 8 greedy tokens: ids, per-step top-8 over the last 64 prompt steps and the
    generated steps, full logits and residuals at the last prompt step -> golden_long_bf16_bf16.npz."""
    prompt = synth.prompt_ids(LONG_PROMPT_LEN, seed=0)
    path, digest = synth.ensure_model("bf16", seed=0, max_seq_len=LONG_MAX_SEQ)
    out = {"digest": np.array(digest), "prompt": np.array(prompt, dtype=np.int32), "max_seq_len": np.array(LONG_MAX_SEQ)}
    r = run_reference(path, prompt, LONG_NEW, torch.bfloat16, keep_logits_at=(LONG_PROMPT_LEN - 1,),
                      keep_res_at=(LONG_PROMPT_LEN - 1,))
    first = LONG_PROMPT_LEN - 64  # keep the per-step statistics of the tail only (the file stays small)
    for k in ("margin", "lsum", "lsq", "top8_i", "top8_v"):
        r[k] = r[k][first:]
    r["stats_first_step"] = np.array(first)
    out.update(r)
    np.savez_compressed(HERE / "golden_long_bf16_bf16.npz", **out)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--parts", nargs="+", default=["quant", "format", "tiny"])
    ap.add_argument("--full-configs", nargs="+", default=["bf16_fp16", "int8_fp16", "int4_fp16", "bf16_bf16"])
    args = ap.parse_args()
    if "long" in args.parts:
        part_long()
    if "quant" in args.parts:
        part_quant()
    if "format" in args.parts:
        part_format()
    if "tiny" in args.parts:
        part_tiny()
    if "full" in args.parts:
        part_full(args.full_configs)


if __name__ == "__main__":
    main()
