"""Calibrated int4 weights (GPTQ) written in the unchanged .cudallm int4 layout.

    python -m cudallm_b200.gptq SRC_BF16.cudallm DST_INT4.cudallm [--tokens 1024] [--seed 7]
    python -m cudallm_b200.gptq --eval | --eval-engine BF16 INT4_A [INT4_B ...] [--eval-tokens 64]

The reference quantiser (wasiqnauman/cudallm python/cudallm/quantize.py:14-29, restated in quantize.py) rounds
every weight to its nearest level independently (RTN). This module instead chooses the levels with the GPTQ
procedure (Frantar, Ashkboos, Hoefler, Alistarh, "GPTQ: Accurate Post-Training Quantization for Generative
Pre-trained Transformers", 2022): for a linear layer y = W x with calibration inputs X, it minimises
||(W - Q) X||^2 column by column, quantising one input column at a time and spreading that column's rounding
error over the columns not yet quantised with the inverse of the input Hessian H = X^T X (through the upper
Cholesky factor of H^-1). Layers are processed in order, each calibrated on inputs produced by the layers
before it already quantised.

The output is an ordinary int4 file: the same packed nibbles (q + 8, even column in the low nibble), fp16
scales per 128-column group (max |w| / 7 of the group's weights at the moment its first column is reached)
and the same tensor table, so the loader, the batch-1 and batched engines and the reference's own tools read
it unchanged; only the chosen codes differ from RTN. The tied token embedding / lm_head stays RTN (its rows
are also looked up as embeddings, where error feedback across columns has no meaning).

Calibration data: seeded random token sequences (no text corpus is available here), run through a float32
restatement of the Llama-3.2 forward pass in this module (RMSNorm, rotate-half RoPE with the file's inv_freq,
causal GQA attention, SwiGLU). `--eval` compares files by teacher-forced logits against the bf16 model on a
different seeded sequence (relative L2 error, top-1 agreement, mean KL divergence).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

from . import format as fmt
from .quantize import INT4_GROUP, quantize_int4_groups

LINEARS = ("wqkv", "wo", "w_gate_up", "w_down")


def gptq_int4(w: np.ndarray, hessian: np.ndarray, group: int = INT4_GROUP, damp: float = 0.01) -> tuple[np.ndarray, np.ndarray]:
    """GPTQ codes of w [rows][cols] (float32) for inputs with Hessian `hessian` [cols][cols] (X^T X), in the
    .cudallm int4 layout: (packed uint8 [rows][cols/2], fp16 scales [rows][cols/group]). Columns are taken in
    order in blocks of one group; a column whose Hessian diagonal is zero (an input that never varies) is
    quantised as zero. `damp` adds that fraction of the mean Hessian diagonal to the diagonal."""
    W = torch.from_numpy(np.array(w, dtype=np.float32, copy=True))
    rows, cols = W.shape
    if cols % group or group % 2:
        raise ValueError("gptq_int4: cols must be a multiple of the (even) group size")
    H = torch.from_numpy(np.array(hessian, dtype=np.float64, copy=True))
    if H.shape != (cols, cols):
        raise ValueError("gptq_int4: hessian must be [cols][cols]")
    dead = torch.diagonal(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    H += damp * torch.mean(torch.diagonal(H)) * torch.eye(cols, dtype=H.dtype)
    hinv = torch.cholesky_inverse(torch.linalg.cholesky(H))
    U = torch.linalg.cholesky(hinv, upper=True).to(torch.float32)  # H^-1 = U^T U
    codes = torch.empty((rows, cols), dtype=torch.int8)
    scales = torch.empty((rows, cols // group), dtype=torch.float16)
    for b0 in range(0, cols, group):
        b1 = b0 + group
        W1 = W[:, b0:b1].clone()
        E1 = torch.empty_like(W1)
        U1 = U[b0:b1, b0:b1]
        s = torch.amax(torch.abs(W1), dim=1) / 7.0
        s = torch.where(s == 0, torch.ones_like(s), s)
        s16 = s.to(torch.float16)
        sf = s16.to(torch.float32)
        scales[:, b0 // group] = s16
        for i in range(group):
            col = W1[:, i]
            q = torch.clamp(torch.round(col / sf), -8, 7)  # round half to even, as the reference's np.rint
            err = (col - q * sf) / U1[i, i]
            W1[:, i:] -= err[:, None] * U1[i, i:][None, :]
            E1[:, i] = err
            codes[:, b0 + i] = q.to(torch.int8)
        if b1 < cols:
            W[:, b1:] -= E1 @ U[b0:b1, b1:]
    u = (codes.numpy().astype(np.int16) + 8).astype(np.uint8)
    packed = (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)
    return packed, scales.numpy()


# ---- float32 forward pass used for calibration and evaluation ------------------------------------------

def _rms(x: torch.Tensor, g: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps) * g


def _rope(v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """v [T][heads][d], rotate-half: (a c - b s, b c + a s) over the two halves of each head."""
    half = v.shape[-1] // 2
    a, b = v[..., :half], v[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1)


class _File:
    """Tensors of a .cudallm file as float32 torch tensors (quantised ones dequantised), read on demand."""

    def __init__(self, path: Path | str):
        self.path = Path(path)
        self.hdr = fmt.read_header(self.path)
        self.table = {e["name"]: e for e in fmt.read_table(self.path)}

    def vec(self, name: str) -> torch.Tensor:
        return torch.from_numpy(fmt.load_tensor(self.path, self.table[name]).astype(np.float32))

    def mat(self, name: str) -> torch.Tensor:
        e = self.table[name + ".weight"]
        w = fmt.load_tensor(self.path, e)
        if e["dtype"] == fmt.BF16:
            return torch.from_numpy(fmt.bf16_bits_to_f32(w))
        s = fmt.load_tensor(self.path, self.table[name + ".scales"])
        if e["dtype"] == fmt.I8:
            return torch.from_numpy(w.astype(np.float32) * s.astype(np.float32)[:, None])
        from .quantize import dequantize_int4_groups
        return torch.from_numpy(dequantize_int4_groups(w, s))


class _Layer:
    def __init__(self, f: _File, i: int, override: dict | None = None):
        p = f"layers.{i}."
        self.attn_norm = f.vec(p + "attn_norm.weight")
        self.ffn_norm = f.vec(p + "ffn_norm.weight")
        self.w = {n: (override[n] if override and n in override else f.mat(p + n)) for n in LINEARS}


def _layer_forward(L: _Layer, x: torch.Tensor, hdr: dict, cos: torch.Tensor, sin: torch.Tensor,
                   capture: dict | None = None) -> torch.Tensor:
    """x [T][H] (one causal sequence) -> layer output; capture[name] gets each linear's input [T][K]."""
    T = x.shape[0]
    NH, KV, D, I = hdr["n_heads"], hdr["n_kv_heads"], hdr["head_dim"], hdr["intermediate_size"]
    eps = hdr["rms_eps"]
    xn = _rms(x, L.attn_norm, eps)
    qkv = xn @ L.w["wqkv"].T
    q = _rope(qkv[:, :NH * D].view(T, NH, D), cos, sin)
    k = _rope(qkv[:, NH * D:(NH + KV) * D].view(T, KV, D), cos, sin)
    v = qkv[:, (NH + KV) * D:].view(T, KV, D)
    rep = NH // KV
    k = k.repeat_interleave(rep, dim=1)
    v = v.repeat_interleave(rep, dim=1)
    s = torch.einsum("thd,shd->hts", q, k) * (1.0 / np.sqrt(D))
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool), diagonal=1)
    s = s.masked_fill(mask[None], float("-inf"))
    att = torch.einsum("hts,shd->thd", torch.softmax(s, dim=-1), v).reshape(T, NH * D)
    h = x + att @ L.w["wo"].T
    hn = _rms(h, L.ffn_norm, eps)
    gu = hn @ L.w["w_gate_up"].T
    act = gu[:, :I] / (1.0 + torch.exp(-gu[:, :I])) * gu[:, I:]
    if capture is not None:
        capture["wqkv"], capture["wo"], capture["w_gate_up"], capture["w_down"] = xn, att, hn, act
    return h + act @ L.w["w_down"].T


def _rope_tables(f: _File, T: int) -> tuple[torch.Tensor, torch.Tensor]:
    ang = torch.arange(T, dtype=torch.float32)[:, None] * f.vec("rope.inv_freq")[None, :]
    return torch.cos(ang), torch.sin(ang)


def _embed(f: _File, tokens: list[int]) -> torch.Tensor:
    e = f.table["tok_embeddings.weight"]
    rows = np.asarray(tokens)
    w = np.memmap(f.path, dtype=np.uint16 if e["dtype"] == fmt.BF16 else np.uint8, mode="r", offset=e["offset"],
                  shape=(e["rows"], e["cols"] if e["dtype"] != fmt.I4X2 else e["cols"] // 2))
    if e["dtype"] == fmt.BF16:
        return torch.from_numpy(fmt.bf16_bits_to_f32(np.array(w[rows])))
    return f.mat("tok_embeddings")[rows]


# ---- calibrated file ---------------------------------------------------------------------------------

def calibrate(src: Path | str, dst: Path | str, n_tokens: int = 1024, seq_len: int = 256, seed: int = 7,
              damp: float = 0.01, log=print) -> dict:
    """Writes dst, an int4 .cudallm whose layer weights are GPTQ-quantised from the bf16 file src on n_tokens
    seeded random tokens (sequences of seq_len); the tied embedding is quantised by RTN. Returns a summary."""
    f = _File(src)
    hdr = dict(f.hdr)
    if hdr["weight_dtype"] != fmt.WEIGHT_BF16:
        raise ValueError("calibrate: the source file must hold bf16 weights")
    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(seed)
    n_seq = max(1, n_tokens // seq_len)
    seqs = [rng.integers(0, hdr["vocab_size"], seq_len).tolist() for _ in range(n_seq)]
    cos, sin = _rope_tables(f, seq_len)
    xs = [_embed(f, s) for s in seqs]
    out: dict[str, tuple[np.ndarray, np.ndarray]] = {}
    t0 = time.time()
    err = {"gptq": 0.0, "rtn": 0.0}
    with torch.no_grad():
        for li in range(hdr["n_layers"]):
            L = _Layer(f, li)
            H = {n: None for n in LINEARS}
            for x in xs:
                cap: dict = {}
                _layer_forward(L, x, hdr, cos, sin, cap)
                for n in LINEARS:
                    xx = cap[n].double()
                    H[n] = xx.T @ xx if H[n] is None else H[n] + xx.T @ xx
            quant = {}
            for n in LINEARS:
                w = L.w[n].numpy()
                packed, scales = gptq_int4(w, H[n].numpy(), damp=damp)
                out[f"layers.{li}.{n}"] = (packed, scales)
                from .quantize import dequantize_int4_groups
                wq = dequantize_int4_groups(packed, scales)
                rp, rs = quantize_int4_groups(w)
                wr = dequantize_int4_groups(rp, rs)
                Hn = H[n].float()
                for key, a in (("gptq", wq), ("rtn", wr)):
                    d = torch.from_numpy(w - a)
                    err[key] += float(torch.sum((d @ Hn) * d))
                quant[n] = torch.from_numpy(wq)
            Lq = _Layer(f, li, override=quant)
            xs = [_layer_forward(Lq, x, hdr, cos, sin) for x in xs]
            log(f"layer {li}: done ({time.time() - t0:.0f} s)")
    # Tied embedding / lm_head: RTN, as the reference's quantiser does.
    emb = f.mat("tok_embeddings").numpy()
    tensors = []
    for name in fmt.expected_names(hdr["n_layers"], True):
        if name == "tok_embeddings.weight":
            ep, es = quantize_int4_groups(emb)
            tensors.append((name, fmt.I4X2, emb.shape[0], emb.shape[1], ep.tobytes()))
            tensors.append(("tok_embeddings.scales", fmt.F16, es.shape[0], es.shape[1], es.tobytes()))
        elif name == "tok_embeddings.scales" or name.endswith(".scales"):
            continue
        elif name.endswith(".weight") and any(name.endswith(n + ".weight") for n in LINEARS):
            key = name[: -len(".weight")]
            packed, scales = out[key]
            cols = packed.shape[1] * 2
            tensors.append((name, fmt.I4X2, packed.shape[0], cols, packed.tobytes()))
            tensors.append((key + ".scales", fmt.F16, scales.shape[0], scales.shape[1], scales.tobytes()))
        else:
            e = f.table[name]
            tensors.append((name, e["dtype"], e["rows"], e["cols"], fmt.load_tensor(f.path, e).tobytes()))
    hdr["weight_dtype"] = fmt.WEIGHT_INT4
    hdr["group_size"] = INT4_GROUP
    tmp = Path(str(dst) + ".partial")
    fmt.write_cudallm(tmp, hdr, tensors)
    os.replace(tmp, dst)
    return {"calibration_tokens": n_seq * seq_len, "seed": seed, "damp": damp, "seconds": time.time() - t0,
            "weighted_error_gptq_over_rtn": err["gptq"] / err["rtn"] if err["rtn"] else float("nan")}


# ---- evaluation ------------------------------------------------------------------------------------------

def evaluate(ref: Path | str, candidates: list[Path | str], n_tokens: int = 64, seed: int = 11) -> dict:
    """Teacher-forced logits of each candidate file against the reference file's on one seeded sequence."""
    torch.set_num_threads(os.cpu_count() or 1)

    def logits(path: Path | str, tokens: list[int]) -> torch.Tensor:
        f = _File(path)
        hdr = f.hdr
        cos, sin = _rope_tables(f, len(tokens))
        with torch.no_grad():
            x = _embed(f, tokens)
            for li in range(hdr["n_layers"]):
                x = _layer_forward(_Layer(f, li), x, hdr, cos, sin)
            x = _rms(x, f.vec("norm.weight"), hdr["rms_eps"])
            return x @ f.mat("tok_embeddings").T

    vocab = fmt.read_header(ref)["vocab_size"]
    tokens = np.random.default_rng(seed).integers(0, vocab, n_tokens).tolist()
    base = logits(ref, tokens)
    pb = torch.log_softmax(base, dim=-1)
    res = {}
    for c in candidates:
        lc = logits(c, tokens)
        pc = torch.log_softmax(lc, dim=-1)
        res[str(c)] = {
            "logits_rel_l2": float(torch.linalg.norm(lc - base) / torch.linalg.norm(base)),
            "top1_agreement": float(torch.mean((torch.argmax(lc, -1) == torch.argmax(base, -1)).float())),
            "mean_kl": float(torch.mean(torch.sum(torch.exp(pb) * (pb - pc), dim=-1))),
        }
    return {"tokens": n_tokens, "seed": seed, "results": res}


def layer_errors(ref: Path | str, candidates: list[Path | str], layers: list[int], n_tokens: int = 256,
                 seed: int = 11) -> dict:
    """Relative output error ||(W - Wq) X|| / ||W X|| of every linear of the given layers, for each candidate
    file's weights Wq, on inputs X that the reference (bf16) model produces for a seeded held-out sequence. A
    local measure of quantisation quality that does not depend on how the whole network amplifies errors."""
    torch.set_num_threads(os.cpu_count() or 1)
    f = _File(ref)
    hdr = f.hdr
    tokens = np.random.default_rng(seed).integers(0, hdr["vocab_size"], n_tokens).tolist()
    cos, sin = _rope_tables(f, n_tokens)
    cands = [_File(c) for c in candidates]
    res = {str(c): {} for c in candidates}
    with torch.no_grad():
        x = _embed(f, tokens)
        for li in range(max(layers) + 1):
            L = _Layer(f, li)
            cap: dict = {}
            x_next = _layer_forward(L, x, hdr, cos, sin, cap)
            if li in layers:
                for n in LINEARS:
                    ref_out = cap[n] @ L.w[n].T
                    for c, cf in zip(candidates, cands):
                        wq = cf.mat(f"layers.{li}.{n}")
                        res[str(c)][f"layers.{li}.{n}"] = float(torch.linalg.norm(cap[n] @ (L.w[n] - wq).T) /
                                                                torch.linalg.norm(ref_out))
            x = x_next
    return {"tokens": n_tokens, "seed": seed, "results": res}


def evaluate_engine(ref: Path | str, candidates: list[Path | str], n_tokens: int = 64, seed: int = 11) -> dict:
    """As evaluate, with every file run by this library's decode engine on the GPU (persistent step, fp16 KV):
    the quality the engine actually serves."""
    from .engine import Engine

    def logits(path: Path | str, tokens: list[int]) -> np.ndarray:
        out = []
        with Engine(path) as eng:
            for t in tokens:
                _, lg = eng.step(t, want_logits=True)
                out.append(np.asarray(lg, dtype=np.float64))
        return np.stack(out)

    def log_softmax(a: np.ndarray) -> np.ndarray:
        m = a.max(axis=-1, keepdims=True)
        return a - m - np.log(np.sum(np.exp(a - m), axis=-1, keepdims=True))

    vocab = fmt.read_header(ref)["vocab_size"]
    tokens = np.random.default_rng(seed).integers(0, vocab, n_tokens).tolist()
    base = logits(ref, tokens)
    pb = log_softmax(base)
    res = {}
    for c in candidates:
        lc = logits(c, tokens)
        pc = log_softmax(lc)
        res[str(c)] = {"logits_rel_l2": float(np.linalg.norm(lc - base) / np.linalg.norm(base)),
                       "top1_agreement": float(np.mean(np.argmax(lc, -1) == np.argmax(base, -1))),
                       "mean_kl": float(np.mean(np.sum(np.exp(pb) * (pb - pc), axis=-1)))}
    return {"tokens": n_tokens, "seed": seed, "engine": True, "results": res}


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="GPTQ-calibrated int4 .cudallm files")
    ap.add_argument("paths", nargs="+")
    ap.add_argument("--eval", action="store_true", help="paths = reference file then candidates (CPU forward)")
    ap.add_argument("--eval-engine", action="store_true", help="as --eval, run by the decode engine on the GPU")
    ap.add_argument("--tokens", type=int, default=1024)
    ap.add_argument("--seq-len", type=int, default=256)
    ap.add_argument("--seed", type=int, default=7)
    ap.add_argument("--damp", type=float, default=0.01)
    ap.add_argument("--eval-tokens", type=int, default=64)
    args = ap.parse_args(argv)
    if args.eval or args.eval_engine:
        ev = evaluate_engine if args.eval_engine else evaluate
        print(json.dumps(ev(args.paths[0], args.paths[1:], args.eval_tokens)))
        return 0
    if len(args.paths) != 2:
        ap.error("calibration takes SRC and DST")
    print(json.dumps(calibrate(args.paths[0], args.paths[1], args.tokens, args.seq_len, args.seed, args.damp,
                               log=lambda m: print(m, file=sys.stderr, flush=True))))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
