"""Python interface of libcudallm.so.

The public names and their arguments are those of wasiqnauman/cudallm's Python package
(python/cudallm/engine.py): `Engine(path, matvec=, attn=, fuse=, cuda_graph=, max_seq_len=, matvec_rpb=)`
with `step`, `step_debug`, `reset`, `pos`, `close`; the single-kernel hooks `kernel_matvec`,
`kernel_rmsnorm`, `kernel_rope_kv`, `kernel_attention`, `kernel_silu_mul`, `kernel_argmax`; and
`CudaLLMError(code, message)` for every nonzero return code. Code written against that package runs
against this one. Everything is bound through `abi` (signatures generated from include/cudallm.h).

Additions: `Engine(kv_dtype=, device=, path_kind=)` (cudallm_create_ex), `synchronize`, `step_async`,
`decode_path`, `stream_handle`, `device`, tracing and knobs; `BatchEngine` (cudallm_batch_*);
`kernel_gemm` (the batched path's tensor-core GEMM).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import abi
from .abi import CudaLLMError, addr, check, lib
from .paths import LIB_PATH

__all__ = ["BatchEngine", "CudaLLMError", "Engine", "LIB_PATH", "kernel_argmax", "kernel_attention", "kernel_gemm",
           "kernel_matvec", "kernel_rmsnorm", "kernel_rope_kv", "kernel_silu_mul", "lib"]

IMPLS = ("naive", "opt")
WEIGHT_CODES = {"bf16": 1, "int8": 3, "int4": 4}
EPILOGUES = ("store", "add", "swiglu")
KV_DTYPES = ("fp16", "bf16")
PATHS = ("auto", "persistent", "per_op")
BATCH_ATTN = ("auto", "stream", "split")


def _index(names: tuple[str, ...], v) -> int:
    """Position of a name in `names`, or an integer code passed through."""
    return names.index(v) if isinstance(v, str) else int(v)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _half_bits(a) -> np.ndarray:
    """Own copy of fp16 data (given as float16 values or as their uint16 bits) as uint16 bits."""
    a = np.asarray(a)
    return np.array(a.view(np.uint16) if a.dtype == np.float16 else a, dtype=np.uint16, order="C", copy=True)


class _Owned:
    """A handle of the library, released by `close` (also on `with` exit and garbage collection)."""

    _destroy = ""

    def __init__(self):
        self._h: ctypes.c_void_p | None = None

    def _handle(self) -> ctypes.c_void_p:
        if self._h is None:
            raise CudaLLMError(5, f"{type(self).__name__} is closed")
        return self._h

    def close(self) -> None:
        h, self._h = self._h, None
        if h is not None:
            getattr(lib(), self._destroy)(h)

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        if getattr(self, "_h", None) is not None:
            self.close()


def _config_dict(info) -> dict:
    return {name: getattr(info, name) for name, _ in info._fields_}


class Engine(_Owned):
    """Batch-1 decode of one sequence (cudallm_create / cudallm_step ...)."""

    _destroy = "cudallm_destroy"

    def __init__(self, path: Path | str, *, matvec: str = "opt", attn: str = "opt", fuse: bool = True,
                 cuda_graph: bool = True, max_seq_len: int = 0, matvec_rpb: int = 0, kv_dtype: str = "fp16",
                 device: int = -1, path_kind: str = "auto"):
        super().__init__()
        L = lib()
        opts = abi.struct("cudallm_options")(IMPLS.index(matvec), IMPLS.index(attn), int(bool(fuse)),
                                             int(bool(cuda_graph)), int(max_seq_len), int(matvec_rpb))
        ex = abi.struct("cudallm_options_ex")()
        L.cudallm_default_options_ex(ctypes.byref(ex))
        ex.kv_dtype, ex.device, ex.path = KV_DTYPES.index(kv_dtype), int(device), PATHS.index(path_kind)
        h = ctypes.c_void_p()
        check(L.cudallm_create_ex(str(path).encode(), ctypes.byref(opts), ctypes.byref(ex), ctypes.byref(h)))
        self._h = h
        info = abi.struct("cudallm_config_info")()
        check(L.cudallm_get_config(h, ctypes.byref(info)))
        self.config = _config_dict(info)

    @property
    def pos(self) -> int:
        return lib().cudallm_pos(self._handle())

    @property
    def decode_path(self) -> str:
        return {1: "persistent", 2: "per_op"}.get(lib().cudallm_engine_path(self._handle()), "unknown")

    @property
    def stream_handle(self) -> int:
        """The engine's cudaStream_t as an integer (for torch.cuda.ExternalStream)."""
        return lib().cudallm_engine_stream(self._handle()) or 0

    @property
    def device(self) -> int:
        return lib().cudallm_engine_device(self._handle())

    def reset(self) -> None:
        check(lib().cudallm_reset(self._handle()))

    def synchronize(self) -> None:
        check(lib().cudallm_synchronize(self._handle()))

    def step(self, token: int | None = None, *, want_logits: bool = False) -> tuple[int, np.ndarray | None]:
        """Feeds `token` (None: the previous argmax); returns (next token, logits if asked)."""
        nxt = np.zeros(1, dtype=np.int32)
        logits = np.empty(self.config["vocab"], dtype=np.float32) if want_logits else None
        check(lib().cudallm_step(self._handle(), -1 if token is None else int(token), addr(logits), addr(nxt)))
        return int(nxt[0]), logits

    def step_async(self, token: int | None = None) -> None:
        """Enqueues one step; nothing is waited for or copied back."""
        check(lib().cudallm_step(self._handle(), -1 if token is None else int(token), None, None))

    def prefill(self, tokens, *, want_logits: bool = False) -> tuple[int, np.ndarray | None]:
        """Feeds a prompt 64 tokens per batched step (cudallm_prefill): (argmax after the last token, its
        logits if asked); a following step(None) continues from that argmax."""
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        nxt = np.zeros(1, dtype=np.int32)
        logits = np.empty(self.config["vocab"], dtype=np.float32) if want_logits else None
        check(lib().cudallm_prefill(self._handle(), addr(t), t.size, addr(logits), addr(nxt)))
        return int(nxt[0]), logits

    def step_debug(self, token: int | None = None) -> tuple[int, np.ndarray, np.ndarray]:
        """One step without graph replay: (next token, logits, residuals [n_layers + 1][hidden])."""
        c = self.config
        nxt = np.zeros(1, dtype=np.int32)
        logits = np.empty(c["vocab"], dtype=np.float32)
        residuals = np.empty((c["n_layers"] + 1, c["hidden"]), dtype=np.float32)
        check(lib().cudallm_step_debug(self._handle(), -1 if token is None else int(token), addr(residuals),
                                       addr(logits), addr(nxt)))
        return int(nxt[0]), logits, residuals

    def set_knob(self, name: str, value: int) -> None:
        """Tuning / test knob of the persistent step (cudallm_debug_set)."""
        check(lib().cudallm_debug_set(self._handle(), name.encode(), int(value)))

    def set_sampling(self, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0, seed: int = 0) -> None:
        """Next-token rule (cudallm_set_sampling): temperature 0 = greedy; else top-k / top-p sampling drawn
        from (seed, position)."""
        check(lib().cudallm_set_sampling(self._handle(), float(temperature), int(top_k), float(top_p), int(seed)))

    def trace(self, enable: bool = True) -> None:
        """Per-CTA timestamps of each following step (persistent path only)."""
        check(lib().cudallm_debug_trace(self._handle(), int(bool(enable))))

    def read_trace(self, grid: int = 1024, slots: int = 82 * 6) -> tuple[np.ndarray, np.ndarray]:
        """Last traced step: (uint64 [grid][ops][6] per-CTA stamps, uint64 [256][5] tile stamps of CTA 0),
        nanoseconds (layout in csrc/engine/decode_step.h)."""
        buf = np.zeros(grid * slots + 256 * 5, dtype=np.uint64)
        shape = np.zeros(2, dtype=np.int32)
        check(lib().cudallm_debug_read_trace(self._handle(), addr(buf), buf.size, addr(shape), addr(shape) + 4))
        n = int(shape[0]) * int(shape[1])
        return buf[:n].reshape(int(shape[0]), int(shape[1]) // 6, 6), buf[n:n + 256 * 5].reshape(256, 5)


class BatchEngine(_Owned):
    """Batched decode of up to 64 independent sequences on one GPU (cudallm_batch_*)."""

    _destroy = "cudallm_batch_destroy"

    def __init__(self, path: Path | str, *, n_seq: int = 64, max_seq_len: int = 0, kv_dtype: str = "fp16",
                 device: int = -1, cuda_graph: bool = True, attn: str = "auto"):
        super().__init__()
        L = lib()
        opts = abi.struct("cudallm_batch_options")()
        L.cudallm_default_batch_options(ctypes.byref(opts))
        opts.n_seq, opts.max_seq_len, opts.kv_dtype = int(n_seq), int(max_seq_len), KV_DTYPES.index(kv_dtype)
        opts.device, opts.cuda_graph, opts.attn_mode = int(device), int(bool(cuda_graph)), BATCH_ATTN.index(attn)
        h = ctypes.c_void_p()
        check(L.cudallm_batch_create(str(path).encode(), ctypes.byref(opts), ctypes.byref(h)))
        self._h = h
        info = abi.struct("cudallm_config_info")()
        check(L.cudallm_batch_get_config(h, ctypes.byref(info)))
        self.config = _config_dict(info)
        self.n_seq = int(n_seq)

    def pos(self, seq: int) -> int:
        return lib().cudallm_batch_pos(self._handle(), int(seq))

    @property
    def stream_handle(self) -> int:
        return lib().cudallm_batch_stream(self._handle()) or 0

    def reset(self, seq: int = -1) -> None:
        check(lib().cudallm_batch_reset(self._handle(), int(seq)))

    def synchronize(self) -> None:
        check(lib().cudallm_batch_synchronize(self._handle()))

    def set_knob(self, name: str, value: int) -> None:
        check(lib().cudallm_batch_debug_set(self._handle(), name.encode(), int(value)))

    def knob(self, name: str) -> int:
        out = np.zeros(1, dtype=np.int64)
        check(lib().cudallm_batch_debug_get(self._handle(), name.encode(), addr(out)))
        return int(out[0])

    def _tokens(self, tokens) -> np.ndarray | None:
        if tokens is None:
            return None
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if t.shape != (self.n_seq,):
            raise ValueError(f"tokens must have shape ({self.n_seq},)")
        return t

    def step(self, tokens=None, *, want_logits: bool = False) -> tuple[np.ndarray, np.ndarray | None]:
        """One step of every sequence: tokens [n_seq] (-1 = that sequence's previous argmax; None = all -1)
        -> (next token per sequence, logits [n_seq][vocab] if asked)."""
        t = self._tokens(tokens)
        nxt = np.empty(self.n_seq, dtype=np.int32)
        logits = np.empty((self.n_seq, self.config["vocab"]), dtype=np.float32) if want_logits else None
        check(lib().cudallm_batch_step(self._handle(), addr(t), addr(nxt), addr(logits)))
        return nxt, logits

    def step_async(self, tokens=None) -> None:
        """Enqueues one step; nothing is waited for or copied back."""
        check(lib().cudallm_batch_step(self._handle(), addr(self._tokens(tokens)), None, None))

    def prefill(self, seq: int, tokens, *, want_logits: bool = False) -> tuple[int, np.ndarray | None]:
        """Prompt prefill of one sequence, 64 of its tokens per batched step (cudallm_batch_prefill)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        nxt = np.zeros(1, dtype=np.int32)
        logits = np.empty(self.config["vocab"], dtype=np.float32) if want_logits else None
        check(lib().cudallm_batch_prefill(self._handle(), int(seq), addr(t), t.size, addr(logits), addr(nxt)))
        return int(nxt[0]), logits


def kernel_matvec(impl: str | int, wtype: str | int, epilogue: str | int, fuse_norm: bool | int, rpb: int,
                  w: np.ndarray, scales: np.ndarray | None, x: np.ndarray, norm_w: np.ndarray | None, eps: float,
                  y_init: np.ndarray | None, rows: int, cols: int) -> np.ndarray:
    """y = W x with the epilogue (store / add onto y_init / swiglu -> rows/2 outputs), optional fused RMSNorm."""
    ep = _index(EPILOGUES, epilogue)
    n_out = rows // 2 if ep == 2 else rows
    wb = np.ascontiguousarray(w)
    sb = None if scales is None else np.ascontiguousarray(scales)
    y = np.zeros(n_out, dtype=np.float32) if y_init is None else np.array(y_init, dtype=np.float32, copy=True)
    if y.shape != (n_out,):
        raise ValueError(f"y_init must have shape ({n_out},)")
    xv = _f32(x)
    nv = None if norm_w is None else _f32(norm_w)
    wcode = WEIGHT_CODES[wtype] if isinstance(wtype, str) else int(wtype)
    check(lib().cudallm_kernel_matvec(_index(IMPLS, impl), wcode, ep, int(bool(fuse_norm)), int(rpb), addr(wb), wb.nbytes,
                                      addr(sb), 0 if sb is None else sb.nbytes, addr(xv), addr(nv), float(eps), addr(y),
                                      int(rows), int(cols)))
    return y


def kernel_rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    xv, wv = _f32(x), _f32(w)
    y = np.empty_like(xv)
    check(lib().cudallm_kernel_rmsnorm(addr(xv), addr(wv), float(eps), addr(y), xv.size))
    return y


def kernel_rope_kv(fused: bool | int, qkv: np.ndarray, inv_freq: np.ndarray, pos: int, k_cache: np.ndarray,
                   v_cache: np.ndarray, nh: int, nkv: int, hd: int,
                   max_seq: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """RoPE on q and k, k/v written at `pos` of the fp16 caches: returns (qkv, k_cache, v_cache) (new arrays)."""
    q = np.array(qkv, dtype=np.float32, copy=True)
    f = _f32(inv_freq)
    k, v = _half_bits(k_cache), _half_bits(v_cache)
    check(lib().cudallm_kernel_rope_kv(int(bool(fused)), addr(q), addr(f), int(pos), addr(k), addr(v), nh, nkv, hd,
                                       max_seq))
    return q, k.view(np.float16), v.view(np.float16)


def kernel_attention(impl: str | int, q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, ctx: int, nh: int,
                     nkv: int, hd: int, max_seq: int) -> np.ndarray:
    """Decode attention of nh query heads over the first ctx cached positions (fp16 caches [nkv][max_seq][hd])."""
    qv = _f32(q)
    k, v = _half_bits(k_cache), _half_bits(v_cache)
    out = np.empty(nh * hd, dtype=np.float32)
    check(lib().cudallm_kernel_attention(_index(IMPLS, impl), addr(qv), addr(k), addr(v), int(ctx), addr(out), nh, nkv,
                                         hd, max_seq))
    return out


def kernel_silu_mul(gu: np.ndarray) -> np.ndarray:
    g = _f32(gu)
    act = np.empty(g.size // 2, dtype=np.float32)
    check(lib().cudallm_kernel_silu_mul(addr(g), addr(act), act.size))
    return act


def kernel_argmax(logits: np.ndarray) -> int:
    lg = _f32(logits)
    idx = np.full(1, -1, dtype=np.int32)
    check(lib().cudallm_kernel_argmax(addr(lg), lg.size, addr(idx)))
    return int(idx[0])


def kernel_gemm(w_bits: np.ndarray, x_bits: np.ndarray, *, x_lo_bits: np.ndarray | None = None, ksplit: int = 1,
                epilogue: str = "store", y: np.ndarray | None = None) -> np.ndarray:
    """Batched-path GEMM hook: w_bits [n][k], x_bits (plus optional x_lo_bits, added to x) [batch][k] bf16 bits
    (uint16) -> fp32 [batch][n] (store / add onto y) or [batch][n/2] (swiglu)."""
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    lo = None if x_lo_bits is None else np.ascontiguousarray(x_lo_bits, dtype=np.uint16)
    if lo is not None and lo.shape != x.shape:
        raise ValueError("x_lo_bits must have the shape of x_bits")
    n, k = w.shape
    ep = EPILOGUES.index(epilogue)
    shape = (x.shape[0], n // 2 if ep == 2 else n)
    out = np.zeros(shape, dtype=np.float32) if y is None else np.array(y, dtype=np.float32, copy=True)
    check(lib().cudallm_kernel_gemm(addr(w), addr(x), addr(lo), addr(out), n, k, x.shape[0], int(ksplit), ep))
    return out
