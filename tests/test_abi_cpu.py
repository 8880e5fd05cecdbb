"""CPU: the C-ABI library loads, exports every symbol include/cudallm.h declares, and reports the
host-side errors (arguments, files) with the reference's error codes without touching a GPU."""
from __future__ import annotations

import ctypes
import re
import struct
import subprocess
from pathlib import Path

import numpy as np
import pytest

from cudallm_b200 import abi
from cudallm_b200 import engine as E
from cudallm_b200 import format as fmt

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "cudallm.h"

ERR_INVALID_ARG, ERR_IO, ERR_FORMAT = 1, 2, 3


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(cudallm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_reference_abi():
    names = declared_functions()
    reference_15 = ["cudallm_last_error", "cudallm_default_options", "cudallm_create", "cudallm_destroy",
                    "cudallm_get_config", "cudallm_reset", "cudallm_pos", "cudallm_step", "cudallm_step_debug",
                    "cudallm_kernel_matvec", "cudallm_kernel_rmsnorm", "cudallm_kernel_rope_kv",
                    "cudallm_kernel_attention", "cudallm_kernel_silu_mul", "cudallm_kernel_argmax"]
    assert set(reference_15) <= set(names)


def test_library_exports_every_declared_symbol(native_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(E.LIB_PATH)], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    assert set(abi.declarations()[1]) == set(declared_functions())


def test_struct_layouts():
    """The structs generated from the header have the reference's sizes (cudallm.h:18-32) and the additive ones."""
    assert ctypes.sizeof(abi.struct("cudallm_options")) == 24
    assert ctypes.sizeof(abi.struct("cudallm_config_info")) == 56
    assert ctypes.sizeof(abi.struct("cudallm_options_ex")) == 32
    assert ctypes.sizeof(abi.struct("cudallm_batch_options")) == 40


def test_signatures_follow_the_header():
    _, funcs = abi.declarations()
    args, ret = funcs["cudallm_kernel_matvec"]
    assert len(args) == 15 and ret is ctypes.c_int
    assert args[6] is ctypes.c_ulonglong and args[11] is ctypes.c_float
    assert funcs["cudallm_last_error"] == ([], ctypes.c_char_p)
    assert funcs["cudallm_create"][0][2] is ctypes.POINTER(ctypes.c_void_p)
    assert funcs["cudallm_debug_set"][0] == [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_longlong]


def test_default_options(native_lib):
    o = abi.struct("cudallm_options")()
    native_lib.cudallm_default_options(ctypes.byref(o))
    assert (o.matvec_impl, o.attn_impl, o.fuse, o.cuda_graph, o.max_seq_len, o.matvec_rpb) == (1, 1, 1, 1, 0, 0)
    native_lib.cudallm_default_options(None)  # NULL-safe
    ex = abi.struct("cudallm_options_ex")()
    native_lib.cudallm_default_options_ex(ctypes.byref(ex))
    assert (ex.struct_size, ex.kv_dtype, ex.device, ex.path) == (32, 0, -1, 0)


def _create(native_lib, path, **over) -> tuple[int, str]:
    o = abi.struct("cudallm_options")()
    native_lib.cudallm_default_options(ctypes.byref(o))
    for k, v in over.items():
        setattr(o, k, v)
    h = ctypes.c_void_p(123)
    rc = native_lib.cudallm_create(str(path).encode() if path is not None else None, ctypes.byref(o), ctypes.byref(h))
    msg = native_lib.cudallm_last_error().decode()
    if rc == 0:
        native_lib.cudallm_destroy(h)
    return rc, msg


def test_create_null_arguments(native_lib):
    rc, msg = _create(native_lib, None)
    assert rc == ERR_INVALID_ARG and "null" in msg


def test_create_missing_file(native_lib, tmp_path):
    rc, msg = _create(native_lib, tmp_path / "nope.cudallm")
    assert rc == ERR_IO and "cannot open" in msg


def _header_bytes(**over) -> bytes:
    h = {"weight_dtype": 1, "hidden_size": 2048, "intermediate_size": 8192, "n_layers": 16, "n_heads": 32,
         "n_kv_heads": 8, "head_dim": 64, "vocab_size": 128256, "max_seq_len": 4096, "rms_eps": 1e-5,
         "rope_theta": 500000.0, "group_size": 0}
    h.update(over)
    return fmt.pack_header(h, 99)


@pytest.mark.parametrize("case", ["bad_magic", "truncated", "wrong_hidden", "bad_dtype", "bad_max_seq", "no_table"])
def test_create_bad_files(native_lib, tmp_path, case):
    p = tmp_path / f"{case}.cudallm"
    if case == "bad_magic":
        p.write_bytes(b"XXXX" + _header_bytes()[4:])
    elif case == "truncated":
        p.write_bytes(_header_bytes()[:100])
    elif case == "wrong_hidden":
        p.write_bytes(_header_bytes(hidden_size=1024))
    elif case == "bad_dtype":
        p.write_bytes(_header_bytes(weight_dtype=2))
    elif case == "bad_max_seq":
        p.write_bytes(_header_bytes(max_seq_len=100))
    else:
        p.write_bytes(_header_bytes())  # header claims 99 tensors, no table follows
    rc, msg = _create(native_lib, p)
    assert rc == ERR_FORMAT, msg


def test_create_bad_table_entry(native_lib, tmp_path):
    """A table whose first entry has the wrong name is rejected as FORMAT before any device work."""
    entries, _ = fmt.plan_layout([("rope.inv_freqX", fmt.F32, 32, 1)] + [("x", fmt.F32, 1, 1)] * 98)
    p = tmp_path / "t.cudallm"
    p.write_bytes(_header_bytes() + fmt.pack_table(entries))
    rc, msg = _create(native_lib, p)
    assert rc == ERR_FORMAT and "rope.inv_freqX" in msg


def test_options_rejected_before_device_work(native_lib, model_path):
    path, _ = model_path("int8")
    rc, msg = _create(native_lib, path, matvec_impl=0, fuse=0)
    assert rc == ERR_INVALID_ARG and "naive matvec requires bf16" in msg
    rc, msg = _create(native_lib, path, matvec_rpb=3)
    assert rc == ERR_INVALID_ARG
    rc, msg = _create(native_lib, path, max_seq_len=100)
    assert rc == ERR_INVALID_ARG
    rc, msg = _create(native_lib, path, max_seq_len=8192)
    assert rc == ERR_INVALID_ARG and "exceeds" in msg
    rc, msg = _create(native_lib, path, matvec_impl=5)
    assert rc == ERR_INVALID_ARG


def test_null_engine_calls(native_lib):
    assert native_lib.cudallm_pos(None) == -1
    native_lib.cudallm_destroy(None)
    assert native_lib.cudallm_reset(None) == ERR_INVALID_ARG
    assert native_lib.cudallm_step(None, 0, None, None) == ERR_INVALID_ARG
    assert native_lib.cudallm_synchronize(None) == ERR_INVALID_ARG
    info = abi.struct("cudallm_config_info")()
    assert native_lib.cudallm_get_config(None, ctypes.byref(info)) == ERR_INVALID_ARG


def test_kernel_hooks_reject_bad_arguments(native_lib):
    x = np.zeros(2048, dtype=np.float32)
    with pytest.raises(E.CudaLLMError) as e:
        E.kernel_matvec(2, "bf16", "store", 0, 0, np.zeros((4, 2048), np.uint16), None, x, None, 1e-5, None, 4, 2048)
    assert e.value.code == ERR_INVALID_ARG
    with pytest.raises(E.CudaLLMError) as e:
        E.kernel_matvec("naive", "int8", "store", 0, 0, np.zeros((4, 2048), np.int8), np.ones(4, np.float32), x, None,
                        1e-5, None, 4, 2048)
    assert e.value.code == ERR_INVALID_ARG and "naive requires bf16" in str(e.value)
    with pytest.raises(E.CudaLLMError) as e:
        E.kernel_matvec("opt", "int4", "store", 0, 0, np.zeros((4, 1024), np.uint8), None, x, None, 1e-5, None, 4, 2048)
    assert e.value.code == ERR_INVALID_ARG and "scales" in str(e.value)
    with pytest.raises(E.CudaLLMError) as e:
        E.kernel_matvec("opt", "bf16", "store", 0, 3, np.zeros((4, 2048), np.uint16), None, x, None, 1e-5, None, 4, 2048)
    assert e.value.code == ERR_INVALID_ARG
    with pytest.raises(E.CudaLLMError) as e:  # w smaller than rows x row bytes
        E.kernel_matvec("opt", "bf16", "store", 0, 0, np.zeros((2, 2048), np.uint16), None, x, None, 1e-5, None, 4, 2048)
    assert e.value.code == ERR_INVALID_ARG
    with pytest.raises(E.CudaLLMError) as e:
        E.kernel_attention("opt", np.zeros(32 * 64), np.zeros((8, 100, 64), np.float16), np.zeros((8, 100, 64), np.float16),
                           10, 32, 8, 64, 100)
    assert e.value.code == ERR_INVALID_ARG and "128" in str(e.value)
    with pytest.raises(E.CudaLLMError) as e:
        E.kernel_rope_kv(1, np.zeros(48 * 64), np.zeros(32), 4096, np.zeros((8, 4096, 64), np.float16),
                         np.zeros((8, 4096, 64), np.float16), 32, 8, 64, 4096)
    assert e.value.code == ERR_INVALID_ARG
    with pytest.raises(E.CudaLLMError) as e:
        E.kernel_argmax(np.zeros(0, np.float32))
    assert e.value.code == ERR_INVALID_ARG


def test_header_struct_offsets():
    raw = _header_bytes()
    assert len(raw) == 256
    assert struct.unpack_from("<Q", raw, 64)[0] == 256


# ---- batched entry points (cudallm_batch_*): host-side checks, no GPU ----

def _batch_create(lib, path, **overrides):
    o = abi.struct("cudallm_batch_options")()
    lib.cudallm_default_batch_options(ctypes.byref(o))
    for k, v in overrides.items():
        setattr(o, k, v)
    h = ctypes.c_void_p()
    rc = lib.cudallm_batch_create(str(path).encode(), ctypes.byref(o), ctypes.byref(h))
    assert h.value is None  # nothing is created on failure
    return rc, lib.cudallm_last_error().decode()


def test_batch_options_layout_and_defaults(native_lib):
    o = abi.struct("cudallm_batch_options")()
    native_lib.cudallm_default_batch_options(ctypes.byref(o))
    assert (o.struct_size, o.n_seq, o.max_seq_len, o.kv_dtype, o.device, o.cuda_graph, o.attn_mode) == (40, 64, 0, 0, -1, 1, 0)
    native_lib.cudallm_default_batch_options(None)  # NULL-safe


def test_batch_create_rejects_before_device_work(native_lib, model_path, tmp_path):
    rc, _ = _batch_create(native_lib, tmp_path / "missing.cudallm")
    assert rc == ERR_IO
    path, _ = model_path("int8")
    rc, msg = _batch_create(native_lib, path)
    assert rc == ERR_INVALID_ARG and "bf16 and int4" in msg
    for bad in ({"n_seq": 0}, {"n_seq": 65}, {"max_seq_len": 100}, {"max_seq_len": 8192}, {"kv_dtype": 2},
                {"struct_size": 36}, {"attn_mode": 3}):
        rc, msg = _batch_create(native_lib, path, **bad)
        assert rc == ERR_INVALID_ARG, (bad, msg)


def test_null_batch_engine_calls(native_lib):
    assert native_lib.cudallm_batch_pos(None, 0) == -1
    native_lib.cudallm_batch_destroy(None)
    assert native_lib.cudallm_batch_reset(None, -1) == ERR_INVALID_ARG
    assert native_lib.cudallm_batch_step(None, None, None, None) == ERR_INVALID_ARG
    assert native_lib.cudallm_batch_synchronize(None) == ERR_INVALID_ARG
    assert native_lib.cudallm_batch_stream(None) is None
    info = abi.struct("cudallm_config_info")()
    assert native_lib.cudallm_batch_get_config(None, ctypes.byref(info)) == ERR_INVALID_ARG
    o = abi.struct("cudallm_batch_options")()
    native_lib.cudallm_default_batch_options(ctypes.byref(o))
    assert native_lib.cudallm_batch_create(None, ctypes.byref(o), None) == ERR_INVALID_ARG
    assert native_lib.cudallm_batch_debug_set(None, b"pdl", 1) == ERR_INVALID_ARG
    v = ctypes.c_longlong(0)
    assert native_lib.cudallm_batch_debug_get(None, b"pdl", ctypes.byref(v)) == ERR_INVALID_ARG


def test_null_engine_knobs(native_lib):
    assert native_lib.cudallm_debug_set(None, b"wait_limit_ns", 1000) == ERR_INVALID_ARG
    assert b"null or destroyed" in native_lib.cudallm_last_error()
    assert native_lib.cudallm_engine_path(None) == -1
    assert native_lib.cudallm_engine_device(None) == -1
    assert native_lib.cudallm_engine_stream(None) is None
