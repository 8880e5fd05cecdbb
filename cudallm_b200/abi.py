"""ctypes view of libcudallm.so generated from its C header.

The structs and function signatures are read from include/cudallm.h when the library is first loaded, so
the header is the only place they are written down: a symbol or field added there is bound here without
a second table to keep in step. Type mapping: `int` / `float` / `(unsigned) long long` scalars map to their
ctypes types, `const char*` to c_char_p, pointers to a header struct to POINTER(struct), `T**` to
POINTER(c_void_p), and every other pointer (buffers, handles, streams) to c_void_p, so callers pass
addresses as integers (numpy `a.ctypes.data`, torch `t.data_ptr()`) or None.

There is no fallback: if the library is missing or lacks a declared symbol, loading raises.
"""
from __future__ import annotations

import ctypes
import functools
import re
from pathlib import Path

from .paths import LIB_PATH, REPO_ROOT

HEADER = REPO_ROOT / "include" / "cudallm.h"

_SCALARS = {"int": ctypes.c_int, "float": ctypes.c_float, "unsigned long long": ctypes.c_ulonglong,
            "long long": ctypes.c_longlong, "unsigned short": ctypes.c_ushort, "unsigned": ctypes.c_uint, "void": None}


class CudaLLMError(RuntimeError):
    """A nonzero return code of the C ABI, with the library's message for it."""

    def __init__(self, code: int, message: str):
        super().__init__(f"cudallm error {code}: {message}")
        self.code = code


def _strip_comments(text: str) -> str:
    """The header without comments and preprocessor lines."""
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    return re.sub(r"^\s*#[^\n]*", " ", text, flags=re.M)


def _parse_structs(text: str) -> dict[str, type]:
    structs: dict[str, type] = {}
    for body, name in re.findall(r"typedef\s+struct\s*\{(.*?)\}\s*(\w+)\s*;", text, flags=re.S):
        fields = []
        for decl in filter(None, (d.strip() for d in body.split(";"))):
            m = re.match(r"((?:unsigned\s+long\s+long)|(?:unsigned\s+short)|\w+)\s+(.*)$", decl, flags=re.S)
            base = _SCALARS[" ".join(m.group(1).split())]
            for item in (i.strip() for i in m.group(2).split(",")):
                arr = re.match(r"(\w+)\s*\[\s*(\d+)\s*\]", item)
                fields.append((arr.group(1), base * int(arr.group(2))) if arr else (item, base))
        structs[name] = type(name, (ctypes.Structure,), {"_fields_": fields})
    return structs


def _ctype(decl: str, structs: dict[str, type]):
    """ctypes type of one C type spelling (parameter name already removed)."""
    t = " ".join(decl.replace("const", " ").split())
    stars = t.count("*")
    base = t.replace("*", "").strip()
    if stars == 0:
        return _SCALARS[base]
    if base == "char" and stars == 1:
        return ctypes.c_char_p
    if stars == 2:
        return ctypes.POINTER(ctypes.c_void_p)
    if base in structs:
        return ctypes.POINTER(structs[base])
    return ctypes.c_void_p


def _param_type(param: str, structs: dict[str, type]):
    param = param.strip()
    if param in ("void", ""):
        return None
    m = re.match(r"(.*?)(\w+)\s*$", param, flags=re.S)  # drop the parameter name
    return _ctype(m.group(1), structs)


def _parse_functions(text: str, structs: dict[str, type]) -> dict[str, tuple[list, object]]:
    funcs = {}
    for ret, name, params in re.findall(r"([\w\s\*]+?)\s*\b(cudallm_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [t for t in (_param_type(p, structs) for p in params.split(",")) if t is not None] \
            if params.strip() != "void" else []
        funcs[name] = (args, _ctype(ret, structs))
    return funcs


@functools.cache
def declarations() -> tuple[dict[str, type], dict[str, tuple[list, object]]]:
    """(structs, functions) as declared in include/cudallm.h."""
    text = _strip_comments(HEADER.read_text())
    structs = _parse_structs(text)
    return structs, _parse_functions(text, structs)


def struct(name: str) -> type:
    return declarations()[0][name]


@functools.cache
def lib() -> ctypes.CDLL:
    """The loaded library, every declared function bound to its header signature."""
    path = Path(LIB_PATH)
    if not path.exists():
        raise CudaLLMError(6, f"native library missing: {path} (build it with `python -m cudallm_b200.build`)")
    handle = ctypes.CDLL(str(path))
    for name, (args, ret) in declarations()[1].items():
        fn = getattr(handle, name)
        fn.argtypes = args
        fn.restype = ret
    return handle


def check(rc: int) -> None:
    """Raises CudaLLMError for a nonzero return code."""
    if rc != 0:
        msg = lib().cudallm_last_error()
        raise CudaLLMError(rc, msg.decode("utf-8", "replace") if msg else "")


def addr(a) -> int | None:
    """Address of a numpy array's data (None stays None)."""
    return None if a is None else a.ctypes.data
