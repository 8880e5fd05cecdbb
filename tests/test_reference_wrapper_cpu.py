"""CPU: the reference's own ctypes wrapper (wasiqnauman/cudallm python/cudallm/engine.py) drives this library
unchanged when CUDALLM_LIB points at it (python/cudallm/paths.py:10).

The wrapper resolves all 15 symbols of the reference ABI eagerly on first use (engine.py:39-66), so a missing
or renamed symbol fails here. The host-side error paths are then checked through the wrapper's own API, with
the reference's error codes: a missing file (IO), a malformed file (FORMAT), bad options and bad kernel-hook
arguments (INVALID_ARG). Nothing here needs a GPU: every case fails before device work.

Runs in a subprocess (the reference package computes its library path at import). Skipped where the reference
checkout is absent (it is never needed by the product or the GPU tests).
"""
from __future__ import annotations

import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

REF_PY = Path(os.environ.get("CUDALLM_REFERENCE_PYTHON", "/root/reference/python"))

SCRIPT = textwrap.dedent(r'''
    import sys, pathlib, struct
    import numpy as np
    from cudallm import engine as W           # the reference's wrapper
    from cudallm.format import write_cudallm  # the reference's writer, for a well-formed header

    lib = W._lib()                            # eager binding of the 15 symbols
    names = ["cudallm_last_error", "cudallm_default_options", "cudallm_create", "cudallm_destroy",
             "cudallm_get_config", "cudallm_reset", "cudallm_pos", "cudallm_step", "cudallm_step_debug",
             "cudallm_kernel_matvec", "cudallm_kernel_rmsnorm", "cudallm_kernel_rope_kv",
             "cudallm_kernel_attention", "cudallm_kernel_silu_mul", "cudallm_kernel_argmax"]
    for n in names:
        assert getattr(lib, n).restype is not None or n in ("cudallm_default_options", "cudallm_destroy"), n
    assert lib.cudallm_pos(None) == -1
    lib.cudallm_destroy(None)
    o = W.CudallmOptions()
    lib.cudallm_default_options(o)
    assert (o.matvec_impl, o.attn_impl, o.fuse, o.cuda_graph, o.max_seq_len, o.matvec_rpb) == (1, 1, 1, 1, 0, 0)

    def code(fn):
        try:
            fn()
        except W.CudaLLMError as e:
            return e.code, str(e)
        return 0, ""

    tmp = pathlib.Path(sys.argv[1])
    c, msg = code(lambda: W.Engine(tmp / "missing.cudallm"))
    assert c == 2, (c, msg)                                 # IO
    bad = tmp / "bad.cudallm"
    bad.write_bytes(b"NOPE" + bytes(252))
    c, msg = code(lambda: W.Engine(bad))
    assert c == 3, (c, msg)                                 # FORMAT
    x = np.zeros(2048, np.float32)
    c, msg = code(lambda: W.kernel_matvec("naive", "int8", "store", 0, 0, np.zeros((4, 2048), np.int8),
                                          np.ones(4, np.float32), x, None, 1e-5, None, 4, 2048))
    assert c == 1 and "naive requires bf16" in msg, (c, msg)   # INVALID_ARG
    c, msg = code(lambda: W.kernel_attention("opt", np.zeros(2048, np.float32), np.zeros((8, 100, 64), np.float16),
                                             np.zeros((8, 100, 64), np.float16), 10, 32, 8, 64, 100))
    assert c == 1, (c, msg)
    c, msg = code(lambda: W.kernel_argmax(np.zeros(0, np.float32)))
    assert c == 1, (c, msg)
    c, msg = code(lambda: W.kernel_rope_kv(1, np.zeros(48 * 64, np.float32), np.zeros(32, np.float32), 4096,
                                           np.zeros((8, 4096, 64), np.float16), np.zeros((8, 4096, 64), np.float16),
                                           32, 8, 64, 4096))
    assert c == 1, (c, msg)
    print("reference wrapper ok")
''')


@pytest.mark.skipif(not (REF_PY / "cudallm" / "engine.py").exists(), reason="reference checkout absent")
def test_reference_wrapper_binds_and_reports_errors(native_lib, tmp_path):
    from cudallm_b200.paths import LIB_PATH
    env = dict(os.environ, CUDALLM_LIB=str(LIB_PATH), PYTHONPATH=str(REF_PY))
    res = subprocess.run([sys.executable, "-c", SCRIPT, str(tmp_path)], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "reference wrapper ok" in res.stdout
