"""GPU: cudallm_attention_noalloc, the split-K decode attention for callers that cannot allocate device
memory (their memory belongs to another runtime's pool, or their loop must stay out of the driver's
allocator). It works on caller-owned device buffers and keeps its partials in a fixed 1.03 MiB device
array, so it is checked here against the allocating entry point cudallm_kernel_attention (same kernels,
host buffers) and against the float64 oracle (oracle.kernels64.attention64), with the attention tolerance
of the kernel tests (rtol = atol = 1e-4), on calls made back to back so that a call which read the previous
call's leftovers in the shared array would show; and once on a stream of its own, read back on that stream.

Named to be collected last: if it fails, a run that stops at the first failure has run everything else.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from cudallm_b200 import engine as E
from oracle import kernels64 as K

pytestmark = pytest.mark.gpu

NH, NKV, HD = 32, 8, 64
TOL = dict(rtol=1e-4, atol=1e-4)


def _case(seed: int, max_seq: int):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(NH * HD).astype(np.float32)
    k = rng.standard_normal((NKV, max_seq, HD)).astype(np.float16)
    v = rng.standard_normal((NKV, max_seq, HD)).astype(np.float16)
    return q, k, v


def _noalloc(lib, q, k, v, ctx: int, max_seq: int, nh: int = NH, nkv: int = NKV,
             own_stream: bool = False) -> tuple[int, np.ndarray]:
    """One call on device buffers the test owns (the test may allocate; the entry point does not). With
    own_stream the call runs on a fresh stream and the output is read back on that stream without a device
    synchronisation in between."""
    dev = torch.device("cuda:0")
    dq = torch.from_numpy(q).to(dev)
    dk = torch.from_numpy(k.view(np.uint16).view(np.int16)).to(dev)
    dv = torch.from_numpy(v.view(np.uint16).view(np.int16)).to(dev)
    dout = torch.full((nh * HD,), float("nan"), dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.Stream(dev) if own_stream else torch.cuda.current_stream(dev)
    rc = lib.cudallm_attention_noalloc(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ctx, dout.data_ptr(), nh, nkv, HD,
                                       max_seq, ctypes.c_void_p(stream.cuda_stream))
    with torch.cuda.stream(stream):
        host = dout.to("cpu", non_blocking=False)
    stream.synchronize()
    return rc, host.numpy()


@pytest.fixture(scope="module")
def lib(native_lib):
    torch.cuda.init()
    return native_lib


def test_two_calls_in_a_row_match_allocating_entry_point(lib):
    # first call: long context; second call: a shorter context with a larger cache, so most partial slots
    # the first call wrote are stale while the second runs; then the first inputs again
    calls = [(1, 4096, 3000), (2, 8192, 129), (1, 4096, 3000)]
    outs = []
    for seed, max_seq, ctx in calls:
        q, k, v = _case(seed, max_seq)
        rc, out = _noalloc(lib, q, k, v, ctx, max_seq)
        assert rc == 0, lib.cudallm_last_error()
        ref = E.kernel_attention("opt", q, k, v, ctx, NH, NKV, HD, max_seq)
        assert np.all(np.isfinite(out))
        assert np.allclose(out, ref, **TOL), (seed, max_seq, ctx)
        assert np.allclose(out, K.attention64(q, k, v, ctx, NH, NKV), **TOL), (seed, max_seq, ctx)
        outs.append(out)
    assert np.allclose(outs[0], outs[2], **TOL)


def test_on_a_stream_of_its_own(lib):
    q, k, v = _case(4, 2048)
    rc, out = _noalloc(lib, q, k, v, 1500, 2048, own_stream=True)
    assert rc == 0, lib.cudallm_last_error()
    assert np.allclose(out, K.attention64(q, k, v, 1500, NH, NKV), **TOL)


def test_full_capacity(lib):
    q, k, v = _case(3, 8192)
    rc, out = _noalloc(lib, q, k, v, 8192, 8192)
    assert rc == 0, lib.cudallm_last_error()
    assert np.allclose(out, E.kernel_attention("opt", q, k, v, 8192, NH, NKV, HD, 8192), **TOL)
    assert np.allclose(out, K.attention64(q, k, v, 8192, NH, NKV), **TOL)


@pytest.mark.parametrize("nh, nkv, max_seq", [(32, 8, 8320), (64, 16, 128)], ids=["max_seq", "heads"])
def test_rejects_sizes_beyond_the_fixed_scratch(lib, nh, nkv, max_seq):
    # validation happens before any device access, so small buffers suffice
    q = np.zeros(nh * HD, dtype=np.float32)
    k = np.zeros((1, 128, HD), dtype=np.float16)
    rc, _ = _noalloc(lib, q, k, k, 1, max_seq, nh=nh, nkv=nkv)
    assert rc == 1  # CUDALLM_ERR_INVALID_ARG
    assert b"8192" in lib.cudallm_last_error()
