"""Shared fixtures. CPU tests (-m "not gpu") need no GPU; GPU tests (-m gpu) drive libcudallm.so through
its C ABI and compare against the CPU oracle / the golden fixtures made from the reference."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a); run with -m gpu")


@pytest.fixture(scope="session")
def native_lib():
    """The built library; GPU tests fail (not skip) when it is missing: there is no fallback path."""
    from cudallm_b200 import engine as E
    from cudallm_b200.paths import LIB_PATH
    if not LIB_PATH.exists():
        pytest.fail(f"native library missing: {LIB_PATH} (run python -m cudallm_b200.build)")
    return E.lib()


@pytest.fixture(scope="session")
def golden():
    def load(name: str) -> dict:
        path = GOLDEN / f"golden_{name}.npz"
        if not path.exists():
            pytest.fail(f"golden fixture missing: {path} (tests/golden/make_golden.py)")
        with np.load(path, allow_pickle=False) as z:
            return {k: z[k] for k in z.files}
    return load


@pytest.fixture(scope="session")
def model_path():
    """dtype -> path of the seeded synthetic Llama-3.2-1B file (generated on first use, cached)."""
    from cudallm_b200 import synth
    cache: dict = {}

    def get(dtype: str, max_seq_len: int = 4096):
        key = (dtype, max_seq_len)
        if key not in cache:
            cache[key] = synth.ensure_model(dtype, seed=0, max_seq_len=max_seq_len)
        return cache[key]
    return get
