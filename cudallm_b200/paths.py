"""Filesystem locations used by the package, the tests and bench.py."""
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_ROOT = PKG_DIR.parent
# The native library; CUDALLM_LIB overrides it, the same switch wasiqnauman/cudallm's
# python/cudallm/paths.py:10 uses, so either project's wrapper can drive either library.
LIB_PATH = Path(os.environ.get("CUDALLM_LIB", PKG_DIR / "lib" / "libcudallm.so"))
BIN_DIR = PKG_DIR / "bin"
# Generated synthetic model files (multi-GB) live outside the repository.
MODEL_DIR = Path(os.environ.get("CUDALLM_MODEL_DIR", "/tmp/cudallm_b200_models"))
