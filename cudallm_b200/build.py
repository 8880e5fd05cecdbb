"""Builds the native library (lib/libcudallm.so) and the command-line tools (bin/) for sm_100a.

Usage: python -m cudallm_b200.build [--force] [--jobs N]

Every CUDA source is compiled by nvcc for `-gencode arch=compute_100a,code=sm_100a` only; C++ sources
are compiled by nvcc's host compiler with the same include paths. Outputs stay inside the package
directory so they travel with the source tree. A build is skipped when the stamp (hash of every source,
header and flag) matches the previous build.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OBJ = PKG / "_obj"
LIB_DIR = PKG / "lib"
BIN_DIR = PKG / "bin"
LIB_PATH = LIB_DIR / "libcudallm.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O3",
              "-Xptxas", "-warn-spills", *ARCH]
INCLUDES = [f"-I{CSRC}", f"-I{INCLUDE}"]

# The command-line tools (each a main linked with the library's objects); every other source is the library.
TOOLS = {
    "cudallm_bench": "tools/bench_main.cpp",
    "cudallm_kernelbench": "tools/kernelbench_main.cpp",
    "cudallm_bandwidth": "tools/bandwidth_main.cpp",
}


def nvcc() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(p).exists():
        raise RuntimeError("nvcc not found (needs the CUDA 12.9 toolkit)")
    return p


def _lib_sources() -> list[Path]:
    tool_paths = {CSRC / t for t in TOOLS.values()}
    srcs = sorted(p for p in CSRC.rglob("*") if p.suffix in (".cu", ".cpp") and p not in tool_paths)
    return srcs


def _stamp(files: list[Path]) -> str:
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS + INCLUDES).encode())
    for f in sorted(files):
        h.update(str(f.relative_to(ROOT)).encode())
        h.update(f.read_bytes())
    return h.hexdigest()


def _compile(src: Path) -> Path:
    rel = src.relative_to(CSRC)
    out = OBJ / (str(rel).replace("/", "__") + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, *INCLUDES, "-c", str(src), "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip():
        sys.stderr.write(res.stderr)
    return out


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    all_files = [p for p in CSRC.rglob("*") if p.is_file()] + [p for p in INCLUDE.rglob("*.h")]
    stamp = _stamp(all_files)
    stamp_file = OBJ / "stamp"
    tool_bins = [BIN_DIR / name for name, rel in TOOLS.items() if (CSRC / rel).exists()]
    if (not force and stamp_file.exists() and stamp_file.read_text() == stamp and LIB_PATH.exists()
            and all(b.exists() for b in tool_bins)):
        return LIB_PATH
    OBJ.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    BIN_DIR.mkdir(parents=True, exist_ok=True)
    lib_srcs = _lib_sources()
    tool_srcs = [CSRC / t for t in TOOLS.values() if (CSRC / t).exists()]
    jobs = jobs or max(1, min(16, os.cpu_count() or 1))
    with ThreadPoolExecutor(jobs) as ex:
        lib_objs = list(ex.map(_compile, lib_srcs))
        tool_objs = list(ex.map(_compile, tool_srcs))
    link = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB_PATH), *map(str, lib_objs)]
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(link)}\n{res.stdout}\n{res.stderr}")
    for (name, rel), obj in zip([(n, r) for n, r in TOOLS.items() if (CSRC / r).exists()], tool_objs):
        exe = BIN_DIR / name
        cmd = [nvcc(), *ARCH, "-cudart", "static", "-o", str(exe), str(obj), *map(str, lib_objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    stamp_file.write_text(stamp)
    if verbose:
        print(f"built {LIB_PATH}")
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="build libcudallm.so and the tools for sm_100a")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args(argv)
    build(force=args.force, jobs=args.jobs, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
