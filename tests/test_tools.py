"""The command-line tools cudallm_bench, cudallm_kernelbench and cudallm_bandwidth (cudallm_b200/bin/).

They replace wasiqnauman/cudallm's tools of the same names, so they must accept the flags its bench scripts
pass and write the JSON keys those scripts read:
  * bench/bench_decode.py:33-35 runs `cudallm_bench --model M --prompt-len P --gen G --reps R --matvec X
    --attn Y --fuse F --graph G --json OUT` and reads decode_tok_s_median / achieved_gbps_median (:41);
  * bench/sweep_matvec.py:24 runs `cudallm_kernelbench --op shapes --wtype W --rpb N --json OUT` and reads
    weighted_us (:30);
  * bench/bench_bandwidth.py:10 runs `cudallm_bandwidth --json OUT`; bench/common.py:55-60 reads
    read_gbps_best.
CPU tests check the argument handling (it happens before any CUDA call); GPU tests run those exact command
lines on the seeded model and check the keys and that the numbers are sane.
"""
from __future__ import annotations

import json
import subprocess

import pytest

from cudallm_b200.paths import BIN_DIR

TOOLS = ("cudallm_bench", "cudallm_kernelbench", "cudallm_bandwidth")


def _run(args: list, timeout: int = 600) -> subprocess.CompletedProcess:
    return subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("tool", TOOLS)
def test_tool_built_and_prints_usage(native_lib, tool):
    exe = BIN_DIR / tool
    assert exe.exists(), f"{exe} missing (python -m cudallm_b200.build)"
    res = _run([exe, "--help"])
    assert res.returncode == 0 and "usage:" in res.stdout


@pytest.mark.parametrize("tool, args, needle", [
    ("cudallm_bench", [], "--model is required"),
    ("cudallm_bench", ["--model", "m", "--matvec", "fast"], "opt|naive"),
    ("cudallm_bench", ["--model", "m", "--gen", "0"], "--gen and --reps must be >= 1"),
    ("cudallm_bench", ["--model", "m", "--fuse", "2"], "expects 0 or 1"),
    ("cudallm_kernelbench", ["--op", "conv"], "matvec|shapes|attention"),
    ("cudallm_kernelbench", ["--op", "matvec", "--wtype", "bf16"], "--rows and --cols are required"),
    ("cudallm_kernelbench", ["--op", "shapes", "--rpb", "3"], "--rpb must be"),
    ("cudallm_kernelbench", ["--op", "attention", "--ctx", "9000"], "--ctx must be in"),
    ("cudallm_bandwidth", ["--bogus", "1"], "unknown option"),
])
def test_tool_rejects_bad_arguments(native_lib, tool, args, needle):
    res = _run([BIN_DIR / tool, *args])
    assert res.returncode == 2 and needle in res.stderr, res.stderr


@pytest.mark.gpu
def test_bench_as_bench_decode_runs_it(model_path, tmp_path):
    path, _ = model_path("bf16")
    out = tmp_path / "bench.json"
    res = _run([BIN_DIR / "cudallm_bench", "--model", path, "--prompt-len", 128, "--gen", 64, "--reps", 2, "--matvec",
                "opt", "--attn", "opt", "--fuse", 1, "--graph", 1, "--json", out])
    assert res.returncode == 0, res.stderr
    d = json.loads(out.read_text())
    for k in ("tool", "model", "weight_dtype", "options", "prompt_len", "gen", "reps", "decode_tok_s",
              "decode_tok_s_median", "ms_per_token_median", "weight_bytes", "kv_bytes_per_token_avg", "bytes_per_token",
              "achieved_gbps_median", "gpu_name"):
        assert k in d, k
    assert d["weight_bytes"] == 2471764096
    assert d["kv_bytes_per_token_avg"] == 16 * 2 * 8 * 64 * 2 * (128 + 32)
    assert d["options"]["path"] == "persistent"
    assert 500 < d["decode_tok_s_median"] < 10000 and len(d["decode_tok_s"]) == 2


@pytest.mark.gpu
@pytest.mark.parametrize("fuse, graph", [(0, 0), (1, 1)])
def test_bench_per_op_and_seeded_prompt(model_path, tmp_path, fuse, graph):
    path, _ = model_path("int4")
    out = tmp_path / "bench.json"
    res = _run([BIN_DIR / "cudallm_bench", "--model", path, "--prompt-len", 32, "--gen", 16, "--reps", 1, "--warmup", 0,
                "--fuse", fuse, "--graph", graph, "--path", "per_op", "--kv", "bf16", "--prompt-seed", 0, "--json", out])
    assert res.returncode == 0, res.stderr
    d = json.loads(out.read_text())
    assert d["options"]["path"] == "per_op" and d["weight_dtype"] == "int4" and d["prompt"] == "seed 0"
    assert d["decode_tok_s_median"] > 50


@pytest.mark.gpu
def test_kernelbench_as_sweep_matvec_runs_it(tmp_path):
    out = tmp_path / "kb.json"
    res = _run([BIN_DIR / "cudallm_kernelbench", "--op", "shapes", "--wtype", "int8", "--rpb", 4, "--iters", 20,
                "--json", out])
    assert res.returncode == 0, res.stderr
    d = json.loads(out.read_text())
    assert [r["name"] for r in d["results"]] == ["qkv", "wo", "gate_up", "down", "lm_head"]
    us = [r["median_us"] for r in d["results"]]
    assert d["weighted_us"] == pytest.approx(16 * sum(us[:4]) + us[4])
    assert all(r["gbps"] > 100 for r in d["results"])
    res = _run([BIN_DIR / "cudallm_kernelbench", "--op", "attention", "--impl", "opt", "--ctx", 4000, "--iters", 20])
    assert res.returncode == 0 and "attention opt" in res.stdout, res.stderr


@pytest.mark.gpu
def test_bandwidth_as_bench_bandwidth_runs_it(tmp_path):
    out = tmp_path / "bw.json"
    res = _run([BIN_DIR / "cudallm_bandwidth", "--json", out])
    assert res.returncode == 0, res.stderr
    d = json.loads(out.read_text())
    for k in ("read_gbps_best", "read_gbps_median", "write_gbps_best", "copy_gbps_best", "memcpy_d2d_gbps_best",
              "bulk_read_gbps_best", "bulk_read_l2_gbps_best", "gpu_name"):
        assert k in d, k
    assert 3000 < d["read_gbps_best"] < 9000
    # bulk copies from an L2-resident buffer outrun HBM (the weight ring's refill after a hand-off relies on it)
    assert d["bulk_read_l2_gbps_best"] > d["bulk_read_gbps_best"]
