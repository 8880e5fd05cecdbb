#!/usr/bin/env python3
"""Benchmark of the decode hot path: batch-1 Llama-3.2-1B decode tok/s and % of the HBM roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--dtype bf16|int8|int4]

Workload (configs[1..2] are reported as extra precisions): seeded synthetic
Llama-3.2-1B weights (cudallm_b200.synth), a 32-token random prompt, greedy decode, bf16 KV cache.
A *step* is one decode token. After W untimed warm-up decode steps, the engine is reset, the prompt is
stepped (untimed), and K decode steps (positions 32 .. 32+K-1) are timed with CUDA events on the
engine's stream, bracketed by a barrier and a device synchronise. With N GPUs (torchrun, one process
per GPU) every rank decodes its own sequence (replicas: the batch-1 path does not shard) and the value
is N*K divided by the slowest rank's time.

Also measured on every rank (unless --quick): batched decode of 64 sequences per GPU
(512-token prompts, then timed greedy decode steps; tensor-core GEMMs) with bf16 and with int4 weights,
reported under "batched" ({"bf16": ..., "int4": ...}) as the whole-job tok/s over all ranks.

On one GPU (unless --quick) the line also carries the configured workloads whatever --steps is:
  * "gen256": the headline precision over the configured 256 decode steps (positions 32..287);
  * "precisions": bf16 / int8 / int4 over the same 256 steps;
  * "sampling": the headline precision over those 256 steps with top-k / top-p sampling fused into the
    step (cudallm_set_sampling with SAMPLING's settings) instead of argmax;
  * "long_context": BASELINE config 4, bf16 weights in a max_seq_len 32896 file: the KV cache is filled by
    the chunked prefill (seeded random tokens, untimed for the decode figures) to 4096 and then 32768 cached
    tokens, and 128 greedy decode steps are timed at each context (bytes per token include the KV read at
    the step's context).

Reported (one JSON line on rank 0): value = tok/s with weights resident; load = wall time of creating the
engine for each precision (reading and uploading the weights); e2e = tok/s through the C ABI
when every step takes its token from the host and returns the next token to the host; roofline of the
persistent decode-step kernel (algorithmic bytes = weight bytes + KV bytes read at the step's context,
the reference's bytes-per-token count, cudallm_bench.cpp:82-87); cpu_baseline = the oracle's restatement
of the reference's CPU model timed on a bounded sample. `--impl reference` times that CPU model alone.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT_LEN = 32
KV_BYTES_PER_TOKEN = 16 * 2 * 8 * 64 * 2  # layers * (K,V) * kv heads * head_dim * 2 bytes


def log(msg: str) -> None:
    print(msg, file=sys.stderr, flush=True)


def dist_info() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def profiled_traffic(dtype: str) -> float | None:
    """DRAM bytes per decode-step launch from the committed ncu summary, if one exists."""
    p = ROOT / "profiles" / "decode_step_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        f = line.split()
        if f and not f[0].startswith("#") and f[0] == dtype:
            return float(f[1])
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        rows = [r for r in csv.reader(io.StringIO(self.out or "")) if len(r) >= 9]
        sm, smax, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = max(smax, float(r[2]))
            except ValueError:
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": smax or None, "reasons": sorted(reasons),
                "samples": len(sm)}


def time_decode(eng, prompt: list[int], steps: int, warmup: int, torch, barrier) -> dict:
    """Device-timed decode steps on the engine's stream (weights resident, no host I/O per step)."""
    stream = torch.cuda.ExternalStream(eng.stream_handle, device=torch.device("cuda", eng.device))
    # Warm-up: a full prompt plus W decode steps, untimed.
    eng.reset()
    for t in prompt:
        eng.step_async(t)
    for _ in range(warmup):
        eng.step_async(None)
    eng.synchronize()
    # Timed: reset, prompt (untimed), then K steps with per-launch events.
    eng.reset()
    for t in prompt:
        eng.step_async(t)
    eng.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier()
    torch.cuda.synchronize(eng.device)
    for i in range(steps):
        starts[i].record(stream)
        eng.step_async(None)
        ends[i].record(stream)
    eng.synchronize()
    torch.cuda.synchronize(eng.device)
    barrier()
    total_ms = starts[0].elapsed_time(ends[-1])
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    return {"total_ms": total_ms, "kernel_ms": per}


def time_e2e(eng, prompt: list[int], steps: int, torch, barrier) -> dict:
    """Same decode, each step through cudallm_step with the token from the host and the next token
    read back to the host (synchronising call)."""
    stream = torch.cuda.ExternalStream(eng.stream_handle, device=torch.device("cuda", eng.device))
    eng.reset()
    nxt = None
    for t in prompt:
        nxt, _ = eng.step(t)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(eng.device)
    t0 = time.perf_counter()
    start.record(stream)
    for _ in range(steps):
        nxt, _ = eng.step(nxt)
    end.record(stream)
    torch.cuda.synchronize(eng.device)
    wall = time.perf_counter() - t0
    barrier()
    return {"total_ms": start.elapsed_time(end), "wall_ms": wall * 1e3}


CONFIG_GEN = 256                           # greedy decode of 256 tokens
SAMPLING = {"temperature": 0.8, "top_k": 40, "top_p": 0.95, "seed": 1}  # the "sampling" figure's settings
LONG_MAX_SEQ, LONG_CTX, LONG_GEN = 32896, (4096, 32768), 128


def time_long_context(args, device: int, torch, peak_gbs: float) -> dict:
    """BASELINE config 4 on the persistent path: one engine (bf16 weights, max_seq_len 32896) steps seeded
    random tokens untimed until `ctx` tokens are cached, then 128 greedy decode steps are timed with per-launch
    CUDA events on the engine's stream; first at 4096 cached tokens, then (continuing the same sequence) at
    32768."""
    from cudallm_b200 import synth
    from cudallm_b200.engine import Engine
    path, _ = synth.ensure_model("bf16", seed=0, max_seq_len=LONG_MAX_SEQ)
    toks = synth.prompt_ids(max(LONG_CTX), seed=0)
    out = {}
    with Engine(path, kv_dtype=args.kv, device=device, max_seq_len=LONG_MAX_SEQ) as eng:
        assert eng.decode_path == "persistent"
        weight_bytes = eng.config["weight_bytes"]
        stream = torch.cuda.ExternalStream(eng.stream_handle, device=torch.device("cuda", device))
        pos = 0
        for ctx in LONG_CTX:
            # The cache is filled by the chunked prefill (64 tokens per batched tensor-core step), untimed for
            # the decode figures; its own rate is reported.
            eng.synchronize()
            t0 = time.perf_counter()
            eng.prefill(toks[pos:ctx])
            fill_s = time.perf_counter() - t0
            n_fill = ctx - pos
            pos = ctx
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(LONG_GEN)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(LONG_GEN)]
            torch.cuda.synchronize(device)
            for i in range(LONG_GEN):
                starts[i].record(stream)
                eng.step_async(None)
                ends[i].record(stream)
            eng.synchronize()
            torch.cuda.synchronize(device)
            pos += LONG_GEN
            total_ms = starts[0].elapsed_time(ends[-1])
            kms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / LONG_GEN
            b = weight_bytes + KV_BYTES_PER_TOKEN * (ctx + (LONG_GEN + 1) / 2)
            out[str(ctx)] = {"tok_s": LONG_GEN / (total_ms * 1e-3), "ms_per_token": total_ms / LONG_GEN,
                             "positions": f"{ctx}..{ctx + LONG_GEN - 1}", "bytes_per_token": int(b),
                             "achieved_gbs": b / (kms * 1e-3) / 1e9, "roofline_frac": b / (kms * 1e-3) / 1e9 / peak_gbs,
                             "fill": {"tokens": n_fill, "seconds": fill_s, "prefill_tok_s": n_fill / fill_s}}
    out["note"] = ("bf16 weights, max_seq_len 32896; cache filled with seeded random tokens by the chunked prefill "
                   "(cudallm_prefill, host-timed, untimed for the decode figures); 128 greedy decode steps timed per "
                   "context with CUDA events")
    return out


BATCH_SEQS, BATCH_PROMPT, BATCH_GEN = 64, 512, 256  # BASELINE config 5, per GPU


def time_batched(args, device: int, torch, barrier, dtype: str = "bf16") -> dict:
    """Batched decode (64 independent sequences on this GPU): every sequence steps a 512-token random
    prompt (untimed), then 256 greedy decode steps are timed with CUDA events on the engine's stream
    (positions 512..767, all 64 sequences per step); then 64 more steps through the C ABI with the tokens
    sent from the host and the next tokens read back each step (e2e)."""
    import numpy as np
    from cudallm_b200 import synth
    from cudallm_b200.engine import BatchEngine
    path, _ = synth.ensure_model(dtype, seed=0, max_seq_len=4096)
    rng = np.random.default_rng([0, device])
    prompts = rng.integers(0, 128256, (BATCH_PROMPT, BATCH_SEQS)).astype(np.int32)
    gen = min(BATCH_GEN, 1024 - BATCH_PROMPT - 64)
    with BatchEngine(path, n_seq=BATCH_SEQS, max_seq_len=1024, kv_dtype=args.kv, device=device) as eng:
        stream = torch.cuda.ExternalStream(eng.stream_handle, device=torch.device("cuda", device))
        for i in range(BATCH_PROMPT):
            eng.step_async(prompts[i])
        eng.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(device)
        start.record(stream)
        for _ in range(gen):
            eng.step_async(None)
        end.record(stream)
        eng.synchronize()
        torch.cuda.synchronize(device)
        barrier()
        ms = start.elapsed_time(end)
        nxt, _ = eng.step(None)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(device)
        e0.record(stream)
        n_e2e = 64
        for _ in range(n_e2e):
            nxt, _ = eng.step(nxt)
        e1.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        e2e_ms = e0.elapsed_time(e1)
        weight_bytes = eng.config["weight_bytes"]
    return {"ms": ms, "steps": gen, "e2e_ms": e2e_ms, "e2e_steps": n_e2e, "weight_bytes": weight_bytes}


def cpu_reference_tokps(path: Path, prompt: list[int], kv: str, n_prompt: int, n_decode: int,
                        time_budget_s: float | None = None) -> dict:
    """The oracle's restatement of the reference CPU model (per-call dequantisation, all host threads)."""
    import torch
    from oracle.refmodel import RefModel
    ref = RefModel(path, kv_dtype=torch.float16 if kv == "fp16" else torch.bfloat16, cache_dense=False)
    logits = None
    for t in prompt[:n_prompt]:
        logits, _ = ref.step(t)
    t0 = time.perf_counter()
    done = 0
    for _ in range(n_decode):
        logits, _ = ref.step(int(torch.argmax(logits)))
        done += 1
        if time_budget_s is not None and time.perf_counter() - t0 > time_budget_s:
            break
    dt = time.perf_counter() - t0
    return {"tok_s": done / dt, "steps": done, "seconds": dt, "threads": torch.get_num_threads()}


def run_reference_arm(args) -> None:
    rank, world, _ = dist_info()
    if rank != 0:
        return
    from cudallm_b200 import synth
    path, _ = synth.ensure_model(args.dtype, seed=0, max_seq_len=4096)
    prompt = synth.prompt_ids(PROMPT_LEN, seed=0)
    import torch
    warm = cpu_reference_tokps(path, prompt, args.kv, n_prompt=4, n_decode=max(1, args.warmup))
    del warm
    r = cpu_reference_tokps(path, prompt, args.kv, n_prompt=8, n_decode=args.steps, time_budget_s=args.ref_budget_s)
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": metric_name(args.dtype), "value": r["tok_s"], "unit": "tok/s",
        "n_gpus": world, "steps": r["steps"], "warmup": args.warmup, "ms_per_step": 1e3 / r["tok_s"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.dtype, "data": "synthetic",
        "config": config_block(args),
        "cpu_baseline": {"value": r["tok_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
                         "sample": f"{r['steps']} greedy decode steps after an 8-token prefix of the prompt, "
                                   f"{args.dtype} weights dequantised per call (reference.py:47-55), torch threads="
                                   f"{r['threads']} of {cores} host cores"},
        "e2e": {"value": r["tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    del torch
    print(json.dumps(line), flush=True)


def max_over_ranks(v: float) -> float:
    """Largest value over all ranks (device tensor under NCCL, host tensor under gloo)."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return v
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    x = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(x, op=dist.ReduceOp.MAX)
    return float(x.item())


def aggregate_tok_s(per_rank_ms: float, steps: int) -> float:
    """Whole-job tok/s: every rank decodes `steps` tokens; the job takes as long as the slowest rank."""
    import torch.distributed as dist
    world = dist.get_world_size() if dist.is_initialized() else 1
    return world * steps / (max_over_ranks(per_rank_ms) * 1e-3)


def metric_name(dtype: str) -> str:
    return f"bs1 decode tok/s ({dtype} weights), Llama-3.2-1B"


def config_block(args) -> dict:
    return {"workload": f"llama3.2-1b batch-1 greedy decode: prompt {PROMPT_LEN}, timed decode steps at positions "
                        f"{PROMPT_LEN}..{PROMPT_LEN + args.steps - 1}, {args.dtype} weights, {args.kv} KV cache",
            "model": "Llama-3.2-1B (seeded synthetic weights, N(0,0.02) bf16, seed 0)",
            "global_batch": 1, "seq_len": PROMPT_LEN + args.steps, "parallelism": f"replicas x{dist_info()[1]}",
            "l2": "inputs larger than L2: every step streams all weights (0.64-2.47 GB > 126 MB L2)",
            "compute": f"{args.dtype} weights, fp32 activations and accumulation"}


def run_ours(args) -> None:
    rank, world, local_rank = dist_info()
    # Native libraries (NCCL prints its version banner at communicator creation) may write to file
    # descriptor 1; until the result line, descriptor 1 points at stderr so stdout carries that line only.
    sys.stdout.flush()
    saved_stdout = os.dup(1)
    os.dup2(2, 1)
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(minutes=10), device_id=torch.device("cuda", local_rank))

    def barrier():
        if world > 1:
            dist.barrier()

    from cudallm_b200 import synth
    from cudallm_b200.engine import Engine
    prompt = synth.prompt_ids(PROMPT_LEN, seed=0)
    dtypes = [args.dtype] + ([d for d in ("int8", "int4") if d != args.dtype] if (world == 1 and not args.quick) else [])
    results = {}
    peaks = measured_peaks()
    for dt in dtypes:
        path, digest = synth.ensure_model(dt, seed=0, max_seq_len=4096)
        barrier()
        t_create = time.perf_counter()
        with Engine(path, kv_dtype=args.kv, device=local_rank) as eng:
            load_s = time.perf_counter() - t_create  # cudallm_create: parse, read and upload every weight
            assert eng.decode_path == "persistent"
            weight_bytes = eng.config["weight_bytes"]
            if dt == args.dtype:
                with ClockSampler(local_rank) as clk:
                    t = time_decode(eng, prompt, args.steps, args.warmup, torch, barrier)
                clocks = clk.summary()
                e = time_e2e(eng, prompt, args.steps, torch, barrier)
            else:
                t, e, clocks = None, None, None
            # The configured workload (256 decode steps) on one GPU, whatever --steps is.
            # (the headline run is reused when it timed exactly that; the other precisions time it here)
            reuse = t is not None and args.steps == CONFIG_GEN
            t256 = (t if reuse else time_decode(eng, prompt, CONFIG_GEN, args.warmup, torch, lambda: None)) \
                if world == 1 else None
            # The same 256 steps with top-k / top-p sampling fused into the step instead of argmax.
            t_sample = None
            if world == 1 and not args.quick and dt == args.dtype:
                eng.set_sampling(SAMPLING["temperature"], SAMPLING["top_k"], SAMPLING["top_p"], SAMPLING["seed"])
                t_sample = time_decode(eng, prompt, CONFIG_GEN, args.warmup, torch, lambda: None)
                eng.set_sampling(0.0)
        results[dt] = {"t": t, "e": e, "clocks": clocks, "weight_bytes": weight_bytes, "t256": t256,
                       "t_sample": t_sample, "load_s": load_s}

    head = results[args.dtype]
    total_ms = max_over_ranks(head["t"]["total_ms"])
    e2e_ms = max_over_ranks(head["e"]["total_ms"])
    kernel_ms = head["t"]["kernel_ms"]
    avg_kernel_ms = sum(kernel_ms) / len(kernel_ms)
    avg_ctx = PROMPT_LEN + (args.steps + 1) / 2
    bytes_per_step = head["weight_bytes"] + KV_BYTES_PER_TOKEN * avg_ctx
    achieved = bytes_per_step / (avg_kernel_ms * 1e-3) / 1e9

    def summarise(t: dict, weight_bytes: int, steps: int) -> dict:
        kms = sum(t["kernel_ms"]) / len(t["kernel_ms"])
        b = weight_bytes + KV_BYTES_PER_TOKEN * (PROMPT_LEN + (steps + 1) / 2)
        return {"tok_s": steps / (t["total_ms"] * 1e-3), "bytes_per_token": int(b),
                "roofline_frac": (b / (kms * 1e-3) / 1e9) / peaks["hbm_gbs"], "achieved_gbs": b / (kms * 1e-3) / 1e9,
                "ms_per_token": t["total_ms"] / steps, "positions": f"{PROMPT_LEN}..{PROMPT_LEN + steps - 1}"}

    extra = {dt: summarise(r["t256"], r["weight_bytes"], CONFIG_GEN) for dt, r in results.items() if r["t256"]}
    gen256 = extra.get(args.dtype)
    ts = results[args.dtype].get("t_sample")
    sampling = None
    if ts:
        sampling = dict(summarise(ts, results[args.dtype]["weight_bytes"], CONFIG_GEN), **SAMPLING)
        if gen256:
            sampling["us_per_token_over_greedy"] = 1e3 * (sampling["ms_per_token"] - gen256["ms_per_token"])
    long_context = time_long_context(args, local_rank, torch, peaks["hbm_gbs"]) if (world == 1 and not args.quick) else None

    batched = {}
    if not args.quick:
        for bdt in ("bf16", "int4"):
            b = time_batched(args, local_rank, torch, barrier, bdt)
            b_ms = max_over_ranks(b["ms"])
            b_e2e_ms = max_over_ranks(b["e2e_ms"])
            avg_ctx_b = BATCH_PROMPT + (b["steps"] + 1) / 2
            b_bytes = b["weight_bytes"] + BATCH_SEQS * KV_BYTES_PER_TOKEN * avg_ctx_b
            b_gbs = b_bytes / (b_ms / b["steps"] * 1e-3) / 1e9
            batched[bdt] = {
                "metric": f"batched decode aggregate tok/s ({bdt} weights)",
                "value": world * BATCH_SEQS * b["steps"] / (b_ms * 1e-3), "unit": "tok/s",
                "per_gpu_tok_s": BATCH_SEQS * b["steps"] / (b_ms * 1e-3), "ms_per_step": b_ms / b["steps"],
                "sequences_per_gpu": BATCH_SEQS, "prompt": BATCH_PROMPT, "timed_decode_steps": b["steps"],
                "kv": args.kv, "bytes_per_step": int(b_bytes), "achieved_gbs": b_gbs,
                "roofline_frac": b_gbs / peaks["hbm_gbs"],
                "e2e": {"value": world * BATCH_SEQS * b["e2e_steps"] / (b_e2e_ms * 1e-3), "unit": "tok/s",
                        "h2d_bytes_per_step": 4 * BATCH_SEQS, "d2h_bytes_per_step": 4 * BATCH_SEQS + 4},
                "scaling": "weak (64 sequences per GPU, no collective)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        path, _ = synth.ensure_model(args.dtype, seed=0, max_seq_len=4096)
        r = cpu_reference_tokps(path, prompt, args.kv, n_prompt=4, n_decode=8, time_budget_s=25.0)
        cpu = {"value": r["tok_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
               "sample": f"{r['steps']} greedy decode steps after a 4-token prefix of the prompt, {args.dtype} "
                         f"weights dequantised per call as reference.py:47-55 does, torch threads={r['threads']}"}

    if world > 1:
        dist.barrier()
    sys.stdout.flush()
    os.dup2(saved_stdout, 1)
    os.close(saved_stdout)
    if rank == 0:
        value = world * args.steps / (total_ms * 1e-3)
        line = {
            "metric": metric_name(args.dtype), "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.dtype, "data": "synthetic", "config": config_block(args),
            "e2e": {"value": world * args.steps / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 16},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": profiled_traffic(args.dtype),
                         "kernel": "decode_step_kernel (one persistent launch per token)",
                         "peak_source": f"{peaks['source']} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                         "algorithmic_bytes_per_launch": int(bytes_per_step)},
            "cpu_baseline": cpu,
            "gpu_launches": args.steps,
            "clocks": head["clocks"],
            "gen256": gen256,
            "sampling": sampling,
            "precisions": extra,
            "long_context": long_context,
            "batched": batched,
            "load": {dt: {"seconds": r["load_s"], "gb_per_s": r["weight_bytes"] / r["load_s"] / 1e9,
                          "note": "cudallm_create wall time: header and table checks, the data region read into two "
                                  "alternating pinned buffers while the other uploads; file in the host page cache"}
                     for dt, r in results.items()},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--dtype", choices=("bf16", "int8", "int4"), default="bf16")
    ap.add_argument("--kv", choices=("fp16", "bf16"), default="bf16")
    ap.add_argument("--quick", action="store_true", help="headline precision only")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-budget-s", type=float, default=120.0)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if PROMPT_LEN + args.steps > 4096:
        raise SystemExit("--steps too large for max_seq_len 4096")
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
