"""Kernel timeline of the batched decode step, from CUPTI activity records (torch.profiler).

    python -m cudallm_b200.batch_timeline [--dtype bf16|int4] [--n-seq 64] [--prompt 512] [--steps 4]
                                          [--max-seq 768] [--kv fp16|bf16] [--plain]

Steps a seeded random prompt through a BatchEngine (untimed), then records `--steps` decode steps and
prints, per kernel: launches per step and device time per step; the span of a step; and, for layers 0, 1
and 15, when each of the five operations (QKV, attention, o_proj, gate/up, down) ends, relative to the
step start, with its duration measured end to end from the previous operation's end. With programmatic
dependent launch a kernel starts before its predecessor ends and waits inside, so its own device time
includes that wait; the end-to-end deltas are the figures to read. --plain runs the same steps without
the profiler (a target for ncu).
"""
from __future__ import annotations

import argparse
import collections

import numpy as np

OPS = ["qkv", "attention", "o_proj", "gate_up", "down"]


def run(args) -> None:
    import torch

    from . import synth
    from .engine import BatchEngine

    path, _ = synth.ensure_model(args.dtype, seed=0, max_seq_len=4096)
    rng = np.random.default_rng(0)
    toks = rng.integers(0, 128256, (args.prompt, args.n_seq)).astype(np.int32)
    torch.cuda.init()
    with BatchEngine(path, n_seq=args.n_seq, max_seq_len=args.max_seq, kv_dtype=args.kv) as eng:
        for i in range(args.prompt):
            eng.step_async(toks[i])
        eng.synchronize()
        if args.plain:
            for _ in range(args.steps):
                eng.step_async(None)
            eng.synchronize()
            print("ok")
            return
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(args.steps):
                eng.step_async(None)
            eng.synchronize()
    evs = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA and "Memcpy" not in e.name
           and "Memset" not in e.name]
    evs.sort(key=lambda e: e.time_range.start)
    per_step = len(evs) // args.steps
    agg: dict = collections.defaultdict(lambda: [0, 0.0])
    for e in evs:
        agg[e.name][0] += 1
        agg[e.name][1] += e.time_range.elapsed_us()
    span = (evs[-1].time_range.end - evs[0].time_range.start) / args.steps
    print(f"batched step ({args.dtype} weights): {args.n_seq} sequences, context {args.prompt}..{args.prompt + args.steps}, "
          f"{per_step} launches, span {span:.1f} us per step")
    print("device time per step (includes programmatic-dependent-launch waits):")
    for name, (n, us) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        print(f"  {us / args.steps:9.1f} us  {n // args.steps:3d}x  {name[:100]}")
    last = evs[-per_step:]
    t0 = last[0].time_range.start
    # embedding, then 5 kernels per layer (6 with the split attention), then lm_head and argmax.
    per_layer = (per_step - 3) // 16
    print(f"operation ends (us from the step start) and end-to-end durations, {per_layer} kernels per layer:")
    for layer in (0, 1, 15):
        base = 1 + layer * per_layer
        prev_end = last[base - 1].time_range.end - t0
        row = []
        for k in range(per_layer):
            e = last[base + k]
            end = e.time_range.end - t0
            row.append(f"{e.name.split('(')[0].split('::')[-1][:18]} end {end:7.1f} (+{end - prev_end:5.1f})")
            prev_end = end
        print(f"  L{layer}: " + "; ".join(row))
    lm, am = last[-2], last[-1]
    print(f"  lm_head end {lm.time_range.end - t0:.1f}, argmax end {am.time_range.end - t0:.1f}")


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--dtype", choices=("bf16", "int4"), default="bf16")
    ap.add_argument("--n-seq", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--max-seq", type=int, default=768)
    ap.add_argument("--kv", choices=("fp16", "bf16"), default="fp16")
    ap.add_argument("--plain", action="store_true")
    run(ap.parse_args(argv))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
