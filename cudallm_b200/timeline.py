"""Timeline of one persistent decode step, read from the kernel's own %globaltimer stamps.

    python -m cudallm_b200.timeline [--dtype bf16|int8|int4] [--kv bf16|fp16] [--prompt 32] [--tile-op N]
                                    [--context N]

Runs a seeded prompt through the engine (--context N: N seeded tokens through the chunked prefill, on a
model file with room for 32896 positions), traces the next step (cudallm_debug_trace) and prints:
  * per operation (layers 0, 1, 15 and the lm_head): when the dependency wait begins and ends, when the
    operation ends (median and slowest CTA) and when the copy producer started streaming its weights;
  * per layer, averaged over the 16 layers: the critical duration of each operation (slowest CTA's end
    minus the slowest CTA's wait end) and the median dependency wait;
  * 256 consecutive tiles of CTA 0 starting at weight operation --tile-op (layer*4 + {0 qkv, 1 o-proj,
    2 gate/up, 3 down}, 64 = lm_head): L2 prefetch issued, copy issued, consumer starts waiting, data
    ready, consumer done;
  * for gate/up and down of layer 1, the per-CTA durations (straggler spread) and the slowest SMs.
Times are microseconds from the start of the step. Stamp layout: csrc/engine/decode_step.h.
"""
from __future__ import annotations

import argparse

import numpy as np

LAYERS = 16


def op_names() -> list[str]:
    names = []
    for layer in range(LAYERS):
        names += [f"L{layer}.qkv", f"L{layer}.att", f"L{layer}.wo", f"L{layer}.gu", f"L{layer}.down"]
    return names + ["lm", "end"]


LONG_MAX_SEQ = 32896


def capture(dtype: str, kv: str, prompt: int, tile_op: int | None,
            context: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    from . import synth
    from .engine import Engine
    if context is None:
        path, _ = synth.ensure_model(dtype)
        max_seq = 0  # the file's own
    else:
        path, _ = synth.ensure_model(dtype, seed=0, max_seq_len=LONG_MAX_SEQ)
        max_seq = LONG_MAX_SEQ
    with Engine(path, kv_dtype=kv, max_seq_len=max_seq) as eng:
        if tile_op is not None:
            eng.set_knob("trace_tile_op", tile_op)
        if context is None:
            for t in synth.prompt_ids(prompt):
                eng.step_async(t)
        else:
            eng.prefill(synth.prompt_ids(context, seed=1))
        for _ in range(4):
            eng.step_async(None)
        eng.synchronize()
        eng.trace(True)
        eng.step_async(None)
        tr, tt = eng.read_trace()
    return tr.astype(np.int64), tt.astype(np.int64)


def report(tr: np.ndarray, tt: np.ndarray, tile_op: int) -> None:
    names = op_names()
    t0 = tr[:, 0, 0].min()
    us = lambda a: a / 1e3  # noqa: E731
    print("op        wait_begin  wait_end_max  wait_med  wait_max  end_max  end_med  producer_start_med")
    for k, name in enumerate(names[:-1]):
        if not name.startswith(("L0.", "L1.", "L15.", "lm")):
            continue
        wb, we, oe, pr = (tr[:, k, i] - t0 for i in range(4))
        prod = us(np.median(pr)) if (tr[:, k, 3] > 0).any() and not name.endswith(".att") else float("nan")
        print(f"{name:9s} {us(np.median(wb)):10.1f} {us(we.max()):13.1f} {us(np.median(we - wb)):9.1f} "
              f"{us((we - wb).max()):9.1f} {us(oe.max()):8.1f} {us(np.median(oe)):8.1f} {prod:18.1f}")
    span = us((tr[:, 80, 2] - t0).max())
    waits = us(np.sum([tr[:, k, 1] - tr[:, k, 0] for k in range(81)], axis=0))
    print(f"step span {span:.1f} us; per-CTA total dependency wait: median {np.median(waits):.1f} us, "
          f"max {waits.max():.1f} us")
    print("per layer (mean over 16 layers), us: critical duration / median wait; weight operations also: median "
          "staging (wait end -> vector staged), first tile (staged -> warp 0 done with its first tile), rest")
    for kind in ("qkv", "att", "wo", "gu", "down"):
        ks = [i for i, n in enumerate(names) if n.endswith("." + kind)]
        dur = np.mean([us((tr[:, k, 2] - t0).max() - (tr[:, k, 1] - t0).max()) for k in ks])
        wt = np.mean([us(np.median(tr[:, k, 1] - tr[:, k, 0])) for k in ks])
        line = f"  {kind:5s} {dur:6.2f} / {wt:5.2f}"
        if kind != "att":
            stg = np.mean([us(np.median(tr[:, k, 4] - tr[:, k, 1])) for k in ks])
            first = np.mean([us(np.median(tr[:, k, 5] - tr[:, k, 4])) for k in ks])
            rest = np.mean([us(np.median(tr[:, k, 2] - tr[:, k, 5])) for k in ks])
            line += f"   staging {stg:5.2f}  first tile {first:5.2f}  rest {rest:5.2f}"
        print(line)
    n = int((tt[:, 0] > 0).sum())
    if n:
        tt = tt[:n].astype(np.int64)
        base = tt[0, 0]
        rel = lambda a: np.where(a > 0, (a - base) / 1e3, np.nan)  # noqa: E731
        issue, wstart, ready, done, pref = (rel(tt[:, k]) for k in range(5))
        print(f"{n} tiles of CTA 0 from weight operation {tile_op}: prefetch / issue / wait start / ready / done, us")
        for i in range(min(n, 64)):
            print(f"  {i:3d} {pref[i]:8.2f} {issue[i]:8.2f} {wstart[i]:8.2f} {ready[i]:8.2f} {done[i]:8.2f}   "
                  f"issue->ready {ready[i] - issue[i]:6.2f}  wait {ready[i] - wstart[i]:5.2f}  "
                  f"compute {done[i] - ready[i]:5.2f}")
        print(f"  median issue->ready {np.nanmedian(ready - issue):.2f}, data wait {np.nanmedian(ready - wstart):.2f}, "
              f"compute {np.nanmedian(done - ready):.2f} us")
    sm = tr[:, 81, 3]
    for name in ("L1.gu", "L1.down"):
        k = names.index(name)
        dur = us(tr[:, k, 2] - tr[:, k, 1])
        order = np.argsort(-dur)
        print(f"{name}: per-CTA duration median {np.median(dur):.2f} max {dur.max():.2f} us")
        print("    cta   sm  producer_start  wait_end  staged  first_tile  end   (us from step start)")
        for i in list(order[:6]) + list(order[-6:]):
            st = [us(tr[i, k, j] - t0) for j in (3, 1, 4, 5, 2)]
            print(f"    {int(i):3d} {int(sm[i]):4d} " + "  ".join(f"{v:8.2f}" for v in st))


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--dtype", choices=("bf16", "int8", "int4"), default="bf16")
    ap.add_argument("--kv", choices=("bf16", "fp16"), default="bf16")
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--tile-op", type=int, default=None)
    ap.add_argument("--context", type=int, default=None, help="cached tokens before the traced step (<= 32880)")
    args = ap.parse_args(argv)
    if args.context is not None and not 1 <= args.context <= LONG_MAX_SEQ - 16:
        ap.error(f"--context must be in [1, {LONG_MAX_SEQ - 16}]")
    tr, tt = capture(args.dtype, args.kv, args.prompt, args.tile_op, args.context)
    report(tr, tt, 64 if args.tile_op is None else args.tile_op)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
