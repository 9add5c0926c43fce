"""Live critical-path shares of decode steps, from the diagnostic build.

`python gemma4-webgpu-engine_b200/build_lib.py --trace` builds lib/trace/libgemma4_cuda.so, in
which block 0 of every step kernel stamps %globaltimer right after its programmatic-dependency
wait. Consecutive stamps then measure each launch's share of the live critical path (its own
work after the wait plus the release of the next launch), which a profiler replaying launches
one by one cannot show. Usage, on a GPU:

  python gemma4-webgpu-engine_b200/build_lib.py --trace
  python gemma4-webgpu-engine_b200/trace.py [--batch B] [--ctx-lo L --ctx-hi H] [--steps K]

The product library never contains the stamps (the macro is empty without G4_TRACE).
"""
from __future__ import annotations

import argparse
import collections
import os
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

# Kernel ids written by G4_TRACE_POINT (csrc/*.cu).
_PRO = {0: "x", 1: "norm", 2: "join", 3: "normres", 4: "gelu", 5: "codes"}
_EPI = {0: "y", 1: "gelu-codes", 2: "head"}
_FIXED = {3001: "embed", 3002: "dense (per-layer inputs)", 3003: "per-layer combine",
          3004: "argmax", 3005: "advance", 2256: "attention hd256", 2512: "attention hd512",
          2356: "prefill attention hd256", 2612: "prefill attention hd512",
          5401: "gemm int4 64 tok", 5402: "gemm int4 128 tok", 5801: "gemm int8 64 tok",
          5802: "gemm int8 128 tok", 5411: "gemm int4 64 tok, cluster split",
          5811: "gemm int8 64 tok, cluster split",
          3010: "per-layer tail [prologue]", 3011: "per-layer tail [gate + code exchange]",
          3012: "per-layer tail [projection + release]"}
# Decode attention phases: block 0 of the launch, and the merge from the CTA that runs it
# (column 0, first head group).
for _hd in (256, 512):
    _FIXED.update({2000 + _hd: f"attention hd{_hd} [range, norms]",
                   102000 + _hd: f"attention hd{_hd} [scores, softmax]",
                   202000 + _hd: f"attention hd{_hd} [V wait, PV]",
                   302000 + _hd: f"attention hd{_hd} [partial, count]",
                   402000 + _hd: f"attention hd{_hd} [to the merge]",
                   502000 + _hd: f"attention hd{_hd} [merge]",
                   602000 + _hd: f"attention hd{_hd} [release]"})


# GEMM records (id + offset): block 0's accumulator complete, block 0 done, the last CTA done,
# the latest accumulator-complete time over all CTAs (written by the last CTA).
_GEMM_PHASE = {0: "[block 0 main loop]", 200000: "[block 0 epilogue]", 300000: "[after block 0 done]",
               400000: "[last CTA done -> next]", 500000: "[after the last accumulator]",
               600000: "[after the last CTA start]", 700000: "[after the last dependency wait]"}


def _gemv_name(i: int) -> str:
    bits, pro, epi = (i - 1000) // 100, (i // 10) % 10, i % 10
    return f"gemv int{bits} {_PRO.get(pro, pro)} -> {_EPI.get(epi, epi)}"


def kernel_name(i: int) -> str:
    # GEMV launches stamp three times: after the wait, after the prologue, after the main loop.
    if 1000 <= i < 2000:
        return _gemv_name(i) + " [prologue]"
    if 101000 <= i < 102000:
        return _gemv_name(i - 100000) + " [main loop]"
    if 201000 <= i < 202000:
        return _gemv_name(i - 200000) + " [epilogue + release]"
    if (i % 100000) // 1000 == 5 and i // 100000 in (0, 2, 3, 4, 5, 6, 7) and i % 100000 in _FIXED:
        return _FIXED[i % 100000] + " " + _GEMM_PHASE[i - i % 100000]
    if i in _FIXED:
        return _FIXED[i]
    if 4000 <= i < 4010:
        return f"quantize ({_PRO.get(i - 4000, i)})"
    return str(i)


def summarize(records, steps: int, step_marker: int = 3001):
    """Per-kernel (launches, total us, us per launch) over the last `steps` steps."""
    rec = sorted(records, key=lambda r: r[1])
    starts = [i for i, (k, _) in enumerate(rec) if k == step_marker]
    if len(starts) >= steps:
        rec = rec[starts[-steps]:]
    agg = collections.defaultdict(lambda: [0, 0.0])
    for (k, ta), (_, tb) in zip(rec, rec[1:]):
        d = (tb - ta) / 1000.0
        if d > 5000.0:   # a host gap between steps
            continue
        agg[kernel_name(k)][0] += 1
        agg[kernel_name(k)][1] += d
    return agg


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx-lo", type=int, default=128)
    ap.add_argument("--ctx-hi", type=int, default=128)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--gemm-split-k", type=int, default=0, choices=[0, 1, 2])
    ap.add_argument("--dump", type=int, default=0,
                    help="also print the first N records of the last step in time order")
    args = ap.parse_args()
    import numpy as np
    import __graft_entry__ as entry
    pkg = entry.load_package()
    lib_path = Path(pkg.__file__).resolve().parent / "lib" / "trace" / "libgemma4_cuda.so"
    if not lib_path.exists():
        raise SystemExit(f"{lib_path} missing: run build_lib.py --trace first")
    out = Path(tempfile.mkdtemp()) / "trace.txt"
    os.environ["G4_TRACE_FILE"] = str(out)
    pkg._abi.load(lib_path)
    import torch
    B = args.batch
    rng = np.random.default_rng(0x6E6D6134)
    lens = ([args.ctx_lo] * B if args.ctx_lo == args.ctx_hi
            else [int(v) for v in rng.integers(args.ctx_lo, args.ctx_hi + 1, B)])
    ctx = pkg.engine.Context(device=0, max_seqs=B, max_context=max(lens) + args.steps + 16,
                             max_step_columns=max(B, 512 if max(lens) > 256 else 64),
                             gemm_split_k=args.gemm_split_k)
    ctx.init_random(0x6E6D6134)
    first = [ctx.prefill(b, np.array(pkg.plan.synth_prompt(0x6E6D6134 + b, lens[b]), np.int32), 0, True)
             for b in range(B)]
    ctx.step_stage(np.arange(B), first, lens)
    for _ in range(2):
        ctx.step_run_device(B)
    torch.cuda.synchronize()
    pkg._abi.load().g4_trace_reset()   # keep only the measured steps
    for _ in range(args.steps):
        ctx.step_run_device(B)
    torch.cuda.synchronize()
    ctx.close()   # writes the records
    rec = [tuple(map(int, line.split())) for line in open(out)]
    rec = [r for r in rec if r[0] < 100000000]
    agg = summarize(rec, args.steps)
    tot = sum(v[1] for v in agg.values())
    print(f"B={B}, prompt lengths {args.ctx_lo}..{args.ctx_hi}, last {args.steps} steps: "
          f"{tot / args.steps:.1f} us per step on the critical path")
    print(f"{'kernel':34s} {'launches':>8s} {'us/launch':>10s} {'share':>7s}")
    for k, (n, t) in sorted(agg.items(), key=lambda x: -x[1][1]):
        print(f"{k:34s} {n:8d} {t / n:10.2f} {100 * t / tot:6.1f}%")
    if args.dump:
        # Each record's interval runs to the next record; the last-CTA records of a GEMM carry the
        # latest time over its CTAs, so they sort where that event happened.
        srt = sorted(rec, key=lambda r: r[1])
        starts = [i for i, (k, _) in enumerate(srt) if k == 3001]
        last = srt[starts[-1]:] if starts else srt
        print(f"first {args.dump} records of the last step (us from its start, us to the next record):")
        for (k, ta), (_, tb) in zip(last[:args.dump], last[1:args.dump + 1]):
            print(f"{(ta - last[0][1]) / 1000.0:10.2f} {(tb - ta) / 1000.0:8.2f}  {kernel_name(k)}")


if __name__ == "__main__":
    main()
