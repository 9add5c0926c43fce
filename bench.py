"""Benchmark: decode tokens/s of the quantized Gemma-4-E2B hot path on B200.

Workload (one replica per GPU): the seeded synthetic Gemma-4-E2B-shaped model,
a 128-token prompt (untimed prefill), then greedy decode steps at batch 1. `value` is tokens/s of
the device-resident decode chain (each step's token stays on the device and feeds the next
step); `e2e` is the same through the public C ABI (g4_decode: host token in, host token out,
copies inside the timed region). `roofline` is the quantized GEMV (BASELINE config 1 shape,
6144 x 1536 int4 x int8) timed live over weight copies larger than L2. `--batch 64` runs the
batched-decode variant (config 4 shape at its contexts).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B]

Under torchrun each rank is an independent replica on its own GPU (weak scaling, no
collectives on the data path); rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SEED = 0x6E6D6134
PROMPT = 128
METRIC = "decode tok/s (B=1, B=64) per B200 & box; quant GEMV HBM GB/s vs peak"

# Algorithmic bytes of one B=1 decode token on the synthetic Gemma-4-E2B shape: int4 linears
# incl. the tied int4 lm_head, the I8 PLE linears, the bf16 per_layer_model_projection, the f16
# row scales, the two gathered embedding rows and the f32 KV rows attention reads.
def token_bytes(ctx_len: int) -> dict:
    H, V, NL, PD = 1536, 262144, 35, 256
    glob = {4, 9, 14, 19, 24, 29, 34}
    w = 0
    scales = 0
    kv = 0
    for L in range(NL):
        hd = 512 if L in glob else 256
        prod = L < 15
        rows = {"q": (8 * hd, H), "o": (H, 8 * hd), "gate": (6144, H), "up": (6144, H), "down": (H, 6144)}
        if prod:
            rows.update({"k": (hd, H), "v": (hd, H)})
        for n, k in rows.values():
            w += n * k // 2
            scales += 2 * n
        w += PD * H + H * PD          # I8 PLE gate / projection
        scales += 2 * (PD + H)
        span = ctx_len if L in glob else min(ctx_len, 512)
        kv += 2 * span * hd * 4
    w += V * H // 2                    # lm_head (tied to the int4 embedding)
    scales += 2 * V
    w += NL * PD * H * 2               # per_layer_model_projection bf16
    gathers = H // 2 + 2 + NL * PD // 2 + 2 * NL
    return {"weights": w, "scales": scales, "kv": kv, "gathers": gathers,
            "total": w + scales + kv + gathers}


GEMV_N, GEMV_K = 6144, 1536
GEMV_BYTES = GEMV_N * GEMV_K // 2 + 2 * GEMV_N + GEMV_K + 2 * GEMV_N  # W + scales + x(int8) + y(f16)
# dram__bytes_read.sum + dram__bytes_write.sum of one config-1 GEMV launch, from the ncu capture
# summarised in profiles/qgemv_stream_config1.md.
GEMV_TRAFFIC = 4_793_856


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock and throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(
                    ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                     "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                self.samples.append([x.strip() for x in out.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self) -> dict:
        sm = [float(s[1]) for s in self.samples if len(s) >= 9 and s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if len(s) >= 9 and s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            if len(s) >= 9:
                for n, v in zip(names, s[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.samples)}


def cpu_baseline(steps: int, n_threads: int) -> dict:
    """The oracle port on the host cores: a bounded sample of the same decode workload."""
    from oracle import oracle as O
    O.build()
    O.threads(n_threads)
    m = O.Model(SEED)
    prompt = O.synth_prompt(SEED, PROMPT)
    s = O.Sequence(m, PROMPT + steps + 8)
    s.forward(prompt[:-1], 0, False, False)
    tok, _, _ = s.forward(prompt[-1:], PROMPT - 1, True, True)
    t0 = time.perf_counter()
    for i in range(steps):
        tok, _, _ = s.forward(np.array([tok], np.int32), PROMPT + i, True, True)
    dt = time.perf_counter() - t0
    m.close()
    return {"value": steps / dt, "unit": "tokens/s", "cores": n_threads, "kind": "port",
            "sample": f"{steps} B=1 decode steps of config 2 after a 128-token prompt (oracle, "
                      f"{n_threads} threads, {dt:.1f} s)"}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args) -> None:
    """--impl reference: the reference's own CPU arithmetic (the oracle port, all host cores)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    n = len(os.sched_getaffinity(0))
    times = []
    steps_per_sample = 2
    from oracle import oracle as O
    O.build()
    O.threads(n)
    m = O.Model(SEED)
    prompt = O.synth_prompt(SEED, PROMPT)
    s = O.Sequence(m, PROMPT + (args.warmup + args.steps) * steps_per_sample + 8)
    s.forward(prompt[:-1], 0, False, False)
    tok, _, _ = s.forward(prompt[-1:], PROMPT - 1, True, True)
    pos = PROMPT
    for it in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        for _ in range(steps_per_sample):
            tok, _, _ = s.forward(np.array([tok], np.int32), pos, True, True)
            pos += 1
        if it >= args.warmup:
            times.append(time.perf_counter() - t0)
    m.close()
    total = args.steps * steps_per_sample
    v = total / sum(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int4xint8/f32",
        "data": "synthetic (seeded random-init Gemma-4-E2B shape)",
        "config": {"workload": "config 2: B=1 greedy decode after a 128-token prompt",
                   "global_batch": 1, "seq_len": PROMPT, "parallelism": "replicas"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": n, "kind": "port",
                         "sample": f"{steps_per_sample} decode steps per step, oracle port "
                                   "(the reference is TypeScript/WGSL and cannot run here)"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def measure_gemv(pkg, torch, copies: int, iters: int) -> dict:
    """the int4 x int8 GEMV [6144 x 1536], timed over `copies` distinct weight
    buffers (together larger than L2) with CUDA events on the launching stream."""
    lib = pkg._abi.load()
    g = torch.Generator(device="cuda").manual_seed(SEED)
    ws = [torch.randint(0, 256, (GEMV_N * GEMV_K // 2,), dtype=torch.uint8, device="cuda", generator=g)
          for _ in range(copies)]
    sc = (torch.rand(GEMV_N, device="cuda", generator=g) * 9e-3 + 1e-3).half().view(torch.int16)
    x = (torch.randint(-127, 128, (GEMV_K,), device="cuda", generator=g).float() * 0.02)
    y = torch.empty(GEMV_N, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def launch(w):
        rc = lib.g4_op_qgemv(w.data_ptr(), sc.data_ptr(), x.data_ptr(), 0.02, 0.0, 4, GEMV_N, GEMV_K, 1,
                             y.data_ptr(), None, sp)
        assert rc == 0, pkg._abi.last_error()

    for w in ws[:8]:
        launch(w)
    torch.cuda.synchronize()
    # One launch per weight copy, recorded into a CUDA graph so the host's per-call cost is not
    # in the timed region; the graph replays `iters / copies` times.
    graph = None
    try:
        side = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            sp = side.cuda_stream
            for w in ws:
                launch(w)
        torch.cuda.synchronize()
    except Exception:  # capture refused: time eager launches instead (host-bound)
        graph = None
        sp = stream.cuda_stream
    reps = max(1, iters // copies)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        if graph is not None:
            graph.replay()
        else:
            for w in ws:
                launch(w)
    e1.record(stream)
    torch.cuda.synchronize()
    per = e0.elapsed_time(e1) / (reps * copies) / 1e3
    del ws
    return {"seconds_per_launch": per, "gbs": GEMV_BYTES / per / 1e9,
            "timing": "cuda graph of launches" if graph is not None else "eager launches"}


def run_gemv_only(pkg, torch, args, world, rank) -> None:
    """Config 1 as its own line: GB/s of the GEMV over 64 distinct weight copies, each launch
    chained to the previous one (programmatic dependent launch inside one CUDA graph)."""
    peaks = load_peaks()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        g = measure_gemv(pkg, torch, copies=64, iters=64 * max(args.steps, 10))
    if world > 1:
        t = torch.tensor([g["seconds_per_launch"]], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        g["seconds_per_launch"] = float(t.item())
        g["gbs"] = GEMV_BYTES / g["seconds_per_launch"] / 1e9
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({
        "metric": "quant GEMV HBM GB/s (config 1, int4 x int8, 6144 x 1536)", "value": world * g["gbs"],
        "unit": "GB/s", "n_gpus": world, "steps": max(args.steps, 10), "warmup": args.warmup,
        "ms_per_step": 64 * g["seconds_per_launch"] * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int4xint8 (int32 acc)", "data": "synthetic (seeded)",
        "config": {"workload": "config 1: 64 distinct 6144x1536 int4 weight copies (302 MB > L2), one graph",
                   "l2": "inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": g["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": g["gbs"] / peaks["hbm_gbs"], "traffic": GEMV_TRAFFIC,
                     "peak_source": peaks["source"], "us_per_launch": g["seconds_per_launch"] * 1e6},
        "gpu_launches": 64 * max(args.steps, 10), "clocks": clocks.summary()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=120)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=24)
    ap.add_argument("--only-gemv", action="store_true",
                    help="BASELINE config 1 alone: the int4 x int8 GEMV [6144 x 1536] line")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("at least 3 warm-up steps")
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import __graft_entry__ as entry
    world, rank, local = dist_env()
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.cuda.current_device()
    pkg = entry.load_package()
    if args.only_gemv:
        run_gemv_only(pkg, torch, args, world, rank)
        return
    engine = pkg.engine
    B = args.batch
    total_steps = args.warmup + args.steps
    max_ctx = PROMPT + total_steps + 8
    ctx = engine.Context(device=dev, max_seqs=B, max_context=max_ctx, max_step_columns=max(B, 64))
    ctx.init_random(SEED)
    prompts = [np.array(pkg.plan.synth_prompt(SEED + b, PROMPT), np.int32) for b in range(B)]
    first = [ctx.prefill(b, prompts[b], 0, True) for b in range(B)]
    torch.cuda.synchronize()

    # ---- device-resident decode chain (value)
    ctx.step_stage(np.arange(B), first, [PROMPT] * B)
    stream = torch.cuda.ExternalStream(ctx.stream())
    for _ in range(args.warmup):
        ctx.step_run_device(B)
    torch.cuda.synchronize()
    launches_per_step = ctx.launches()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            ctx.step_run_device(B)
        e1.record(stream)
        torch.cuda.synchronize()
    dev_s = e0.elapsed_time(e1) / 1e3
    if world > 1:
        t = torch.tensor([dev_s], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dev_s = float(t.item())
    ctx.step_read_tokens(B)

    # ---- end to end through the C ABI: host token in, host token out, every step, over the
    # same positions (the KV rows past the prompt are rewound, src/kv.ts:247-254)
    for b in range(B):
        ctx.kv_truncate(b, PROMPT)
    pos_now = PROMPT
    prev = [int(t) for t in first]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for i in range(args.steps):
        if B == 1:
            prev = [ctx.decode(0, prev[0], pos_now + i)]
        else:
            prev = list(ctx.decode_batch(np.arange(B), prev, [pos_now + i] * B))
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_s = max(e2.elapsed_time(e3) / 1e3, time.perf_counter() - h0)
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_s = float(t.item())

    # ---- roofline of the dominant kernel (quant GEMV, config 1 shape)
    gemv = measure_gemv(pkg, torch, copies=64, iters=640)
    peaks = load_peaks()
    ctx_mid = PROMPT + args.warmup + args.steps // 2
    tb = token_bytes(ctx_mid)
    value = world * B * args.steps / dev_s
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dev_s / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4xint8 (int32 acc) / f32", "data": "synthetic (seeded random-init Gemma-4-E2B shape)",
        "config": {"workload": f"config {'2' if B == 1 else '4-shape'}: B={B} greedy decode after a "
                               f"{PROMPT}-token prompt, contexts {PROMPT}..{PROMPT + total_steps}",
                   "global_batch": world * B, "seq_len": PROMPT, "parallelism": f"replicas x{world}",
                   "l2": "weights (0.93 GB per token) exceed L2 every step"},
        "e2e": {"value": world * B * args.steps / e2e_s, "unit": "tokens/s",
                "h2d_bytes_per_step": 12 * B, "d2h_bytes_per_step": 4 * B},
        "gpu_launches": launches_per_step * args.steps,
        "token_bytes": tb["total"],
        "token_hbm_gbs": tb["total"] * B * args.steps / dev_s / 1e9 if B == 1 else None,
        "roofline": {"bound": "hbm", "kernel": "qgemv-4bit 6144x1536 (config 1)",
                     "achieved": gemv["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gemv["gbs"] / peaks["hbm_gbs"], "traffic": GEMV_TRAFFIC,
                     "peak_source": peaks["source"], "bytes_per_launch": GEMV_BYTES,
                     "us_per_launch": gemv["seconds_per_launch"] * 1e6, "timing": gemv["timing"]},
        "clocks": clocks.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_steps, len(os.sched_getaffinity(0)))
    ctx.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
