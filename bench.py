"""Benchmark: decode tokens/s of the quantized Gemma-4-E2B hot path on B200.

One GPU (the default): `value` is BASELINE config 2 -- the seeded synthetic Gemma-4-E2B-shaped
model, a 128-token prompt (untimed prefill), then K greedy decode steps at batch 1 -- as tokens/s
of the device-resident decode chain (each step's token stays on the device and feeds the next
step); `e2e` is the same through the public C ABI (g4_decode: host token in, host token out,
copies inside the timed region). `roofline` is the quantized GEMV (BASELINE config 1 shape,
6144 x 1536 int4 x int8) timed live over weight copies larger than L2. The same line carries the
other BASELINE configs as keys: `config1_gemv`, `config3_prefill` (2048-token prefill),
`config4_b64` (64 sequences, prompts U[128,4096], 256 greedy steps) and `config5_box` (512
sequences of 512-token prompts, 256 greedy steps, PLE table in 128 MiB slices). `cpu_baseline`
is the oracle port on the host cores (all threads and one thread).

Several GPUs (torchrun): one independent replica per GPU; `value` is config 5 -- the box's 512
sequences split over the replicas (strong scaling) -- over K steps, and `config5_box` the same
over the full 256 steps. The process group (gloo) carries only barriers and the max / sum of the
measured figures.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--quick]
                  [--batch B [--ctx-lo L --ctx-hi H]] [--box] [--workload decode|prefill]
                  [--only-gemv]
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
DTYPE = "int4xint8 (int32 acc) / f32"
DATA = "synthetic (seeded random-init Gemma-4-E2B shape)"
B64, B64_LO, B64_HI, B64_STEPS = 64, 128, 4096, 256
BOX_SEQS, BOX_PROMPT, BOX_STEPS = 512, 512, 256
CTX_KW: dict = {}    # extra g4_config fields from the command line (engine.Context keywords)

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
# dram__bytes_read.sum + dram__bytes_write.sum of one config-1 GEMV launch, from an ncu capture
# of this kernel (int8 codes in) on the config-1 shape (the weights cross DRAM once).
GEMV_TRAFFIC = 4_779_776


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

    def __init__(self, dev: int, active: bool = True):
        self.active = active
        self.gpu = str(dev)
        try:   # the physical GPU behind the device ordinal, whatever CUDA_VISIBLE_DEVICES says
            import torch
            self.gpu = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
        except Exception:
            pass
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
        if self.active:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
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


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def oracle_decode_rate(prompt_len: int, steps: int, n_threads: int, warmup: int = 0) -> tuple:
    """The oracle port decoding one sequence after a `prompt_len`-token prompt (the prefill is
    untimed set-up): (tokens/s, seconds, per-step seconds)."""
    from oracle import oracle as O
    O.build()
    O.threads(n_threads)
    m = O.Model(SEED)
    prompt = O.synth_prompt(SEED, prompt_len)
    s = O.Sequence(m, prompt_len + warmup + steps + 8)
    s.forward(prompt[:-1], 0, False, False)
    tok, _, _ = s.forward(prompt[-1:], prompt_len - 1, True, True)
    pos = prompt_len
    for _ in range(warmup):
        tok, _, _ = s.forward(np.array([tok], np.int32), pos, True, True)
        pos += 1
    per = []
    for _ in range(steps):
        t0 = time.perf_counter()
        tok, _, _ = s.forward(np.array([tok], np.int32), pos, True, True)
        per.append(time.perf_counter() - t0)
        pos += 1
    m.close()
    return steps / sum(per), sum(per), per


def cpu_baseline(prompt_len: int, steps: int, n_threads: int, workload: str) -> dict:
    """The oracle port on the host cores: a bounded sample of the same decode workload, on all
    threads and on one thread."""
    v, dt, _ = oracle_decode_rate(prompt_len, steps, n_threads)
    v1, dt1, _ = oracle_decode_rate(prompt_len, 3, 1)
    return {"value": v, "unit": "tokens/s", "cores": n_threads, "kind": "port",
            "cpu_model": cpu_model(),
            "single_thread": {"value": v1, "unit": "tokens/s", "cores": 1, "steps": 3,
                              "seconds": dt1},
            "sample": f"{steps} B=1 decode steps after a {prompt_len}-token prompt ({workload}; "
                      f"oracle, {n_threads} threads, {dt:.1f} s; a batch of sequences costs the "
                      f"CPU the same per token)"}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


L2_NOTE = "weights (0.93 GB per step) exceed L2 every step"


def line_config(world: int) -> dict:
    """The `config` of the bench line; both arms print the same one for the same N. One GPU:
    BASELINE config 2. Several (torchrun): config 5, the box's 512 sequences over the replicas."""
    if world == 1:
        return {"workload": f"config 2: B=1 greedy decode after a {PROMPT}-token prompt",
                "global_batch": 1, "seq_len": PROMPT, "parallelism": "replicas x1", "l2": L2_NOTE}
    return {"workload": f"config 5: {BOX_SEQS} sequences over {world} replicas, {BOX_PROMPT}-token "
                        "prompts, greedy decode, PLE table in 128 MiB slices",
            "global_batch": BOX_SEQS, "seq_len": BOX_PROMPT, "parallelism": f"replicas x{world}",
            "l2": L2_NOTE}


def run_reference(args) -> None:
    """--impl reference: the reference's own CPU arithmetic (the oracle port; the reference is
    TypeScript/WGSL and cannot run here) on all host cores, on the repo arm's config. Each step
    is a bounded sample of two decode steps of one sequence at the workload's prompt length;
    rank 0 alone runs under torchrun."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    n = len(os.sched_getaffinity(0))
    prompt_len = PROMPT if world == 1 else BOX_PROMPT
    per_sample = 2
    v, total_s, per = oracle_decode_rate(prompt_len, args.steps * per_sample, n,
                                         warmup=args.warmup * per_sample)
    v1, dt1, _ = oracle_decode_rate(prompt_len, 2, 1)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total_s / args.steps,
        "higher_is_better": True, "scaling": "weak" if world == 1 else "strong",
        "vs_baseline": None, "dtype": DTYPE, "data": DATA, "config": line_config(world),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": n, "kind": "port",
                         "cpu_model": cpu_model(),
                         "single_thread": {"value": v1, "unit": "tokens/s", "cores": 1,
                                           "steps": 2, "seconds": dt1},
                         "sample": f"{per_sample} B=1 decode steps per step after a {prompt_len}-token "
                                   "prompt, oracle port on all host threads (the reference is "
                                   "TypeScript/WGSL and cannot run here; a batch costs the CPU the "
                                   "same per token)"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def gemv_shape(bits: int) -> tuple:
    """(N, K, algorithmic bytes per launch) of the GEMV line: BASELINE config 1 at 4 bits; at 2
    bits the checkpoint's consumer gate / up projection [12288 x 1536] on the interleaved tile
    layout (the same 4.7 MB of weights)."""
    n, k = (GEMV_N, GEMV_K) if bits == 4 else (2 * GEMV_N, GEMV_K)
    return n, k, n * k * bits // 8 + 2 * n + k + 2 * n


def measure_gemv(pkg, torch, copies: int, iters: int, bits: int = 4, codes_input: bool = True) -> dict:
    """the int4 x int8 GEMV [6144 x 1536] (or the 2-bit line, gemv_shape),
    timed over `copies` distinct weight buffers (together larger than L2) with CUDA events on the
    launching stream. The activations are the config's int8 codes (scale 0.02) fed to
    g4_op_qgemv_codes, or (codes_input False) the same values as f32 through g4_op_qgemv, whose
    prologue snaps them."""
    lib = pkg._abi.load()
    n, k, nbytes = gemv_shape(bits)
    g = torch.Generator(device="cuda").manual_seed(SEED)
    ws = [torch.randint(0, 256, (n * k * bits // 8,), dtype=torch.uint8, device="cuda", generator=g)
          for _ in range(copies)]
    sc = (torch.rand(n, device="cuda", generator=g) * 9e-3 + 1e-3).half().view(torch.int16)
    codes = torch.randint(-127, 128, (k,), device="cuda", generator=g).to(torch.int8)
    x = codes.float() * 0.02
    y = torch.empty(n, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    fn = lib.g4_op_qgemv_codes if codes_input else lib.g4_op_qgemv
    src = codes if codes_input else x

    def launch(w):
        rc = fn(w.data_ptr(), sc.data_ptr(), src.data_ptr(), 0.02, 0.0, bits, n, k, 1, y.data_ptr(), None, sp)
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
    return {"seconds_per_launch": per, "gbs": nbytes / per / 1e9, "bytes_per_launch": nbytes,
            "timing": "cuda graph of launches" if graph is not None else "eager launches"}


def reduce_max(torch, vals, world):
    """Elementwise max over ranks of a few host floats (gloo: CPU tensors)."""
    if world == 1:
        return list(vals)
    t = torch.tensor(list(vals), dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(v) for v in t]


def reduce_sum(torch, vals, world):
    if world == 1:
        return list(vals)
    t = torch.tensor(list(vals), dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
    return [float(v) for v in t]


def barrier(torch, world):
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def run_gemv_only(pkg, torch, args, world, rank) -> None:
    """Config 1 as its own line: GB/s of the GEMV over 64 distinct weight copies, each launch
    chained to the previous one (programmatic dependent launch inside one CUDA graph)."""
    peaks = load_peaks()
    bits = args.gemv_bits
    n, k, nbytes = gemv_shape(bits)
    barrier(torch, world)
    with ClockSampler(torch.cuda.current_device(), rank == 0) as clocks:
        g = measure_gemv(pkg, torch, copies=64, iters=64 * max(args.steps, 10), bits=bits,
                         codes_input=args.gemv_input == "codes")
    g["seconds_per_launch"] = reduce_max(torch, [g["seconds_per_launch"]], world)[0]
    g["gbs"] = nbytes / g["seconds_per_launch"] / 1e9
    if rank != 0:
        return
    what = ("config 1, int4 x int8, 6144 x 1536" if bits == 4 else
            "2-bit tile layout x int8, 12288 x 1536 (checkpoint consumer gate / up)")
    print(json.dumps({
        "metric": f"quant GEMV HBM GB/s ({what})", "value": world * g["gbs"],
        "unit": "GB/s", "n_gpus": world, "steps": max(args.steps, 10), "warmup": args.warmup,
        "ms_per_step": 64 * g["seconds_per_launch"] * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": f"int{bits}xint8 (int32 acc)", "data": "synthetic (seeded)",
        "config": {"workload": f"64 distinct {n}x{k} {bits}-bit weight copies ({64 * nbytes / 1e6:.0f} MB > L2), "
                               "one graph", "l2": "inputs larger than L2",
                   "input": "int8 activation codes (g4_op_qgemv_codes)" if args.gemv_input == "codes"
                            else "f32 activations snapped in the prologue (g4_op_qgemv)"},
        "roofline": {"bound": "hbm", "achieved": g["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": g["gbs"] / peaks["hbm_gbs"], "traffic": GEMV_TRAFFIC if bits == 4 else None,
                     "bytes_per_launch": nbytes,
                     "peak_source": peaks["source"], "us_per_launch": g["seconds_per_launch"] * 1e6},
        "gpu_launches": 64 * max(args.steps, 10), "clocks": clocks.summary()}), flush=True)


PREFILL_LAYERS = 15


def prefill_ops(n: int) -> int:
    """Algorithmic int8 ops of an n-token prefill with the KV-sharing exit: 2 x producer-layer
    linear parameters x (n - 1) columns, plus the last position through all layers and the head."""
    H, PD, V = 1536, 256, 262144
    prod_params = mlp = 0
    for L in range(35):
        hd = 512 if L in {4, 9, 14, 19, 24, 29, 34} else 256
        p = 8 * hd * H + H * 8 * hd + 3 * 6144 * H + 2 * PD * H + (2 * hd * H if L < 15 else 0)
        mlp += p
        if L < PREFILL_LAYERS:
            prod_params += p
    return 2 * prod_params * (n - 1) + 2 * (mlp + V * H)


def measure_prefill(pkg, torch, dev, n, steps, warmup, world, rank) -> dict:
    """prefill of n random ids with the KV-sharing exit (positions 0..n-2 run
    the producer layers only, the last position all layers and the head), one chunk: the
    projections run as tcgen05 int8 GEMMs over all n-1 columns. Each step rewinds the KV
    (src/kv.ts:247-254) and prefills again; the ids go host->device and the token comes back
    inside every step, so the device-timed and the end-to-end figures share one loop shape."""
    ctx = pkg.engine.Context(device=dev, max_seqs=1, max_context=n + 8, max_step_columns=n, **CTX_KW)
    ctx.init_random(SEED)
    prompt = np.array(pkg.plan.synth_prompt(SEED + 7919 * rank, n), np.int32)
    stream = torch.cuda.ExternalStream(ctx.stream())
    for _ in range(warmup):
        ctx.kv_truncate(0, 0)
        ctx.prefill(0, prompt, 0, True)
    torch.cuda.synchronize()
    launches = ctx.launches()
    barrier(torch, world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev, rank == 0) as clocks:
        torch.cuda.nvtx.range_push("timed")   # lets a profiler keep only these launches
        e0.record(stream)
        for _ in range(steps):
            ctx.kv_truncate(0, 0)
            ctx.prefill(0, prompt, 0, True)
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    # End to end (host ids in, host token out) on its own clock, without the sampler's
    # nvidia-smi processes starting inside the timed region.
    barrier(torch, world)
    h0 = time.perf_counter()
    for _ in range(steps):
        ctx.kv_truncate(0, 0)
        ctx.prefill(0, prompt, 0, True)
    torch.cuda.synchronize()
    wall = time.perf_counter() - h0
    dev_s, wall = reduce_max(torch, [max(e0.elapsed_time(e1) / 1e3, 1e-9), wall], world)
    ctx.close()
    ops = prefill_ops(n)
    peaks = load_peaks()
    int8_peak = 2 * peaks.get("bf16_tflops", 1590.0)
    achieved = ops * steps / dev_s / 1e12
    return {"value": world * n * steps / dev_s, "unit": "tokens/s", "steps": steps,
            "ms_per_step": 1000 * dev_s / steps, "launches_per_step": launches,
            "e2e": {"value": world * n * steps / wall, "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * n, "d2h_bytes_per_step": 4},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOP/s",
                         "frac": achieved / int8_peak, "traffic": None,
                         "peak_source": "2 x measured dense bf16 (int8 tensor rate)",
                         "ops_per_step": ops,
                         "kernel": "whole prefill (int8 GEMMs + attention + rest)"},
            "clocks": clocks.summary()}


def run_prefill(pkg, torch, args, world, rank, dev) -> None:
    """Config 3 as its own line (one prefill per 20 --steps, at least one)."""
    r = measure_prefill(pkg, torch, dev, args.tokens, max(1, args.steps // 20), args.warmup, world, rank)
    if rank != 0:
        return
    n = args.tokens
    print(json.dumps({
        "metric": "prefill tokens/s (config 3, 2048-token prompt, KV-sharing exit)",
        "value": r["value"], "unit": "tokens/s", "n_gpus": world, "steps": r["steps"],
        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": DTYPE, "data": DATA,
        "config": {"workload": f"config 3: prefill of {n} random ids, producer layers for 0..{n - 2}, "
                               "all layers + head for the last", "global_batch": world,
                   "seq_len": n, "parallelism": f"replicas x{world}", "l2": "weights exceed L2"},
        "e2e": r["e2e"], "gpu_launches": r["launches_per_step"] * r["steps"],
        "roofline": r["roofline"], "clocks": r["clocks"]}), flush=True)


def measure_decode(pkg, torch, dev, seq_ids, lens, steps, warmup, world, rank, slice_bytes=0,
                   gemm_split_k=0) -> dict:
    """Greedy decode of the sequences `seq_ids` (prompt b: `lens[i]` seeded ids from seed
    SEED + b) on one replica: every prompt is prefilled (untimed), `warmup` steps run and are
    rewound, then exactly `steps` steps from the prompts are timed twice:
      * device chain: one CUDA graph per step, each step's token and position stay on the device
        and feed the next (CUDA events on the context's stream);
      * end to end through the C ABI (g4_decode / g4_decode_batch): host tokens in, host tokens
        out every step, the copies inside the timed region (the KV rows past the prompts rewound
        first, src/kv.ts:247-254).
    Returns the slowest rank's times."""
    B = len(seq_ids)
    max_ctx = max(lens) + max(steps, warmup) + 8
    chunk = max(B, 512 if max(lens) > 256 else 64)
    ctx = pkg.engine.Context(device=dev, max_seqs=B, max_context=max_ctx, max_step_columns=chunk,
                             ple_slice_bytes=slice_bytes, gemm_split_k=gemm_split_k, **CTX_KW)
    ctx.init_random(SEED)
    prompts = [np.array(pkg.plan.synth_prompt(SEED + int(s), lens[i]), np.int32)
               for i, s in enumerate(seq_ids)]
    torch.cuda.synchronize()
    p0 = time.perf_counter()
    first = [ctx.prefill(b, prompts[b], 0, True) for b in range(B)]
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - p0
    stream = torch.cuda.ExternalStream(ctx.stream())

    ctx.step_stage(np.arange(B), first, lens)
    for _ in range(warmup):
        ctx.step_run_device(B)
    torch.cuda.synchronize()
    launches = ctx.launches()
    for b in range(B):
        ctx.kv_truncate(b, lens[b])
    ctx.step_stage(np.arange(B), first, lens)
    barrier(torch, world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev, rank == 0) as clocks:
        torch.cuda.nvtx.range_push("timed")    # lets a profiler keep only these launches
        e0.record(stream)
        for _ in range(steps):
            ctx.step_run_device(B)
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    dev_s = e0.elapsed_time(e1) / 1e3
    dev_tokens = ctx.step_read_tokens(B)

    # The C-ABI path launches its own graph (host-staged tokens): warm it as well, so the timed
    # region holds no graph capture.
    for b in range(B):
        ctx.kv_truncate(b, lens[b])
    prev = [int(t) for t in first]
    for i in range(warmup):
        if B == 1:
            prev = [ctx.decode(0, prev[0], lens[0] + i)]
        else:
            prev = list(ctx.decode_batch(np.arange(B), prev, [lens[b] + i for b in range(B)]))
    torch.cuda.synchronize()
    for b in range(B):
        ctx.kv_truncate(b, lens[b])
    prev = [int(t) for t in first]
    barrier(torch, world)
    h0 = time.perf_counter()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for i in range(steps):
        if B == 1:
            prev = [ctx.decode(0, prev[0], lens[0] + i)]
        else:
            prev = list(ctx.decode_batch(np.arange(B), prev, [lens[b] + i for b in range(B)]))
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_s = max(e2.elapsed_time(e3) / 1e3, time.perf_counter() - h0)
    ctx.close()
    if [int(t) for t in dev_tokens] != [int(t) for t in prev]:
        raise RuntimeError("the device chain and the C-ABI decode disagree on the last tokens")
    # Algorithmic bytes of the timed steps: weights and scales once per step, each sequence's
    # KV rows at its own position.
    tb = token_bytes(lens[0])
    kv = sum(token_bytes(lens[b] + i)["kv"] for b in range(B) for i in range(0, steps, max(1, steps // 16)))
    kv *= steps / len(range(0, steps, max(1, steps // 16)))
    step_bytes = tb["weights"] + tb["scales"] + kv / steps
    dev_s, e2e_s = reduce_max(torch, [dev_s, e2e_s], world)
    total_bytes, total_seqs = reduce_sum(torch, [step_bytes * steps, B], world)
    return {"dev_s": dev_s, "e2e_s": e2e_s, "launches_per_step": launches, "step_bytes": step_bytes,
            "all_ranks_bytes": total_bytes, "seqs": int(total_seqs), "prefill_s": prefill_s,
            "prefill_tokens": sum(lens), "clocks": clocks.summary()}


def decode_summary(r: dict, steps: int, world: int, peaks: dict, h2d_per_seq=12, d2h_per_seq=4) -> dict:
    """Throughput keys of one decode workload: tokens of all ranks over the slowest rank's time;
    the HBM fraction is the algorithmic bytes all ranks moved over (N x measured peak)."""
    gbs = r["all_ranks_bytes"] / r["dev_s"] / 1e9
    return {"value": r["seqs"] * steps / r["dev_s"], "unit": "tokens/s", "steps": steps,
            "ms_per_step": 1000 * r["dev_s"] / steps,
            "e2e": {"value": r["seqs"] * steps / r["e2e_s"], "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d_per_seq * r["seqs"], "d2h_bytes_per_step": d2h_per_seq * r["seqs"]},
            "step_bytes_per_replica": r["step_bytes"], "hbm_gbs_all_replicas": gbs,
            "hbm_frac": gbs / (world * peaks["hbm_gbs"]),
            "prefill_tokens_per_s": r["prefill_tokens"] / r["prefill_s"],
            "gpu_launches_per_step": r["launches_per_step"], "clocks": r["clocks"]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=24)
    ap.add_argument("--quick", action="store_true",
                    help="one GPU: the config 2 line alone (no config 1/3/4/5 keys)")
    ap.add_argument("--only-gemv", action="store_true",
                    help="BASELINE config 1 alone: the int4 x int8 GEMV [6144 x 1536] line")
    ap.add_argument("--gemv-bits", type=int, default=4, choices=[2, 4],
                    help="with --only-gemv: 2 times the checkpoint's 2-bit consumer gate / up instead")
    ap.add_argument("--gemv-input", default="codes", choices=["codes", "f32"],
                    help="with --only-gemv: int8 activation codes (config 1) or f32 activations")
    ap.add_argument("--batch", type=int, default=0,
                    help="a decode line of this many sequences instead of the default workloads")
    ap.add_argument("--ctx-lo", type=int, default=PROMPT,
                    help="with --batch: prompt lengths uniform in [ctx-lo, ctx-hi] (seeded)")
    ap.add_argument("--ctx-hi", type=int, default=PROMPT)
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill"])
    ap.add_argument("--box", action="store_true",
                    help="config 5 as the line on any number of GPUs (the default under torchrun)")
    ap.add_argument("--tokens", type=int, default=2048, help="prefill workload: prompt length")
    ap.add_argument("--gemm-split-k", type=int, default=0, choices=[0, 1, 2],
                    help="g4_config.gemm_split_k: 0 cluster, 1 none, 2 workspace")
    ap.add_argument("--gemm-shadow-min-columns", type=int, default=0,
                    help="g4_config.gemm_shadow_min_columns: 0 default (every tensor-core step), negative off")
    args = ap.parse_args()
    CTX_KW["gemm_shadow_min_columns"] = args.gemm_shadow_min_columns
    if args.warmup < 3:
        ap.error("at least 3 warm-up steps")
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import __graft_entry__ as entry
    world, rank, local = dist_env()
    pkg = entry.load_package()
    # Replicas share nothing on the data path: the group (gloo, host memory) carries only the
    # barriers before timing and the max / sum of the measured figures.
    torch.cuda.set_device(local if world > 1 else 0)
    if world > 1:
        pkg.replicas.init_group(torch, "gloo", 300.0)
    dev = torch.cuda.current_device()
    try:
        if args.only_gemv:
            run_gemv_only(pkg, torch, args, world, rank)
        elif args.workload == "prefill":
            run_prefill(pkg, torch, args, world, rank, dev)
        else:
            run_decode(pkg, torch, args, world, rank, dev)
    finally:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


def run_decode(pkg, torch, args, world, rank, dev) -> None:
    peaks = load_peaks()
    box = args.box or world > 1
    if box:
        lo, hi = pkg.replicas.replica_slice(BOX_SEQS, world, rank)
        seq_ids = list(range(lo, hi))
        lens = [BOX_PROMPT] * len(seq_ids)
        slice_bytes = 128 << 20
    elif args.batch:
        seq_ids = list(range(args.batch))
        rng = np.random.default_rng(SEED + 1000 * rank)
        lens = ([args.ctx_lo] * args.batch if args.ctx_lo == args.ctx_hi
                else [int(v) for v in rng.integers(args.ctx_lo, args.ctx_hi + 1, args.batch)])
        slice_bytes = 0
    else:
        seq_ids, lens, slice_bytes = [0], [PROMPT], 0
    r = measure_decode(pkg, torch, dev, seq_ids, lens, args.steps, args.warmup, world, rank,
                       slice_bytes, args.gemm_split_k)
    main_s = decode_summary(r, args.steps, world, peaks)
    if box:
        config = line_config(world) if world > 1 else dict(line_config(2), parallelism="replicas x1")
        scaling = "strong"
    elif args.batch:
        config = {"workload": f"B={args.batch} greedy decode, prompt lengths "
                              f"{'U[%d,%d]' % (args.ctx_lo, args.ctx_hi) if args.ctx_lo != args.ctx_hi else args.ctx_lo} (seeded)",
                  "global_batch": world * args.batch, "seq_len": max(lens),
                  "parallelism": f"replicas x{world}", "l2": L2_NOTE}
        scaling = "weak"
    else:
        config = line_config(1)
        scaling = "weak"
    gemv = measure_gemv(pkg, torch, copies=64, iters=640)
    gemv_f32 = measure_gemv(pkg, torch, copies=64, iters=640, codes_input=False)
    gemv_s, gemv_f32_s = reduce_max(torch, [gemv["seconds_per_launch"], gemv_f32["seconds_per_launch"]], world)
    gemv_gbs = GEMV_BYTES / gemv_s / 1e9
    line = {
        "metric": METRIC, "value": main_s["value"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": main_s["ms_per_step"],
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": DTYPE,
        "data": DATA, "config": config, "e2e": main_s["e2e"],
        "gpu_launches": r["launches_per_step"] * args.steps,
        "step_bytes": r["step_bytes"], "step_hbm_gbs": main_s["hbm_gbs_all_replicas"] / world,
        "step_hbm_frac": main_s["hbm_frac"], "prefill_tokens_per_s": main_s["prefill_tokens_per_s"],
        "roofline": {"bound": "hbm", "kernel": "qgemv-4bit 6144x1536 (config 1)",
                     "achieved": gemv_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gemv_gbs / peaks["hbm_gbs"], "traffic": GEMV_TRAFFIC,
                     "peak_source": peaks["source"], "bytes_per_launch": GEMV_BYTES,
                     "us_per_launch": gemv_s * 1e6, "timing": gemv["timing"],
                     "input": "int8 activation codes (config 1), g4_op_qgemv_codes",
                     "f32_input": {"achieved": GEMV_BYTES / gemv_f32_s / 1e9, "us_per_launch": gemv_f32_s * 1e6,
                                   "via": "g4_op_qgemv (f32 x snapped in the prologue)"}},
        "clocks": main_s["clocks"],
    }
    if box:
        # The same box workload over the BASELINE's full 256 greedy steps.
        rb = measure_decode(pkg, torch, dev, seq_ids, lens, BOX_STEPS, args.warmup, world, rank, slice_bytes)
        line["config5_box"] = dict(decode_summary(rb, BOX_STEPS, world, peaks), replicas=world,
                                   sequences=BOX_SEQS)
    elif not args.batch and not args.quick:
        # One GPU, default run: BASELINE configs 1, 3, 4 and 5 as extra keys beside config 2.
        line["config1_gemv"] = {"value": gemv_gbs, "unit": "GB/s", "frac": gemv_gbs / peaks["hbm_gbs"],
                                "us_per_launch": gemv_s * 1e6,
                                "workload": "64 distinct 6144x1536 int4 weight copies, one graph, int8 activation codes",
                                "f32_input_gbs": GEMV_BYTES / gemv_f32_s / 1e9}
        rng = np.random.default_rng(SEED)
        b64_lens = [int(v) for v in rng.integers(B64_LO, B64_HI + 1, B64)]
        r4 = measure_decode(pkg, torch, dev, list(range(B64)), b64_lens, B64_STEPS, args.warmup, world, rank)
        line["config4_b64"] = dict(decode_summary(r4, B64_STEPS, world, peaks),
                                   contexts=f"U[{B64_LO},{B64_HI}] seeded, mean {np.mean(b64_lens):.0f}")
        r5 = measure_decode(pkg, torch, dev, list(range(BOX_SEQS)), [BOX_PROMPT] * BOX_SEQS, BOX_STEPS,
                            args.warmup, world, rank, 128 << 20)
        line["config5_box"] = dict(decode_summary(r5, BOX_STEPS, world, peaks), replicas=1,
                                   sequences=BOX_SEQS)
        line["config3_prefill"] = measure_prefill(pkg, torch, dev, 2048, 5, 3, world, rank)
        line["gpu_launches_all_workloads"] = (line["gpu_launches"] + 640
                                              + r4["launches_per_step"] * B64_STEPS
                                              + r5["launches_per_step"] * BOX_STEPS
                                              + line["config3_prefill"]["launches_per_step"] * 5)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(BOX_PROMPT if box else PROMPT, args.cpu_steps,
                                            len(os.sched_getaffinity(0)), config["workload"])
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
