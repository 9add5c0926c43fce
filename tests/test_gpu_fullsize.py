"""Parity at the full Gemma-4-E2B shape on BASELINE configs 3, 4 and 5, through the C ABI.

The oracle's prefill at these sizes takes minutes on the host, so its results are committed
(tests/golden/config{3,4,5}_*.json, made by tests/golden/make_golden.py): the greedy token and a
SHA-256 of the f32 logits of every step. The device must reproduce both bit for bit. Beside the
oracle, each test checks a size-independent property of the path: chunked prefill equals one
chunk (config 3), a batched step equals one-sequence steps column for column (config 4), and a
PLE table in 128 MiB vocab-row slices equals the unsliced table (config 5).
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
SEED = 0x6E6D6134
GOLDEN = Path(__file__).resolve().parent / "golden"


def digest(logits: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(logits, np.float32).tobytes()).hexdigest()


def golden(name: str) -> dict:
    return json.loads((GOLDEN / name).read_text())


def test_config3_prefill_2048(pkg, cuda):
    """2048-token prefill with the KV-sharing exit: positions 0..2046 run the 15 producer layers
    as tensor-core GEMMs over 2047 columns, the last position all 35 layers and the head."""
    g = golden("config3_prefill.json")
    n = g["prompt_len"]
    prompt = np.array(pkg.plan.synth_prompt(g["prompt_seed"], n), np.int32)
    ctx = pkg.engine.Context(device=0, max_seqs=2, max_context=n + 8, max_step_columns=n)
    ctx.init_random(SEED)
    tok = ctx.prefill(0, prompt, 0, True)
    assert tok == g["tokens"][0]
    assert digest(ctx.logits(0)) == g["logits"][0]["sha256"]
    # The next decode step reads the 2048 stored KV rows of every producer layer.
    tok1 = ctx.decode(0, tok, n)
    assert tok1 == g["tokens"][1]
    assert digest(ctx.logits(0)) == g["logits"][1]["sha256"]
    # The same prompt in 512-column chunks (three producer-only chunks, then the last) gives the
    # same logits bit for bit.
    for start in range(0, n, 512):
        t = ctx.prefill(1, prompt[start:start + 512], start, start + 512 >= n)
    assert t == tok
    assert digest(ctx.logits(0)) == g["logits"][0]["sha256"]
    ctx.close()


def test_config4_ragged_b64(pkg, cuda):
    """64 sequences with prompt lengths U[128, 4096]: the batched steps reproduce the oracle's
    tokens and logits for the shortest, the longest and the first sequence, and every one of the
    64 columns equals that sequence decoded alone."""
    g = golden("config4_ragged.json")
    lens = g["lens"]
    B, steps = len(lens), g["decode_steps"]
    ctx = pkg.engine.Context(device=0, max_seqs=B, max_context=max(lens) + steps + 8,
                             max_step_columns=512)
    ctx.init_random(SEED)
    picks = {int(b): v for b, v in g["sequences"].items()}
    first = []
    for b in range(B):
        first.append(ctx.prefill(b, np.array(pkg.plan.synth_prompt(SEED + b, lens[b]), np.int32), 0, True))
        if b in picks:
            assert first[b] == picks[b]["tokens"][0], b
            assert digest(ctx.logits(0)) == picks[b]["logits"][0]["sha256"], b
    toks = [list(first)]
    for i in range(steps):
        out = ctx.decode_batch(np.arange(B), toks[-1], [lens[b] + i for b in range(B)])
        toks.append([int(t) for t in out])
        for b, v in picks.items():
            assert toks[-1][b] == v["tokens"][i + 1], (b, i)
            assert digest(ctx.logits(b)) == v["logits"][i + 1]["sha256"], (b, i)
    # Column for column: each sequence alone, rewound to its prompt.
    for b in range(B):
        ctx.kv_truncate(b, lens[b])
        prev = first[b]
        for i in range(steps):
            prev = ctx.decode(b, prev, lens[b] + i)
            assert prev == toks[i + 1][b], (b, i)
    ctx.close()


def test_config5_box_sliced_table(pkg, cuda):
    """The box's 512 sequences of 512 tokens on one replica with the PLE table in 128 MiB
    vocab-row slices: 9 slices of 29,952 rows (the last 22,528), results identical to the
    oracle for three sequences and to an unsliced table for all 512."""
    g = golden("config5_box.json")
    S, n, steps = g["sequences_total"], g["prompt_len"], g["decode_steps"]
    prompts = [np.array(pkg.plan.synth_prompt(SEED + b, n), np.int32) for b in range(S)]
    picks = {int(b): v for b, v in g["sequences"].items()}
    runs = []
    for slice_bytes in (128 << 20, 0):
        ctx = pkg.engine.Context(device=0, max_seqs=S, max_context=n + steps + 8,
                                 max_step_columns=512, ple_slice_bytes=slice_bytes)
        ctx.init_random(SEED)
        assert ctx.ple_slices() == ((9, 29952, 22528) if slice_bytes else (1, 262144, 262144))
        toks = [[ctx.prefill(b, prompts[b], 0, True) for b in range(S)]]
        logits = []
        for i in range(steps):
            toks.append([int(t) for t in ctx.decode_batch(np.arange(S), toks[-1], [n + i] * S)])
            logits.append({b: digest(ctx.logits(b)) for b in picks})
        runs.append((toks, logits))
        ctx.close()
    for toks, logits in runs:
        for b, v in picks.items():
            assert [t[b] for t in toks] == v["tokens"], b
            for i in range(steps):
                assert logits[i][b] == v["logits"][i + 1]["sha256"], (b, i)
    assert runs[0][0] == runs[1][0]
