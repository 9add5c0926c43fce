"""End-to-end parity of the CUDA executor (through the C ABI) against the CPU oracle's forward.

Greedy tokens must be identical and the logits bit-identical: every integer accumulation is
exact and every f32 operation is the same single rounding in the same order on both sides.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import __graft_entry__ as entry

pytestmark = pytest.mark.gpu
SEED = 0x6E6D6134
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def tiny(pkg, O, cuda):
    a = entry.tiny_arch(pkg)
    om = O.Model(SEED, entry.oracle_arch(O, a))
    return a, om


def make_ctx(pkg, a, **kw):
    kw.setdefault("max_seqs", 4)
    kw.setdefault("max_context", 128)
    kw.setdefault("max_step_columns", 16)
    ctx = pkg.engine.Context(device=0, arch=a, **kw)
    ctx.init_random(SEED)
    return ctx


def oracle_run(O, om, prompt, new, max_ctx=128):
    s = O.Sequence(om, max_ctx)
    tok, logits, _ = s.forward(prompt[:-1], 0, False, False) if len(prompt) > 1 else (None, None, None)
    tok, logits, _ = s.forward(prompt[-1:], len(prompt) - 1, True, True, want_logits=True)
    toks, all_logits = [tok], [logits]
    for i in range(1, new):
        tok, logits, _ = s.forward(np.array([toks[-1]], np.int32), len(prompt) + i - 1, True, True,
                                   want_logits=True)
        toks.append(tok)
        all_logits.append(logits)
    return toks, all_logits


def test_weights_match_generator(pkg, O, tiny):
    a, om = tiny
    ctx = make_ctx(pkg, a)
    names = ["model.language_model.layers.0.self_attn.q_proj.weight",
             "model.language_model.layers.1.self_attn.k_proj.weight_scale",
             "model.language_model.layers.3.mlp.down_proj.weight",
             "model.language_model.layers.2.per_layer_input_gate.weight",
             "model.language_model.layers.2.per_layer_projection.weight_scale",
             "model.language_model.layers.1.self_attn.q_norm.weight",
             "model.language_model.embed_tokens.embedding_quantized",
             "model.language_model.embed_tokens_per_layer.embedding_quantized",
             "model.language_model.embed_tokens_per_layer.embedding_scale",
             "model.language_model.per_layer_model_projection.weight",
             "model.language_model.norm.weight"]
    for n in names:
        np.testing.assert_array_equal(ctx.download(n), om.tensor(n), err_msg=n)
    for n in ["model.language_model.layers.0.self_attn.q_proj.input_activation_scale",
              "model.language_model.layers.3.mlp.down_proj.output_activation_scale",
              "model.language_model.layers.2.layer_scalar", "lm_head.input_activation_scale"]:
        assert np.float32(ctx.scalar(n)) == np.float32(om.scalar(n)), n
    ctx.close()


@pytest.mark.parametrize("graphs", [True, False])
def test_generation_bit_exact(pkg, O, tiny, graphs):
    a, om = tiny
    ctx = make_ctx(pkg, a, use_graphs=graphs)
    prompt = O.synth_prompt(SEED, 20, a.vocab_size)
    want, want_logits = oracle_run(O, om, prompt, 8)
    first = ctx.prefill(0, prompt, 0, True)
    got = [first]
    np.testing.assert_array_equal(ctx.logits(0).view(np.uint32), want_logits[0].view(np.uint32))
    for i in range(1, 8):
        got.append(ctx.decode(0, got[-1], len(prompt) + i - 1))
        np.testing.assert_array_equal(ctx.logits(0).view(np.uint32), want_logits[i].view(np.uint32))
    assert got == want
    ctx.close()


def test_engine_generate_lookahead(pkg, O, tiny):
    a, om = tiny
    ctx = make_ctx(pkg, a)
    model = pkg.engine.Gemma4Mobile(ctx)
    prompt = O.synth_prompt(SEED + 1, 33, a.vocab_size)
    want, _ = om.generate(prompt, 10, 128)
    assert list(model.generate(prompt, 10)) == list(want)
    # A second turn that extends the transcript reuses the KV prefix (kv.ts planKvReuse) and
    # matches a cold run of the longer prompt.
    longer = np.concatenate([prompt, np.array(want[:5], np.int32), [7, 8]]).astype(np.int32)
    want2, _ = om.generate(longer, 6, 128)
    assert list(model.generate(longer, 6, lookahead=False)) == list(want2)
    ctx.close()


def test_batch_matches_single(pkg, O, tiny):
    """Column-for-column contract: a batched step computes each sequence exactly as alone."""
    a, om = tiny
    ctx = make_ctx(pkg, a, max_seqs=12, max_step_columns=16)
    B = 11  # more than one 8-column launch group
    prompts = [O.synth_prompt(SEED + 10 + b, 5 + b, a.vocab_size) for b in range(B)]
    toks = [ctx.prefill(b, prompts[b], 0, True) for b in range(B)]
    pos = [len(p) for p in prompts]
    for step in range(3):
        out = ctx.decode_batch(np.arange(B), toks, pos)
        for b in range(B):
            ref, _ = om.generate(prompts[b], step + 2, 128)
            assert out[b] == ref[step + 1], (step, b)
        toks = list(out)
        pos = [p + 1 for p in pos]
    ctx.close()


def test_batched_decode_tensor_core_path(pkg, O, tiny):
    """B = 20 reaches gemm_min_columns: every calibrated linear of the step runs as the column
    quantize + tcgen05 int8 GEMM, and the lm_head GEMM reduces argmax partials per 128-row tile.
    Tokens equal the oracle's, sequence by sequence, with ragged contexts; the head GEMM's
    softcapped logits are bit-identical to the oracle's."""
    a, om = tiny
    ctx = make_ctx(pkg, a, max_seqs=20, max_step_columns=32)
    B = 20
    prompts = [O.synth_prompt(SEED + 40 + b, 3 + (b % 7), a.vocab_size) for b in range(B)]
    toks = [ctx.prefill(b, prompts[b], 0, True) for b in range(B)]
    pos = [len(p) for p in prompts]
    for step in range(3):
        out = ctx.decode_batch(np.arange(B), toks, pos)
        # The per-layer-input tail of a tensor-core step is its two GEMMs, not the fused launch.
        assert "ple-block" not in [k for k, _ in ctx.launch_list()]
        if step == 0:
            for b in (0, 7, B - 1):
                _, want_logits = oracle_run(O, om, prompts[b], 2)
                np.testing.assert_array_equal(ctx.logits(b).view(np.uint32), want_logits[1].view(np.uint32))
        for b in range(B):
            ref, _ = om.generate(prompts[b], step + 2, 128)
            assert out[b] == ref[step + 1], (step, b)
        toks = list(out)
        pos = [p + 1 for p in pos]
    ctx.close()


def test_batched_decode_split_k_modes_identical(pkg, O, tiny):
    """The three K-split forms of few-tile tensor-core launches (thread-block cluster with a
    distributed-shared-memory sum, none, int32 workspace) give the same logits bit for bit."""
    a, om = tiny
    B = 24
    prompts = [O.synth_prompt(SEED + 70 + b, 4 + (b % 5), a.vocab_size) for b in range(B)]
    runs = []
    for mode in (0, 1, 2):
        ctx = make_ctx(pkg, a, max_seqs=B, max_step_columns=32, gemm_split_k=mode)
        toks = [ctx.prefill(b, prompts[b], 0, True) for b in range(B)]
        pos = [len(p) for p in prompts]
        out = ctx.decode_batch(np.arange(B), toks, pos)
        runs.append((list(out), [ctx.logits(b).copy() for b in (0, 11, B - 1)]))
        ctx.close()
    for toks, logits in runs[1:]:
        assert toks == runs[0][0]
        for la, lb in zip(logits, runs[0][1]):
            np.testing.assert_array_equal(la.view(np.uint32), lb.view(np.uint32))


@pytest.mark.parametrize("n,chunk", [(100, 64), (200, 256), (600, 1024)])
def test_prefill_tensor_core_chunks(pkg, O, tiny, n, chunk):
    """A 100-token prompt in 64-column chunks (64 + 35 producer-only columns on the tensor-core
    path, then the last position on the GEMV path), a 200-token prompt in one 199-column chunk
    (64-token tiles, multi-segment launches over several token tiles) and a 600-token prompt in
    one 599-column chunk (128-token tiles at two CTAs per SM, multi-segment q/k/v and gate/up)
    generate the oracle's tokens; the same prompt with the tensor-core path switched off gives
    the same logits bit for bit."""
    a, om = tiny
    max_ctx = 1024 if n > 256 else 256
    prompt = O.synth_prompt(SEED + 7, n, a.vocab_size)
    want, _ = om.generate(prompt, 4, max_ctx)
    logits = []
    for gmin in (16, 1 << 20):
        ctx = make_ctx(pkg, a, max_step_columns=chunk, max_context=max_ctx, gemm_min_columns=gmin)
        got = [ctx.prefill(0, prompt, 0, True)]
        logits.append(ctx.logits(0).copy())
        for i in range(1, 4):
            got.append(ctx.decode_ahead(0, len(prompt) + i - 1))
        assert got == list(want), gmin
        ctx.close()
    np.testing.assert_array_equal(logits[0].view(np.uint32), logits[1].view(np.uint32))


def test_prefill_chunking_and_sliced_table(pkg, O, tiny):
    a, om = tiny
    prompt = O.synth_prompt(SEED + 3, 40, a.vocab_size)
    want, _ = om.generate(prompt, 4, 128)
    # max_step_columns 8 forces five producer chunks; a 256 KiB PLE slice cap splits the
    # 4096-row table (512 B rows) into 8 slices of 512 rows.
    ctx = make_ctx(pkg, a, max_step_columns=8, ple_slice_bytes=256 * 1024)
    t = ctx.prefill(0, prompt, 0, True)
    got = [t]
    for i in range(1, 4):
        got.append(ctx.decode_ahead(0, len(prompt) + i - 1))
    assert got == list(want)
    ctx.close()


def test_cluster_merged_attention_long_contexts(pkg, O):
    """Decode steps whose one-head attention CTAs of a (column, head) span 9 (sliding window 512)
    and 11 (global, a 700-position cache) blocks: clusters past the portable size of 8, whose
    first block merges the partials from its own shared memory. Logits bit-identical to the
    oracle at B=1, and tokens equal to the oracle's for a three-sequence batch whose contexts
    span 2 to 11 blocks."""
    a = entry.tiny_arch(pkg)
    a.sliding_window = 512
    om = O.Model(SEED, entry.oracle_arch(O, a))
    ctx = make_ctx(pkg, a, max_seqs=4, max_context=700, max_step_columns=64)
    prompt = O.synth_prompt(SEED + 71, 600, a.vocab_size)
    want, want_logits = oracle_run(O, om, prompt, 3, 700)
    tok = ctx.prefill(0, prompt, 0, True)
    got = [tok]
    for i in range(1, 3):
        got.append(ctx.decode(0, got[-1], len(prompt) + i - 1))
        np.testing.assert_array_equal(ctx.logits(0).view(np.uint32), want_logits[i].view(np.uint32))
    assert got == list(want)
    lens = [90, 330, 650]
    prompts = [O.synth_prompt(SEED + 80 + b, n, a.vocab_size) for b, n in enumerate(lens)]
    toks = [ctx.prefill(1 + b, prompts[b], 0, True) for b in range(3)]
    out = ctx.decode_batch(np.arange(1, 4), toks, lens)
    for b in range(3):
        ref, _ = om.generate(prompts[b], 2, 700)
        assert out[b] == ref[1], b
    ctx.close()


def test_invalid_calls(pkg, tiny):
    a, _ = tiny
    ctx = make_ctx(pkg, a)
    with pytest.raises(pkg.G4Error, match="outside the vocabulary"):
        ctx.decode(0, a.vocab_size, 0)
    with pytest.raises(pkg.G4Error, match="gap"):
        ctx.decode(0, 1, 5)
    with pytest.raises(pkg.G4Error, match="sequence"):
        ctx.decode(9, 1, 0)
    with pytest.raises(pkg.G4Error, match="outside the context"):
        ctx.prefill(0, np.ones(200, np.int32), 0, True)
    with pytest.raises(pkg.G4Error, match="unknown tensor"):
        ctx.download("model.language_model.layers.99.mlp.up_proj.weight")
    # A decode step holds one new position per sequence (its attention writes that row itself).
    with pytest.raises(pkg.G4Error, match="twice"):
        ctx.decode_batch([0, 0], [1, 2], [0, 0])
    with pytest.raises(pkg.G4Error, match="twice"):
        ctx.step_stage([1, 1], [1, 2], [0, 0])
    ctx.close()


def test_config2_full_model_greedy_128(pkg, O, cuda):
    """BASELINE config 2 on the full Gemma-4-E2B shape: 128-token prompt, 128 greedy tokens,
    identical to the oracle's tokens (tests/golden/config2_tokens.json, regenerated by
    tests/golden/make_golden.py), with the first steps' logits checked bit for bit live."""
    g = json.loads((GOLDEN / "config2_tokens.json").read_text())
    prompt = np.array(g["prompt"], np.int32)
    ctx = pkg.engine.Context(device=0, max_seqs=1, max_context=256, max_step_columns=64)
    ctx.init_random(SEED)
    om = O.Model(SEED)
    s = O.Sequence(om, 256)
    s.forward(prompt[:-1], 0, False, False)
    t0, l0, _ = s.forward(prompt[-1:], 127, True, True, want_logits=True)
    first = ctx.prefill(0, prompt, 0, True)
    np.testing.assert_array_equal(ctx.logits(0).view(np.uint32), l0.view(np.uint32))
    toks = [first]
    for i in range(1, 128):
        toks.append(ctx.decode_ahead(0, 128 + i - 1))
        if i < 3:
            t, li, _ = s.forward(np.array([toks[-2]], np.int32), 128 + i - 1, True, True, want_logits=True)
            np.testing.assert_array_equal(ctx.logits(0).view(np.uint32), li.view(np.uint32))
    assert toks == g["tokens"]
    ctx.close()
    om.close()


@pytest.mark.parametrize("graphs", [True, False])
def test_verify_pass_matches_sequential_decode(pkg, O, tiny, graphs):
    """g4_verify (GpuExecutor.verify, src/runtime.ts:993-1014): answer[i] is the argmax after
    tokens[i], with the logits of the one-token decode step bit for bit, on a draft that is right,
    one that is wrong after its first token, and widths 2 to 8."""
    a, om = tiny
    prompt = O.synth_prompt(SEED + 9, 30, a.vocab_size)
    n = len(prompt)
    want, want_logits = oracle_run(O, om, prompt, 9)
    ctx = make_ctx(pkg, a, max_seqs=1, use_graphs=graphs)
    assert ctx.prefill(0, prompt, 0, True) == want[0]
    for width in (2, 4, 8):
        ctx.kv_truncate(0, n)
        ans = ctx.verify(0, want[:width], n)
        assert ans == want[1:width + 1], width
        for i in range(width):
            np.testing.assert_array_equal(ctx.logits(i).view(np.uint32), want_logits[i + 1].view(np.uint32))
    # A wrong second token: the first answer is still the greedy token, and the next pass (a
    # plain decode at the accepted position) overwrites the rejected row.
    ctx.kv_truncate(0, n)
    wrong = (want[1] + 1) % a.vocab_size
    ans = ctx.verify(0, [want[0], wrong, want[2]], n)
    assert ans[0] == want[1]
    ctx.kv_truncate(0, n + 1)
    assert ctx.decode(0, want[1], n + 1) == want[2]
    np.testing.assert_array_equal(ctx.logits(0).view(np.uint32), want_logits[2].view(np.uint32))
    with pytest.raises(pkg.G4Error, match="verify pass takes 1 to"):
        ctx.verify(0, want[:9], n)
    ctx.close()


def test_speculative_generate_matches_plain(pkg, O, tiny):
    """Gemma4Mobile.generate with speculation (prompt-lookup drafts checked by verify passes)
    yields the plain greedy ids, in fewer passes when drafts are accepted."""
    a, om = tiny
    base = list(O.synth_prompt(SEED + 21, 12, a.vocab_size))
    prompt = base + base[:8]            # a repeat, so the drafter has something to propose
    plain_ctx = make_ctx(pkg, a, max_seqs=1)
    plain = list(pkg.engine.Gemma4Mobile(plain_ctx).generate(prompt, max_new_tokens=24))
    plain_ctx.close()
    want, _ = om.generate(np.array(prompt, np.int32), 24, 128)
    assert plain == list(want)
    for cols in (2, 4):
        ctx = make_ctx(pkg, a, max_seqs=1)
        stats = pkg.plan.SpeculationStats()
        model = pkg.engine.Gemma4Mobile(ctx)
        spec = list(model.generate(prompt, max_new_tokens=24, speculate=True, max_columns=cols,
                                   stats=stats))
        assert spec == plain, cols
        assert stats.passes + 1 <= 24
        # The transcript the host keeps equals what the caches hold, so a follow-up prompt reuses it.
        assert ctx.kv_length(0) == model.kv_state.length
        assert model.kv_state.tokens == prompt + spec[:-1]
        ctx.close()


def test_verify_full_model(pkg, cuda):
    """Config-2 shape: a verify pass over the golden greedy continuation answers the next golden
    tokens, with logits bit-identical to the sequential decode steps."""
    g = json.loads((GOLDEN / "config2_tokens.json").read_text())
    prompt = np.array(g["prompt"], np.int32)
    toks = g["tokens"]
    logits = {}
    for mode in ("verify", "decode"):
        ctx = pkg.engine.Context(device=0, max_seqs=1, max_context=256, max_step_columns=64)
        ctx.init_random(SEED)
        assert ctx.prefill(0, prompt, 0, True) == toks[0]
        if mode == "verify":
            assert ctx.verify(0, toks[:8], 128) == toks[1:9]
            logits[mode] = [ctx.logits(i).copy() for i in range(8)]
        else:
            got = []
            for i in range(8):
                got.append(ctx.decode(0, toks[i], 128 + i))
                logits.setdefault(mode, []).append(ctx.logits(0).copy())
            assert got == toks[1:9]
        ctx.close()
    for lv, ld in zip(logits["verify"], logits["decode"]):
        np.testing.assert_array_equal(lv.view(np.uint32), ld.view(np.uint32))


def _plan_arch(pkg, a):
    return pkg.plan.Gemma4Arch(
        layer_count=a.layer_count, hidden_size=a.hidden_size,
        global_layers=tuple(L for L in range(a.layer_count) if (a.global_layer_mask >> L) & 1),
        sliding_window=a.sliding_window, kv_producer_layers=a.kv_producer_layers,
        producer_intermediate=a.producer_intermediate, consumer_intermediate=a.consumer_intermediate,
        vocab_size=a.vocab_size)


def _launches(ctx):
    return [(k, r) for k, r in ctx.launch_list()]


def _planned(steps):
    return [(s.kernel, s.modules) for s in steps]


@pytest.mark.parametrize("graphs", [True, False])
def test_executor_launches_match_plan(pkg, O, tiny, graphs):
    """The executor's compiled plan (g4_last_launch_list) is plan.py's dispatch list launch for
    launch: kernel family and covered modules, for prefill chunks, decode steps (eager, captured
    and replayed), a decode batch and the device-resident advancing step."""
    a, _ = tiny
    P = pkg.plan
    arch = _plan_arch(pkg, a)
    ctx = make_ctx(pkg, a, max_seqs=4, use_graphs=graphs)
    prompt = O.synth_prompt(SEED + 31, 10, a.vocab_size)
    ctx.prefill(0, prompt[:9], 0, False)
    assert _launches(ctx) == _planned(P.plan_prefill_chunk(arch, False, 9))
    tok = ctx.prefill(0, prompt[9:], 9, True)
    assert _launches(ctx) == _planned(P.plan_prefill_chunk(arch, True, 1))
    assert ctx.launches() == len(ctx.launch_list())
    for i in range(3):   # eager, captured, replayed
        tok = ctx.decode(0, tok, 10 + i)
        assert _launches(ctx) == _planned(P.plan_decode_step(arch, 1))
    toks = [ctx.prefill(b, prompt[:4 + b], 0, True) for b in (1, 2, 3)]
    ctx.decode_batch([1, 2, 3], toks, [5, 6, 7])
    assert _launches(ctx) == _planned(P.plan_decode_step(arch, 3))
    ctx.step_stage([0], [tok], [13])
    ctx.step_run_device(1)
    assert _launches(ctx) == _planned(P.plan_decode_step(arch, 1, advance=True))
    ctx.close()


def test_executor_launches_match_plan_full_model(pkg, cuda):
    """Gemma-4-E2B shape: one B=1 decode step is planDecodeStep's 215 launches as plan.py lists
    them (embed 3, 35 layers x 6 with the per-layer-input tail as one launch, head 2)."""
    P = pkg.plan
    ctx = pkg.engine.Context(device=0, max_seqs=1, max_context=64, max_step_columns=16)
    ctx.init_random(SEED)
    tok = ctx.prefill(0, np.arange(1, 9, dtype=np.int32), 0, True)
    ctx.decode(0, tok, 8)
    got = _launches(ctx)
    want = _planned(P.plan_decode_step(P.GEMMA4_E2B, 1))
    assert len(got) == 215 and got == want
    ctx.close()


@pytest.mark.parametrize("checkpoint", [False, True])
def test_int8_weight_copies_bit_identical(pkg, O, tiny, checkpoint):
    """Wide tensor-core steps on the int8 weight copies (gemm_shadow_min_columns) give the packed
    path's logits bit for bit: a 600-token prefill chunk and a 40-sequence decode batch, with the
    int4 family and with the checkpoint's 2-bit family; and the copies follow a weight upload."""
    a = entry.tiny_checkpoint_arch(pkg) if checkpoint else tiny[0]
    prompt = O.synth_prompt(SEED + 12, 600, a.vocab_size)
    outs = []
    for shadow in (32, -1):
        ctx = make_ctx(pkg, a, max_seqs=40, max_context=1024, max_step_columns=1024,
                       gemm_shadow_min_columns=shadow)
        t = ctx.prefill(0, prompt, 0, True)
        lg = [ctx.logits(0).copy()]
        toks = [ctx.prefill(b, prompt[:5 + b], 0, True) for b in range(1, 40)]
        out = ctx.decode_batch(np.arange(1, 40), toks, [5 + b for b in range(1, 40)])
        lg += [ctx.logits(c).copy() for c in (0, 38)]
        name = "model.language_model.layers.0.mlp.up_proj.weight"
        w = ctx.download(name)
        w[:4096] ^= 0x33
        ctx.upload(name, w)
        ctx.kv_truncate(0, 0)
        t2 = ctx.prefill(0, prompt, 0, True)
        lg.append(ctx.logits(0).copy())
        outs.append((t, list(out), t2, lg))
        ctx.close()
    assert outs[0][:3] == outs[1][:3]
    for la, lb in zip(outs[0][3], outs[1][3]):
        np.testing.assert_array_equal(la.view(np.uint32), lb.view(np.uint32))
