"""Host-side logic mirrored from the reference's plan.ts, kv.ts and tableSplit.ts (no GPU)."""
from __future__ import annotations

import pytest


@pytest.fixture(scope="module")
def P(pkg):
    return pkg.plan


def test_prefill_chunks(P):
    ch = P.prefill_chunks(0, 128, 64)
    assert [(c.start, c.end) for c in ch] == [(0, 64), (64, 127), (127, 128)]
    assert P.prefill_chunks(0, 1) == [P.PrefillChunk(0, 1, 1)]
    assert P.prefill_chunks(5, 5) == []
    assert [c.length for c in P.prefill_chunks(10, 60, 64)] == [49, 1]
    assert [(c.start, c.end) for c in P.prefill_chunks(0, 385, 64)][-2:] == [(320, 384), (384, 385)]
    with pytest.raises(ValueError):
        P.prefill_chunks(3, 2)
    with pytest.raises(ValueError):
        P.prefill_chunks(0, 5, 0)


def test_kv_roles(P):
    a = P.GEMMA4_E2B
    assert P.kv_role_for_layer(a, 3) == {"kind": "producer", "layer": 3}
    for layer in range(15, 35):
        want = 14 if layer in a.global_layers else 13
        assert P.kv_role_for_layer(a, layer)["readsFrom"] == want
    with pytest.raises(ValueError):
        P.kv_role_for_layer(a, 35)


def test_plan_kv_reuse(P):
    assert P.plan_kv_reuse([], [1, 2]).action == "reset"
    assert P.plan_kv_reuse([1, 2], [1, 2, 3]) == P.KvReusePlan("extend", 2, 2, 1)
    assert P.plan_kv_reuse([1, 2, 9], [1, 2, 3, 4]) == P.KvReusePlan("rewind", 2, 2, 2)
    assert P.plan_kv_reuse([1, 2, 3], [1, 2]).action == "reset"      # strict prefix: reset
    assert P.plan_kv_reuse([1, 2], [1, 2]).action == "reset"         # exact match: reset
    assert P.plan_kv_reuse([7], [1]).action == "reset"
    with pytest.raises(ValueError):
        P.plan_kv_reuse([1], [])
    s = P.KvCacheState()
    s.append([1, 2, 3])
    plan = s.accept_prompt([1, 2, 9, 9])
    assert plan.action == "rewind" and s.tokens == [1, 2]
    with pytest.raises(ValueError):
        s.truncate(5)


def test_table_split_plans(P, pkg, O):
    rows, row_bytes = 262144, 4480
    # At the 128 MiB cap of BASELINE config 5: 29,952 rows per slice, 9 slices, the last 22,528.
    plan = P.plan_table_split(rows, row_bytes, 128 << 20, 128 << 20, 128 << 20)
    assert plan.rows_per_slice == 29952 and len(plan.slices) == 9 and plan.slices[-1][2] == 22528
    assert all(s[1] % 16 == 0 for s in plan.slices)
    assert pkg._abi.plan_table_split(rows, row_bytes, 128 << 20, 128 << 20) == (9, 29952, 22528)
    assert O.plan_table_split(rows, row_bytes, 128 << 20, 128 << 20) == (9, 29952, 22528)
    # A 4 GiB adapter holds the whole table in one buffer.
    whole = P.plan_table_split(rows, row_bytes, 4294967292, 4294967292)
    assert whole.single and whole.slices == ((0, 0, rows),)
    # The 1 GiB limit with the default 256 MiB cap.
    p1 = P.plan_table_split(rows, row_bytes, 1 << 30, 1 << 30)
    assert p1.rows_per_slice == (256 << 20) // row_bytes // 16 * 16
    assert P.plan_table_split(rows, row_bytes, 1000, 1000) is None


def test_decode_census(P):
    steps = P.plan_decode_step(P.GEMMA4_E2B)
    c = P.census(steps)
    assert c["qgemv-4bit"] == 35 * 4 and c["ple-block"] == 35 and "qgemv-8bit" not in c
    assert c["attention-decode"] == 35 and c["argmax-final"] == 1 and c["qgemv-4bit-head"] == 1
    assert len(steps) == 3 + 35 * 6 + 2          # 215 launches per B=1 token
    # Producers store KV; consumers attend over producer 13 / 14's cache.
    assert steps[3].modules.endswith("v_proj") and steps[3 + 6 * 20].modules.endswith("q_proj")
    assert steps[3 + 5].modules == "layers.0.per_layer_input_gate,layers.0.per_layer_projection"
    c12 = P.census(P.plan_decode_step(P.GEMMA4_E2B, cols=12))
    assert c12["qgemv-4bit"] == 35 * 4 * 2 and c12["ple-block"] == 35   # one tail launch for 12
    # Past 16 columns, or with a hidden size the cluster launch does not take, the two GEMVs.
    assert P.census(P.plan_decode_step(P.GEMMA4_E2B, cols=17))["qgemv-8bit"] == 35 * 2 * 3
    odd = P.Gemma4Arch(hidden_size=2560)
    assert P.census(P.plan_decode_step(odd))["qgemv-8bit"] == 35 * 2
    chunk = P.plan_prefill_chunk(P.GEMMA4_E2B, False, cols=8)
    assert len(chunk) == 3 + 15 * 7
    last = P.plan_prefill_chunk(P.GEMMA4_E2B, True, cols=1)
    assert last == P.plan_decode_step(P.GEMMA4_E2B)


def test_greedy_loop_semantics(P):
    calls = []

    def decode(prev, pos):
        calls.append((prev, pos))
        return {10: 11, 11: 12, 12: 99}.get(prev, 5)

    out = list(P.run_greedy_loop(10, 8, {99}, 20, decode))
    assert out == [(10, 0), (11, 1), (12, 2)]          # the stop token is not yielded
    assert calls == [(10, 20), (11, 21), (12, 22)]
    assert list(P.run_greedy_loop(99, 8, {99}, 0, decode)) == []
    assert list(P.run_greedy_loop(10, 1, set(), 0, decode)) == [(10, 0)]
    aborted = iter([False, True])
    assert list(P.run_greedy_loop(10, 5, set(), 0, decode, lambda: next(aborted, True))) == [(10, 0)]


def test_lookup_drafter(P):
    d = P.LookupDrafter()
    assert d.name == "lookup-2-8"
    # The suffix [7, 8] occurred earlier, followed by 9, 10.
    assert d.propose([7, 8, 9, 10, 11, 7, 8], 3) == [9, 10, 11]
    # The most recent earlier occurrence wins; proposals stop at the end of what exists.
    assert d.propose([1, 2, 5, 1, 2, 6, 1, 2], 4) == [6, 1, 2]
    # The longest matching suffix wins over a shorter, more recent one.
    assert d.propose([3, 1, 2, 4, 9, 1, 2, 5, 3, 1, 2], 1) == [4]
    assert d.propose([1, 2, 3], 2) == []          # no earlier occurrence
    assert d.propose([1, 2, 1, 2], 0) == []        # nothing wanted
    assert d.propose([1], 2) == []                 # too short for a 2-gram plus one


class _FakeModel:
    """A deterministic 'model': the next token is a fixed function of the previous one, so a
    greedy run is known and verify's answers are checkable."""

    def __init__(self, table):
        self.table = table
        self.passes = []

    def next(self, t):
        return self.table[t % len(self.table)]

    def decode(self, prev, pos):
        self.passes.append(("decode", pos, 1))
        return self.next(prev)

    def verify(self, tokens, pos):
        self.passes.append(("verify", pos, len(tokens)))
        return [self.next(t) for t in tokens]


@pytest.mark.parametrize("max_columns", [2, 4, 8])
def test_speculative_loop_matches_greedy_loop(P, max_columns):
    table = [3, 4, 5, 3, 6, 7, 3, 4, 9, 2]   # 3 -> 4 -> 6 -> 3 ... repeats, so drafts hit
    prompt = [1, 3, 4, 6, 3, 4]
    m = _FakeModel(table)
    greedy = [t for t, _ in P.run_greedy_loop(m.next(prompt[-1]), 20, set(), len(prompt), m.decode)]
    m2 = _FakeModel(table)
    stats = P.SpeculationStats()
    advanced = []
    spec = [t for t, _ in P.run_speculative_loop(
        m2.next(prompt[-1]), 20, set(), len(prompt), prompt, max_columns, P.LookupDrafter(),
        m2.decode, m2.verify, on_advance=lambda t, p: advanced.append((t, p)), stats=stats)]
    assert spec == greedy
    assert stats.tokens == 19 and stats.passes < 19          # drafts were accepted
    assert stats.acceptance_rate() > 0.5
    assert all(n <= max_columns for _, _, n in m2.passes)
    # Every advanced row is a transcript token at its own position.
    transcript = prompt + greedy
    assert [t for t, _ in advanced] == transcript[len(prompt):len(prompt) + len(advanced)]
    assert [p for _, p in advanced] == list(range(len(prompt), len(prompt) + len(advanced)))


def test_speculative_loop_stops_and_refuses_short_answers(P):
    table = [3, 4, 5, 3, 6, 7, 3, 4, 9, 2]
    prompt = [1, 3, 4, 6, 3, 4]
    m = _FakeModel(table)
    spec = [t for t, _ in P.run_speculative_loop(m.next(prompt[-1]), 20, {3}, len(prompt), prompt, 4,
                                                 P.LookupDrafter(), m.decode, m.verify)]
    assert spec == [6]                   # the stop token (3) is never yielded
    bad = _FakeModel(table)
    with pytest.raises(RuntimeError, match="answered"):
        list(P.run_speculative_loop(6, 20, set(), len(prompt), prompt + [6, 3, 4, 6], 4,
                                    P.LookupDrafter(), bad.decode, lambda toks, pos: [1]))
