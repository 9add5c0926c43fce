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
    assert c["qgemv-4bit"] == 35 * 4 and c["qgemv-8bit"] == 35 * 2
    assert c["attention-blocks"] == 35 and c["argmax-final"] == 1
    assert len(P.plan_prefill_chunk(P.GEMMA4_E2B, False)) == 3 + 15 * 9


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
