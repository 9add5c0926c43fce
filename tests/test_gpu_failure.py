"""Failure detection without a GPU fault.

A bounded device wait is made to give up by arming an mbarrier for bytes no copy delivers (no
faulting access, no trap): the kernel raises the library's device error flag, waits for its own
copy and exits, the call returns G4_ERR_TIMEOUT, and the device stays usable. Device allocation
failure is injected on the host: context creation returns G4_ERR_OOM with the allocation named,
and releases what it had taken.
"""
from __future__ import annotations

import numpy as np
import pytest

import __graft_entry__ as entry

pytestmark = pytest.mark.gpu
SEED = 0x6E6D6134
G4_ERR_OOM, G4_ERR_TIMEOUT = -3, -7


def test_bounded_wait_gives_up_and_device_stays_usable(pkg, lib, O, cuda):
    torch = cuda
    src = torch.arange(256, dtype=torch.int32, device="cuda").to(torch.uint8)
    status = torch.zeros(3, dtype=torch.int32, device="cuda")
    want_sum = int(src.to(torch.int64).sum())
    assert lib.g4_op_wait_probe(src.data_ptr(), 256, 0, 1 << 16, status.data_ptr(), None) == 0
    assert status.tolist() == [1, 1, want_sum]
    # The barrier expects 16 bytes nobody sends: the wait gives up after 2^14 polls.
    rc = lib.g4_op_wait_probe(src.data_ptr(), 256, 16, 1 << 14, status.data_ptr(), None)
    assert rc == G4_ERR_TIMEOUT
    assert "gave up after 16384 polls" in lib.g4_last_error(None).decode()
    assert status.tolist() == [0, 1, want_sum]      # its own copy still landed before exit
    # The flag was cleared and the device still computes: the next probe and a generation work.
    assert lib.g4_op_wait_probe(src.data_ptr(), 256, 0, 1 << 16, status.data_ptr(), None) == 0
    a = entry.tiny_arch(pkg)
    ctx = pkg.engine.Context(device=0, max_seqs=1, max_context=64, max_step_columns=16, arch=a)
    ctx.init_random(SEED)
    prompt = O.synth_prompt(SEED, 12, a.vocab_size)
    got = list(pkg.engine.Gemma4Mobile(ctx).generate(prompt, max_new_tokens=4))
    ctx.close()
    want, _ = O.Model(SEED, entry.oracle_arch(O, a)).generate(prompt, 4, 64)
    assert got == list(want)


def test_step_reports_each_units_error_flag(pkg, lib, O, cuda):
    """A step reads its tokens and one error word (the OR of the four kernel units' sticky
    flags) with a single copy. A flag raised on the host, as a bounded wait that ran out would
    raise it, makes the next token-returning call fail with G4_ERR_TIMEOUT and is cleared; the
    same call then succeeds and the tokens still match the oracle. Covered on the GEMV path
    (B=1) and on the tensor-core path (a 20-column decode batch)."""
    a = entry.tiny_arch(pkg)
    om = O.Model(SEED, entry.oracle_arch(O, a))
    ctx = pkg.engine.Context(device=0, max_seqs=20, max_context=64, max_step_columns=32, arch=a)
    ctx.init_random(SEED)
    prompt = O.synth_prompt(SEED + 5, 9, a.vocab_size)
    want, _ = om.generate(prompt, 3, 64)
    tok = ctx.prefill(0, prompt, 0, True)
    assert tok == want[0]
    for unit in range(4):
        assert lib.g4_debug_raise_error_flag(ctx.h, unit) == 0
        with pytest.raises(pkg._abi.G4Error) as e:
            ctx.decode(0, tok, len(prompt))
        assert e.value.code == G4_ERR_TIMEOUT
        assert "bounded device wait gave up" in str(e.value)
        assert ctx.decode(0, tok, len(prompt)) == want[1]
    B = 20
    prompts = [O.synth_prompt(SEED + 60 + b, 4 + b % 5, a.vocab_size) for b in range(B)]
    toks = [ctx.prefill(b, prompts[b], 0, True) for b in range(B)]
    pos = [len(p) for p in prompts]
    assert lib.g4_debug_raise_error_flag(ctx.h, 2) == 0
    with pytest.raises(pkg._abi.G4Error) as e:
        ctx.decode_batch(np.arange(B), toks, pos)
    assert e.value.code == G4_ERR_TIMEOUT
    out = ctx.decode_batch(np.arange(B), toks, pos)
    for b in (0, 11, B - 1):
        ref, _ = om.generate(prompts[b], 2, 64)
        assert out[b] == ref[1], b
    assert lib.g4_debug_raise_error_flag(ctx.h, 4) == -1      # no such unit
    ctx.close()


def test_wait_probe_rejects_bad_arguments(lib, cuda):
    torch = cuda
    src = torch.zeros(64, dtype=torch.uint8, device="cuda")
    status = torch.zeros(3, dtype=torch.int32, device="cuda")
    assert lib.g4_op_wait_probe(src.data_ptr(), 24, 0, 10, status.data_ptr(), None) == -1   # not x16
    assert lib.g4_op_wait_probe(src.data_ptr() + 8, 16, 0, 10, status.data_ptr(), None) == -1  # unaligned
    assert lib.g4_op_wait_probe(src.data_ptr(), 16, 0, 0, status.data_ptr(), None) == -1    # no polls


def test_allocation_failure_reports_oom_and_releases(pkg, lib, cuda):
    torch = cuda
    a = entry.tiny_arch(pkg)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    failed = 0
    try:
        # Fail the first allocation, then the second, ... until creation needs fewer than nth.
        for nth in range(1, 200):
            lib.g4_debug_fail_allocation(nth)
            try:
                ctx = pkg.engine.Context(device=0, max_seqs=2, max_context=64, max_step_columns=16, arch=a)
            except pkg.G4Error as e:
                assert e.code == G4_ERR_OOM, (nth, e)
                msg = str(e)
                assert "ctx_malloc" in msg and "out of memory" in msg, msg
                assert lib.g4_last_error(None).decode() in msg
                failed += 1
                continue
            lib.g4_debug_fail_allocation(0)
            ctx.close()
            break
    finally:
        lib.g4_debug_fail_allocation(0)
    assert failed >= 15, failed     # every allocation of context creation was made to fail once
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free0 - free1 < (64 << 20), (free0, free1)     # nothing of the failed contexts stays
    ctx = pkg.engine.Context(device=0, max_seqs=2, max_context=64, max_step_columns=16, arch=a)
    ctx.init_random(SEED)
    assert ctx.prefill(0, np.arange(5, dtype=np.int32), 0, True) >= 0
    ctx.close()
