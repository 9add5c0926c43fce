"""g4_op_attention_noalloc: attention whose scratch is a fixed file-scope device array, for
callers that cannot allocate device memory (a host that has handed every byte to its own pools,
a server that must never wait on or fail in the allocator while serving, an embedding whose
allocator belongs to another runtime). It must return exactly what the allocating operator
returns, call after call, although every call reuses the same array.

This file is collected last on purpose (pytest collects test files in name order)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _attention(lib, fn, torch, q, cache, heads, hd, q_count, q_start, kv_len, window, max_ctx):
    out = torch.full((q_count * heads * hd,), float("nan"), dtype=torch.float32, device=q.device)
    rc = getattr(lib, fn)(q.data_ptr(), cache.data_ptr(), out.data_ptr(), heads, hd, q_count,
                          q_start, kv_len, window, max_ctx, None)
    assert rc == 0, lib.g4_last_error(None).decode()
    torch.cuda.synchronize(q.device)
    return out.cpu().numpy()


def _check_sequence(lib, torch, device, cases, seed):
    """Runs `cases` back to back on the shared array, each compared bit for bit with the
    allocating operator (the tolerance these tests use for attention against itself)."""
    heads, max_ctx = 8, 4096
    g = torch.Generator(device=device).manual_seed(seed)
    for i, (hd, q_count, q_start, kv_len, window) in enumerate(cases):
        cache = torch.randn(2 * max_ctx * hd, device=device, generator=g)
        q = torch.randn(q_count * heads * hd, device=device, generator=g)
        want = _attention(lib, "g4_op_attention", torch, q, cache, heads, hd, q_count, q_start,
                          kv_len, window, max_ctx)
        got = _attention(lib, "g4_op_attention_noalloc", torch, q, cache, heads, hd, q_count,
                         q_start, kv_len, window, max_ctx)
        assert not np.isnan(got).any(), f"case {i}"
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=f"case {i}")


@pytest.mark.parametrize("hd,q_count,q_start,kv_len,window", [
    (512, 1, 4095, 4096, 0),     # one row over the full 4,096-position context
    (256, 6, 700, 706, 512),     # a prefill-shaped chunk on a sliding layer
])
def test_noalloc_matches_allocating_operator(cuda, lib, hd, q_count, q_start, kv_len, window):
    # Two calls in a row on the shared array, different inputs.
    _check_sequence(lib, cuda, "cuda:0", [(hd, q_count, q_start, kv_len, window)] * 2, 7 + hd)


def test_noalloc_shrinking_calls_read_no_stale_partials(cuda, lib):
    # A large full-context call fills most of the array; a smaller windowed call and a one-row
    # call after it must read only the partials they wrote themselves.
    _check_sequence(lib, cuda, "cuda:0", [
        (512, 3, 4093, 4096, 0),
        (256, 5, 1000, 1005, 512),
        (512, 1, 70, 71, 0),
    ], 11)


def test_noalloc_keeps_callers_device_and_checks_devices(cuda, lib):
    torch = cuda
    heads, hd, max_ctx = 8, 256, 4096
    q = torch.zeros(heads * hd, device="cuda:0")
    cache = torch.zeros(2 * max_ctx * hd, device="cuda:0")
    out = torch.zeros(heads * hd, device="cuda:0")
    host_out = np.zeros(heads * hd, dtype=np.float32)
    rc = lib.g4_op_attention_noalloc(q.data_ptr(), cache.data_ptr(),
                                     host_out.ctypes.data_as(ctypes.c_void_p), heads, hd, 1, 0, 1,
                                     0, max_ctx, None)
    assert rc == -1 and "q's device" in lib.g4_last_error(None).decode()
    if torch.cuda.device_count() < 2:
        return
    # On a second device: same results, and the caller's current device is left as it was.
    torch.cuda.set_device(0)
    _check_sequence(lib, torch, "cuda:1", [(256, 2, 600, 602, 512), (512, 1, 900, 901, 0)], 13)
    assert torch.cuda.current_device() == 0
    other = torch.zeros(heads * hd, device="cuda:1")
    rc = lib.g4_op_attention_noalloc(q.data_ptr(), cache.data_ptr(), other.data_ptr(), heads, hd,
                                     1, 0, 1, 0, max_ctx, None)
    assert rc == -1 and "q's device" in lib.g4_last_error(None).decode()


def test_noalloc_rejects_oversize_request(cuda, lib):
    torch = cuda
    heads, hd, max_ctx = 8, 512, 4096
    q = torch.zeros(300 * heads * hd, device="cuda")
    cache = torch.zeros(2 * max_ctx * hd, device="cuda")
    out = torch.zeros(300 * heads * hd, device="cuda")
    # 300 rows x 64 blocks x 8 heads x 514 floats is far above the 1,048,576-float array.
    rc = lib.g4_op_attention_noalloc(q.data_ptr(), cache.data_ptr(), out.data_ptr(), heads, hd, 300,
                                     3796, 4096, 0, max_ctx, None)
    assert rc == -1
    assert "static array holds 1048576" in lib.g4_last_error(None).decode()
