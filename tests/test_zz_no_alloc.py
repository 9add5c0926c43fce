"""g4_op_attention_noalloc: attention whose scratch is a fixed file-scope device array, for
callers that cannot allocate device memory (a host that has handed every byte to its own pools,
a server that must never wait on or fail in the allocator while serving, an embedding whose
allocator belongs to another runtime). It must return exactly what the allocating operator
returns, call after call, although every call reuses the same array.

This file is collected last on purpose (pytest collects test files in name order)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _attention(lib, fn, torch, q, cache, heads, hd, q_count, q_start, kv_len, window, max_ctx):
    out = torch.full((q_count * heads * hd,), float("nan"), dtype=torch.float32, device="cuda")
    rc = getattr(lib, fn)(q.data_ptr(), cache.data_ptr(), out.data_ptr(), heads, hd, q_count,
                          q_start, kv_len, window, max_ctx, None)
    assert rc == 0, lib.g4_last_error(None).decode()
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("hd,q_count,q_start,kv_len,window", [
    (512, 1, 4095, 4096, 0),     # one row over the full 4,096-position context
    (256, 6, 700, 706, 512),     # a prefill-shaped chunk on a sliding layer
])
def test_noalloc_matches_allocating_operator(cuda, lib, hd, q_count, q_start, kv_len, window):
    torch = cuda
    heads, max_ctx = 8, 4096
    g = torch.Generator(device="cuda").manual_seed(7 + hd)
    cache = torch.randn(2 * max_ctx * hd, device="cuda", generator=g)
    for call in range(2):  # two calls in a row on the shared array, different inputs
        q = torch.randn(q_count * heads * hd, device="cuda", generator=g)
        want = _attention(lib, "g4_op_attention", torch, q, cache, heads, hd, q_count, q_start,
                          kv_len, window, max_ctx)
        got = _attention(lib, "g4_op_attention_noalloc", torch, q, cache, heads, hd, q_count,
                         q_start, kv_len, window, max_ctx)
        assert not np.isnan(got).any()
        # The tolerance these tests use for attention against itself: bit for bit.
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=f"call {call}")


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
