"""Per-operator parity of the CUDA kernels (through the C ABI) against the CPU oracle.

Integer work (code dots, gathers, argmax) must be bit-exact. f32 kernels evaluate a fixed order
that the oracle mirrors, so they are compared bit for bit as well; against the reference's f64
oracles they are held to the reference's own registry tolerances (src/kernels/*.ts cases).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(0x6E6D6134)


_KEEP = []


@pytest.fixture(autouse=True)
def _keep_alive():
    """Device tensors passed to the C ABI as raw pointers stay referenced for the whole test,
    so the caching allocator cannot hand their memory to the next argument."""
    yield
    _KEEP.clear()


def dev(cuda, a):
    t = cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def call(lib, fn, *args):
    rc = getattr(lib, fn)(*args)
    assert rc == 0, lib.g4_last_error(None).decode()


def p(t):
    return None if t is None else t.data_ptr()


def f16_scales(n, lo=1e-3, hi=1e-2):
    return np.float16(RNG.uniform(lo, hi, n)).view(np.uint16)


def x_on_grid(cols, K, scale):
    # int8 codes uniform in [-127, 127] fed as x = code * scale, plus a few
    # off-grid values so the snap's rounding is exercised.
    codes = RNG.integers(-127, 128, (cols, K))
    x = (codes.astype(np.float32) * np.float32(scale)).astype(np.float32)
    x[:, ::97] += np.float32(scale * 0.31)
    return x


@pytest.mark.parametrize("bits,N,K,cols", [
    (4, 6144, 1536, 1), (4, 1000, 1536, 3), (4, 1536, 6144, 1), (4, 777, 256, 9),
    (8, 256, 1536, 1), (8, 1536, 256, 5), (2, 12288, 1536, 1), (2, 1000, 1024, 3),
])
def test_qgemv_codes_input(cuda, lib, O, bits, N, K, cols):
    """g4_op_qgemv_codes (int8 activation codes in K order, BASELINE config 1's wNa8o8 form) gives
    g4_op_qgemv's accumulators and outputs on x = codes * in_scale, bit for bit (the oracle's
    qgemv on the same x checks both)."""
    wbytes = (N + 15) // 16 * K * 4 if bits == 2 else N * K * bits // 8
    wq = RNG.integers(0, 256, wbytes, dtype=np.uint8)
    sc = f16_scales(N)
    codes = RNG.integers(-127, 128, (cols, K)).astype(np.int8)
    in_s, out_s = np.float32(0.02), np.float32(0.0625)
    x = (codes.astype(np.float32) * in_s).astype(np.float32)
    dw, ds, dx, dc = dev(cuda, wq), dev(cuda, sc), dev(cuda, x), dev(cuda, codes)
    outs = []
    for fn, src in (("g4_op_qgemv", dx), ("g4_op_qgemv_codes", dc)):
        dy = cuda.zeros((cols, N), dtype=cuda.float32, device="cuda")
        dacc = cuda.zeros((cols, N), dtype=cuda.int32, device="cuda")
        call(lib, fn, p(dw), p(ds), p(src), in_s, out_s, bits, N, K, cols, p(dy), p(dacc), None)
        outs.append((host(dacc), host(dy)))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1].view(np.uint32), outs[1][1].view(np.uint32))
    if bits != 2:
        y_ref, acc_ref = O.qgemv(wq, sc, x, in_s, out_s, bits, N, K, cols)
        np.testing.assert_array_equal(outs[1][0], acc_ref)
        np.testing.assert_array_equal(outs[1][1].view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("bits,N,K,cols", [
    (4, 6144, 1536, 1), (4, 1000, 1536, 3), (4, 1536, 6144, 1), (4, 1536, 2048, 2),
    (4, 1536, 4096, 1), (4, 777, 256, 8), (4, 2560, 1536, 13),
    (8, 256, 1536, 1), (8, 1536, 256, 5), (8, 300, 1536, 9),
])
def test_qgemv_exact(cuda, lib, O, bits, N, K, cols):
    wq = RNG.integers(0, 256, N * K * bits // 8, dtype=np.uint8)
    sc = f16_scales(N)
    x = x_on_grid(cols, K, 0.02)
    in_s, out_s = np.float32(0.02), np.float32(0.0625)
    y_ref, acc_ref = O.qgemv(wq, sc, x, in_s, out_s, bits, N, K, cols)
    dw, ds, dx = dev(cuda, wq), dev(cuda, sc), dev(cuda, x)
    dy = cuda.zeros((cols, N), dtype=cuda.float32, device="cuda")
    dacc = cuda.zeros((cols, N), dtype=cuda.int32, device="cuda")
    call(lib, "g4_op_qgemv", p(dw), p(ds), p(dx), in_s, out_s, bits, N, K, cols, p(dy), p(dacc), None)
    np.testing.assert_array_equal(host(dacc), acc_ref)
    np.testing.assert_array_equal(host(dy).view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("bits,N,K,cols,out_s", [
    (4, 6144, 1536, 64, 0.0625), (4, 1000, 1536, 100, 0.0), (4, 1536, 6144, 300, 0.0625),
    (4, 262, 2048, 17, 0.0), (4, 2048, 1536, 129, 0.0625), (8, 256, 1536, 20, 0.0625),
    (8, 1536, 256, 200, 0.0), (8, 300, 1536, 64, 0.0625), (4, 1536, 6144, 64, 0.0625),
    (4, 2048, 256, 33, 0.0), (8, 1536, 256, 64, 0.0625), (4, 40000, 256, 40, 0.0625),
    (8, 38100, 256, 64, 0.0),
])
def test_qgemm_tensor_core_matches_qgemv(cuda, lib, O, bits, N, K, cols, out_s):
    """The tcgen05 int8 GEMM (prefill / batched decode) is column-for-column the qgemv of the
    oracle (src/kernels/qgemm.ts:532-552 contract): y bit-identical, including ragged N (a partial
    128-row tile), ragged columns (partial token tiles), K 6144 (48 pipeline stages) and the K
    splits of few-tile launches (64-token tiles: clusters of 2, 4 or 8 CTAs; wider: workspace)
    and the three-stage, two-CTAs-per-SM form of many-tile 64-token launches."""
    wq = RNG.integers(0, 256, N * K * bits // 8, dtype=np.uint8)
    sc = f16_scales(N)
    x = x_on_grid(cols, K, 0.02)
    in_s, out_s = np.float32(0.02), np.float32(out_s)
    y_ref, _ = O.qgemv(wq, sc, x, in_s, out_s, bits, N, K, cols)
    dy = cuda.full((cols, N), np.nan, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_qgemm", p(dev(cuda, wq)), p(dev(cuda, sc)), p(dev(cuda, x)), in_s, out_s, bits,
         N, K, cols, p(dy), None)
    np.testing.assert_array_equal(host(dy).view(np.uint32), y_ref.view(np.uint32))


def test_qgemv_baseline_config1_fp16(cuda, lib, O):
    """x int8 codes U[-127,127] at static scale 0.02, W int4 U[-8,7] packed 8
    per u32, f16 row scales U[1e-3,1e-2]; int32 accumulators exact, fp16 output within 1e-2."""
    N, K = 6144, 1536
    w = RNG.integers(-8, 8, (N, K))
    u = (w + 8).astype(np.uint8)
    wq = (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8).reshape(-1)
    sc = f16_scales(N)
    codes = RNG.integers(-127, 128, K)
    x = (codes * np.float32(0.02)).astype(np.float32)[None]
    dy = cuda.zeros((1, N), dtype=cuda.float32, device="cuda")
    dacc = cuda.zeros((1, N), dtype=cuda.int32, device="cuda")
    call(lib, "g4_op_qgemv", p(dev(cuda, wq)), p(dev(cuda, sc)), p(dev(cuda, x)), np.float32(0.02),
         np.float32(0.0), 4, N, K, 1, p(dy), p(dacc), None)
    acc_exact = (w.astype(np.int64) @ codes.astype(np.int64)).astype(np.int64)
    np.testing.assert_array_equal(host(dacc)[0], acc_exact)
    y16 = host(dy)[0].astype(np.float16).astype(np.float64)
    y_true = np.float64(0.02) * np.float16(sc.view(np.float16)).astype(np.float64) * acc_exact
    rel = np.abs(y16 - y_true) / np.maximum(np.abs(y_true), 1e-6)
    assert np.max(rel[np.abs(y_true) > 1e-3]) < 1e-2


@pytest.mark.parametrize("bits,N,K", [(4, 512, 1536), (8, 256, 1536)])
def test_qgemv_f32_path(cuda, lib, O, bits, N, K):
    wq = RNG.integers(0, 256, N * K * bits // 8, dtype=np.uint8)
    sc = f16_scales(N)
    x = (RNG.integers(-64, 64, (1, K)) / 8.0).astype(np.float32)
    y_ref, _ = O.qgemv(wq, sc, x, 0.0, 0.0, bits, N, K, 1)
    dy = cuda.zeros((1, N), dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_qgemv", p(dev(cuda, wq)), p(dev(cuda, sc)), p(dev(cuda, x)), 0.0, 0.0, bits, N,
         K, 1, p(dy), None, None)
    np.testing.assert_array_equal(host(dy).view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("bits,N,K,cols,off,stride", [(4, 1536, 6144, 1, 0, 6144),
                                                      (8, 1536, 256, 3, 512, 1024)])
def test_qgemv_gelu(cuda, lib, O, bits, N, K, cols, off, stride):
    wq = RNG.integers(0, 256, N * K * bits // 8, dtype=np.uint8)
    sc = f16_scales(N)
    gate = RNG.normal(0, 2, (cols, K)).astype(np.float32)
    up = RNG.normal(0, 2, (cols, stride)).astype(np.float32)
    act = np.stack([O.gelu_mul(gate[c], up[c, off:off + K]) for c in range(cols)])
    in_s, out_s = np.float32(0.05), np.float32(0.1)
    y_ref, _ = O.qgemv(wq, sc, act, in_s, out_s, bits, N, K, cols)
    dy = cuda.zeros((cols, N), dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_qgemv_gelu", p(dev(cuda, wq)), p(dev(cuda, sc)), p(dev(cuda, gate)),
         p(dev(cuda, up)), off, stride, in_s, out_s, bits, N, K, cols, p(dy), None)
    np.testing.assert_array_equal(host(dy).view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("rows,width", [(1, 1536), (4, 1536), (8, 256), (3, 512), (35, 256)])
def test_norms(cuda, lib, O, rows, width):
    src = RNG.normal(0, 3, rows * width).astype(np.float32)
    res = RNG.normal(0, 1, rows * width).astype(np.float32)
    g = RNG.uniform(0.5, 1.5, width).astype(np.float32)
    g2 = RNG.uniform(0.5, 1.5, width).astype(np.float32)
    eps = np.float32(1e-6)
    ds, dr, dg, dg2 = dev(cuda, src), dev(cuda, res), dev(cuda, g), dev(cuda, g2)
    out = cuda.zeros(rows * width, dtype=cuda.float32, device="cuda")
    hid = cuda.zeros(rows * width, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_rms_norm", p(ds), p(dg), p(out), rows, width, eps, None)
    mirror = O.rms_norm(src, g, rows, width)
    np.testing.assert_array_equal(host(out).view(np.uint32), mirror.view(np.uint32))
    ref = O.rms_norm(src, g, rows, width, ref=True)
    # The reference's norm tolerance: 8 ULP or 3e-4 (src/kernels/mlpEpilogue.ts:340-389).
    assert np.max(np.abs(host(out) - ref)) < 3e-4
    call(lib, "g4_op_rms_norm", p(ds), None, p(out), rows, width, eps, None)
    np.testing.assert_array_equal(host(out).view(np.uint32), O.rms_norm(src, None, rows, width).view(np.uint32))
    call(lib, "g4_op_norm_residual", p(ds), p(dg), p(dr), p(out), rows, width, eps, None)
    np.testing.assert_array_equal(host(out).view(np.uint32),
                                  O.norm_residual(src, g, res, rows, width).view(np.uint32))
    call(lib, "g4_op_norm_residual_norm", p(ds), p(dg), p(dr), p(dg2), np.float32(0.37), p(hid), p(out),
         rows, width, eps, None)
    h_ref, n_ref = O.norm_residual_norm(src, g, res, g2, np.float32(0.37), rows, width)
    np.testing.assert_array_equal(host(hid).view(np.uint32), h_ref.view(np.uint32))
    np.testing.assert_array_equal(host(out).view(np.uint32), n_ref.view(np.uint32))


def test_norm_zero_weight_and_plain_form(cuda, lib, O):
    """A zero gain outputs zeros; the (1 + w) form must not pass (src/kernels/rmsNorm.ts:10-19)."""
    width = 1536
    src = RNG.normal(0, 1, width).astype(np.float32)
    out = cuda.zeros(width, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_rms_norm", p(dev(cuda, src)), p(dev(cuda, np.zeros(width, np.float32))), p(out),
         1, width, np.float32(1e-6), None)
    assert not np.any(host(out))
    g = RNG.uniform(0.5, 1.5, width).astype(np.float32)
    call(lib, "g4_op_rms_norm", p(dev(cuda, src)), p(dev(cuda, g)), p(out), 1, width, np.float32(1e-6), None)
    plain = O.rms_norm(src, g, 1, width, ref=True)
    gemma3 = O.rms_norm(src, (1 + g).astype(np.float32), 1, width, ref=True)
    assert np.max(np.abs(host(out) - plain)) < 3e-4
    assert np.max(np.abs(host(out) - gemma3)) > 0.1


def test_gelu_mul(cuda, lib, O):
    n = 6144
    gate = np.concatenate([RNG.normal(0, 3, n - 8), [0, -0.0, 12, -12, 5.5, -5.5, 1e-4, -30]]).astype(np.float32)
    up = RNG.normal(0, 2, n).astype(np.float32)
    out = cuda.zeros(n, dtype=cuda.float32, device="cuda")
    for srq in (0.0, 0.0625):
        call(lib, "g4_op_gelu_mul", p(dev(cuda, gate)), p(dev(cuda, up)), p(out), n, np.float32(srq), None)
        np.testing.assert_array_equal(host(out).view(np.uint32), O.gelu_mul(gate, up, srq).view(np.uint32))
    call(lib, "g4_op_gelu_mul", p(dev(cuda, gate)), p(dev(cuda, up)), p(out), n, np.float32(0), None)
    ref = O.gelu_mul(gate, up, 0.0, ref=True)
    np.testing.assert_allclose(host(out), ref, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("hd,rot", [(256, 128), (512, 64)])
def test_q_norm_rope_and_kv_store(cuda, lib, O, hd, rot):
    heads, npos, max_ctx, start = 8, 3, 16, 5
    cos_t, sin_t = O.rope_tables(hd, rot, 1e4 if hd == 256 else 1e6, start, npos)
    q = RNG.normal(0, 2, npos * heads * hd).astype(np.float32)
    g = RNG.uniform(0.5, 1.5, hd).astype(np.float32)
    out = cuda.zeros(npos * heads * hd, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_q_norm_rope", p(dev(cuda, q)), p(dev(cuda, g)), p(dev(cuda, cos_t)),
         p(dev(cuda, sin_t)), p(out), npos * heads, hd, heads, np.float32(1e-6), None)
    ref = O.q_norm_rope(q, g, cos_t, sin_t, npos * heads, hd, heads)
    np.testing.assert_array_equal(host(out).view(np.uint32), ref.view(np.uint32))
    k = RNG.normal(0, 2, npos * hd).astype(np.float32)
    v = RNG.normal(0, 2, npos * hd).astype(np.float32)
    cache = np.full(2 * max_ctx * hd, 7.0, np.float32)
    dc = dev(cuda, cache)
    call(lib, "g4_op_kv_norm_rope_store", p(dev(cuda, k)), p(dev(cuda, v)), p(dev(cuda, g)),
         p(dev(cuda, cos_t)), p(dev(cuda, sin_t)), p(dc), npos, hd, start, max_ctx, np.float32(1e-6), None)
    ref_cache = O.kv_norm_rope_store(k, v, g, cos_t, sin_t, cache.copy(), npos, hd, start, max_ctx)
    np.testing.assert_array_equal(host(dc).view(np.uint32), ref_cache.view(np.uint32))


@pytest.mark.parametrize("hd,q_count,q_start,kv_len,window", [
    (256, 1, 0, 1, 512), (256, 1, 200, 201, 512), (256, 1, 700, 701, 512), (512, 1, 300, 301, 0),
    (256, 4, 60, 64, 512), (512, 5, 123, 128, 0), (256, 3, 1000, 1003, 512), (256, 1, 70, 71, 16),
])
def test_attention(cuda, lib, O, hd, q_count, q_start, kv_len, window):
    heads, max_ctx = 8, 1024
    q = RNG.normal(0, 1, q_count * heads * hd).astype(np.float32)
    cache = RNG.normal(0, 1, 2 * max_ctx * hd).astype(np.float32)
    out = cuda.zeros(q_count * heads * hd, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_attention", p(dev(cuda, q)), p(dev(cuda, cache)), p(out), heads, hd, q_count,
         q_start, kv_len, window, max_ctx, None)
    got = host(out)
    mirror = O.attention(q, cache, heads, hd, q_count, q_start, kv_len, window, max_ctx)
    np.testing.assert_array_equal(got.view(np.uint32), mirror.view(np.uint32))
    k = cache[: max_ctx * hd].reshape(max_ctx, hd)[:kv_len]
    v = cache[max_ctx * hd:].reshape(max_ctx, hd)[:kv_len]
    ref = O.ref_attention(q, k, v, heads, hd, q_count, q_start, kv_len, window)
    # The reference's attention gate: cosine >= 0.999 and 1e-4 absolute
    # (src/kernels/attention.ts:1005-1027).
    cos = float(np.dot(got, ref) / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert cos >= 0.999 and np.max(np.abs(got - ref)) < 1e-4


@pytest.mark.parametrize("hd,q_count,q_start,kv_len,window", [
    (256, 300, 200, 500, 128), (256, 97, 0, 97, 512), (512, 130, 70, 200, 0), (512, 3, 5, 8, 0),
    (256, 64, 640, 704, 512), (256, 33, 1000, 1033, 16),
])
def test_attention_prefill_tiled_matches(cuda, lib, O, hd, q_count, q_start, kv_len, window):
    """The query-tiled prefill attention equals the per-(column, block) kernels bit for bit and
    the oracle's mirror, across windows, tile edges and block boundaries."""
    heads, max_ctx = 8, 1200
    q = RNG.normal(0, 1, q_count * heads * hd).astype(np.float32)
    cache = RNG.normal(0, 1, 2 * max_ctx * hd).astype(np.float32)
    dq, dc = dev(cuda, q), dev(cuda, cache)
    out_a = cuda.zeros(q_count * heads * hd, dtype=cuda.float32, device="cuda")
    out_b = cuda.zeros(q_count * heads * hd, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_attention", p(dq), p(dc), p(out_a), heads, hd, q_count, q_start, kv_len, window, max_ctx, None)
    call(lib, "g4_op_attention_prefill", p(dq), p(dc), p(out_b), heads, hd, q_count, q_start, kv_len, window,
         max_ctx, None)
    a, b = host(out_a), host(out_b)
    np.testing.assert_array_equal(b.view(np.uint32), a.view(np.uint32))
    mirror = O.attention(q, cache, heads, hd, q_count, q_start, kv_len, window, max_ctx)
    np.testing.assert_array_equal(b.view(np.uint32), mirror.view(np.uint32))


def test_attention_scale_is_one(cuda, lib, O):
    """Trap 2 (src/kernels/attention.ts:11-18): the kernel matches scale 1.0 and not 1/sqrt(d)."""
    heads, hd, max_ctx, p_ = 8, 256, 256, 99
    q = RNG.normal(0, 1, heads * hd).astype(np.float32)
    cache = RNG.normal(0, 1, 2 * max_ctx * hd).astype(np.float32)
    out = cuda.zeros(heads * hd, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_attention", p(dev(cuda, q)), p(dev(cuda, cache)), p(out), heads, hd, 1, p_, p_ + 1,
         0, max_ctx, None)
    k = cache[: max_ctx * hd].reshape(max_ctx, hd)[: p_ + 1]
    v = cache[max_ctx * hd:].reshape(max_ctx, hd)[: p_ + 1]
    one = O.ref_attention(q, k, v, heads, hd, 1, p_, p_ + 1, 0, 1.0)
    std = O.ref_attention(q, k, v, heads, hd, 1, p_, p_ + 1, 0, 1.0 / np.sqrt(hd))
    got = host(out)
    assert np.max(np.abs(got - one)) < 1e-4
    assert np.max(np.abs(got - std)) > 1e-2


def test_embed_gather_sliced(cuda, lib, O):
    rows, cols, group = 512, 1024, 256
    codes = RNG.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    scales = f16_scales(rows * (cols // group))
    ids = np.array([0, 511, 17, 300, 299, 17], np.int32)
    full = cuda.zeros(len(ids) * cols, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_embed_gather", p(dev(cuda, codes)), p(dev(cuda, scales)), p(dev(cuda, ids)), p(full),
         len(ids), cols, group, np.float32(16.0), 0, 0, None)
    ref = O.embed_gather(codes, scales, ids, cols, group, 16.0)
    np.testing.assert_array_equal(host(full).view(np.uint32), ref.view(np.uint32))
    # Three slices of 176 / 176 / 160 rows: every slot is written by exactly the slice holding it.
    sliced = cuda.full((len(ids) * cols,), -1.0, dtype=cuda.float32, device="cuda")
    row_bytes = cols // 2
    for start, n in ((0, 176), (176, 176), (352, 160)):
        part = dev(cuda, codes[start * row_bytes:(start + n) * row_bytes])
        call(lib, "g4_op_embed_gather", p(part), p(dev(cuda, scales)), p(dev(cuda, ids)), p(sliced),
             len(ids), cols, group, np.float32(16.0), start, n, None)
    np.testing.assert_array_equal(host(sliced).view(np.uint32), ref.view(np.uint32))
    emb = cuda.zeros(len(ids) * 1536, dtype=cuda.float32, device="cuda")
    codes_e = RNG.integers(0, 256, rows * 768, dtype=np.uint8)
    sc_e = f16_scales(rows)
    es = np.float32(np.sqrt(1536.0))
    call(lib, "g4_op_embed_gather", p(dev(cuda, codes_e)), p(dev(cuda, sc_e)), p(dev(cuda, ids)), p(emb),
         len(ids), 1536, 1536, es, 0, 0, None)
    np.testing.assert_array_equal(host(emb).view(np.uint32),
                                  O.embed_gather(codes_e, sc_e, ids, 1536, 1536, es).view(np.uint32))


@pytest.mark.parametrize("N,K,cols", [(8960, 1536, 1), (1000, 1536, 3), (333, 256, 9),
                                      (8960, 1536, 70), (1000, 2048, 40), (130, 1536, 17),
                                      (300, 1536, 100)])
def test_dense_bf16(cuda, lib, O, N, K, cols):
    """One to eight columns: the per-launch kernel; more (prefill): the column-tiled kernel that
    reads the weights once. Both keep the per-lane chunk order, so both are bit-exact."""
    w32 = RNG.uniform(-0.0442, 0.0442, N * K).astype(np.float32)
    w = (w32.view(np.uint32) >> 16).astype(np.uint16)
    x = RNG.normal(0, 1, cols * K).astype(np.float32)
    alpha = np.float32(1536 ** -0.5)
    y = cuda.zeros(cols * N, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_dense_bf16", p(dev(cuda, w)), p(dev(cuda, x)), p(y), N, K, cols, alpha, None)
    np.testing.assert_array_equal(host(y).view(np.uint32), O.dense_bf16(w, x, N, K, cols, alpha).view(np.uint32))


def test_softcap_argmax_ties(cuda, lib, O):
    n = 262144
    logits = RNG.normal(0, 3, n).astype(np.float32)
    logits[[5000, 7, 250000]] = 40.0  # equal maxima: the lowest index wins
    capped = cuda.zeros(n, dtype=cuda.float32, device="cuda")
    tok = cuda.zeros(2, dtype=cuda.int32, device="cuda")
    call(lib, "g4_op_softcap_argmax", p(dev(cuda, logits)), p(capped), p(tok), n, np.float32(30), None)
    ref_capped, ref_tok = O.softcap_argmax(logits, 30.0)
    assert int(host(tok)[0]) == ref_tok == 7
    np.testing.assert_array_equal(host(capped).view(np.uint32), ref_capped.view(np.uint32))


def test_math_against_cuda(cuda, lib, O):
    """The library's exp and tanh against CUDA's expf / tanhf: a few ULP apart, and bit-identical
    to the oracle's restatement."""
    x = np.concatenate([np.linspace(-87, 88, 200001), RNG.normal(0, 5, 20000), [0.0, -0.0, 1e-8]])
    x = x.astype(np.float32)
    n = x.size
    outs = [cuda.zeros(n, dtype=cuda.float32, device="cuda") for _ in range(4)]
    call(lib, "g4_op_math_probe", p(dev(cuda, x)), *(p(o) for o in outs), n, None)
    e, t, ce, ct = (host(o) for o in outs)
    ulp = np.abs(e.view(np.int32).astype(np.int64) - ce.view(np.int32).astype(np.int64))
    assert np.max(ulp[ce > 1e-37]) <= 4
    assert np.max(np.abs(t - ct)) < 4e-7
    oe = np.array([O.lib().g4o_exp(float(v)) for v in x[::101]], np.float32)
    ot = np.array([O.lib().g4o_tanh(float(v)) for v in x[::101]], np.float32)
    np.testing.assert_array_equal(e[::101].view(np.uint32), oe.view(np.uint32))
    np.testing.assert_array_equal(t[::101].view(np.uint32), ot.view(np.uint32))
