"""The checkpoint's 2-bit family on the device (src/kernels/qgemv.ts:693-868, qlayout.ts:160-234,
repack.ts:17-209, plan.ts:116-122): the repack to the interleaved tile layout, the GEMV's integer
path (accumulators and y bit-exact against the oracle) and f32 path (the uncalibrated head: bit-exact
against the oracle's restatement of the kernel's order), the tensor-core GEMM with its 2-bit
unpack (column for column the GEMV), and whole generations of a model whose consumer MLP, embedding
and head are 2-bit (f32 head) matching the oracle token for token."""
from __future__ import annotations

import numpy as np
import pytest

import __graft_entry__ as entry

pytestmark = pytest.mark.gpu
SEED = 0x6E6D6134
RNG = np.random.default_rng(0x2B17)
_KEEP = []


@pytest.fixture(autouse=True)
def _keep_alive():
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


def tile16_numpy(row_words, N, K):
    """rowWordsToTile16 (src/kernels/qlayout.ts:186-206) in numpy."""
    codes = np.zeros((-(-N // 16) * 16, K), np.uint32)
    rw = row_words.reshape(N, K // 16)
    for i in range(16):
        codes[:N, i::16] = (rw >> np.uint32(2 * i)) & np.uint32(3)
    tiles = codes.reshape(-1, 16, K)
    out = np.zeros((tiles.shape[0], K), np.uint32)
    for r in range(16):
        out |= tiles[:, r, :] << np.uint32(2 * r)
    return out.reshape(-1)


def make_2bit(cuda, lib, N, K):
    row_words = RNG.integers(0, 2 ** 32, N * K // 16, dtype=np.uint64).astype(np.uint32)
    d_rows = dev(cuda, row_words)
    d_tiles = cuda.zeros(-(-N // 16) * K, dtype=cuda.int32, device="cuda")
    _KEEP.append(d_tiles)
    call(lib, "g4_op_repack_tile16", d_rows.data_ptr(), d_tiles.data_ptr(), N, K, 0, None)
    return row_words, d_tiles


@pytest.mark.parametrize("N,K", [(21, 512), (12288, 1536), (1536, 12288), (262, 1536)])
def test_repack_matches_layout_and_round_trips(cuda, lib, N, K):
    row_words, d_tiles = make_2bit(cuda, lib, N, K)
    np.testing.assert_array_equal(host(d_tiles).view(np.uint32), tile16_numpy(row_words, N, K))
    back = cuda.zeros(N * K // 16, dtype=cuda.int32, device="cuda")
    call(lib, "g4_op_repack_tile16", back.data_ptr(), d_tiles.data_ptr(), N, K, 1, None)
    np.testing.assert_array_equal(host(back).view(np.uint32), row_words)


def x_on_grid(cols, K, scale):
    codes = RNG.integers(-127, 128, (cols, K))
    x = (codes.astype(np.float32) * np.float32(scale)).astype(np.float32)
    x[:, ::97] += np.float32(scale * 0.31)
    return x


@pytest.mark.parametrize("N,K,cols,out_s", [
    (12288, 1536, 1, 0.0625), (1536, 12288, 1, 0.0), (21, 512, 1, 0.0625), (1000, 1536, 3, 0.0),
    (12288, 1536, 8, 0.0625), (1536, 12288, 5, 0.0625), (262144 // 64, 1536, 2, 0.0),
])
def test_qgemv2_integer_path_exact(cuda, lib, O, N, K, cols, out_s):
    row_words, d_tiles = make_2bit(cuda, lib, N, K)
    sc = np.float16(RNG.uniform(4e-3, 4e-2, N)).view(np.uint16)
    x = x_on_grid(cols, K, 0.02)
    in_s, out_s = np.float32(0.02), np.float32(out_s)
    y_ref, acc_ref = O.qgemv(row_words.view(np.uint8), sc, x, in_s, out_s, 2, N, K, cols)
    dy = cuda.full((cols, N), np.nan, dtype=cuda.float32, device="cuda")
    dacc = cuda.zeros((cols, N), dtype=cuda.int32, device="cuda")
    call(lib, "g4_op_qgemv", d_tiles.data_ptr(), dev(cuda, sc).data_ptr(), dev(cuda, x).data_ptr(),
         in_s, out_s, 2, N, K, cols, dy.data_ptr(), dacc.data_ptr(), None)
    np.testing.assert_array_equal(host(dacc), acc_ref)
    np.testing.assert_array_equal(host(dy).view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("N,K,cols", [(4096, 1536, 1), (21, 512, 1), (333, 1536, 3), (8192, 1536, 8)])
def test_qgemv2_f32_path_matches_oracle(cuda, lib, O, N, K, cols):
    """The uncalibrated head's path (in_scale 0.0): bit for bit the oracle's restatement of the
    kernel's order, and within 1e-5 relative of an f64 sum."""
    row_words, d_tiles = make_2bit(cuda, lib, N, K)
    sc = np.float16(RNG.uniform(4e-3, 4e-2, N)).view(np.uint16)
    x = RNG.normal(0, 1, (cols, K)).astype(np.float32)
    y_ref, _ = O.qgemv(row_words.view(np.uint8), sc, x, 0.0, 0.0, 2, N, K, cols)
    dy = cuda.full((cols, N), np.nan, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_qgemv", d_tiles.data_ptr(), dev(cuda, sc).data_ptr(), dev(cuda, x).data_ptr(),
         0.0, 0.0, 2, N, K, cols, dy.data_ptr(), None, None)
    got = host(dy)
    np.testing.assert_array_equal(got.view(np.uint32), y_ref.view(np.uint32))
    u = np.zeros((N, K), np.float64)
    rw = row_words.reshape(N, K // 16).astype(np.uint64)
    for i in range(16):
        u[:, i::16] = ((rw >> np.uint64(2 * i)) & np.uint64(3)).astype(np.float64) - 2.0
    exact = (x.astype(np.float64) @ u.T) * sc.view(np.float16).astype(np.float64)[None]
    assert np.max(np.abs(got - exact) / np.maximum(np.abs(exact), 1.0)) < 1e-5


@pytest.mark.parametrize("N,K,cols,out_s", [
    (12288, 1536, 64, 0.0625), (1536, 12288, 64, 0.0), (1000, 1536, 100, 0.0625),
    (12288, 1536, 512, 0.0), (262, 1536, 17, 0.0625),
])
def test_qgemm2_tensor_core_matches_qgemv(cuda, lib, O, N, K, cols, out_s):
    """The tcgen05 GEMM with the 2-bit tile unpack (u - 2 into the swizzled int8 tile) is column
    for column the oracle's GEMV, including ragged N and the cluster K split."""
    row_words, d_tiles = make_2bit(cuda, lib, N, K)
    sc = np.float16(RNG.uniform(4e-3, 4e-2, N)).view(np.uint16)
    x = x_on_grid(cols, K, 0.02)
    in_s, out_s = np.float32(0.02), np.float32(out_s)
    y_ref, _ = O.qgemv(row_words.view(np.uint8), sc, x, in_s, out_s, 2, N, K, cols)
    dy = cuda.full((cols, N), np.nan, dtype=cuda.float32, device="cuda")
    call(lib, "g4_op_qgemm", d_tiles.data_ptr(), dev(cuda, sc).data_ptr(), dev(cuda, x).data_ptr(),
         in_s, out_s, 2, N, K, cols, dy.data_ptr(), None)
    np.testing.assert_array_equal(host(dy).view(np.uint32), y_ref.view(np.uint32))


@pytest.fixture(scope="module")
def ckpt(pkg, O, cuda):
    a = entry.tiny_checkpoint_arch(pkg)
    om = O.Model(SEED, entry.oracle_arch(O, a))
    return a, om


def test_checkpoint_family_weights_round_trip(pkg, O, ckpt):
    """2-bit tensors download in the checkpoint's row layout (the device holds the tiles), equal
    to the oracle's generator; an upload of the row layout is repacked on arrival."""
    a, om = ckpt
    ctx = pkg.engine.Context(device=0, max_seqs=2, max_context=64, max_step_columns=16, arch=a)
    ctx.init_random(SEED)
    for n in ["model.language_model.layers.3.mlp.down_proj.weight",
              "model.language_model.layers.2.mlp.gate_proj.weight",
              "model.language_model.layers.0.mlp.up_proj.weight",
              "model.language_model.embed_tokens.embedding_quantized"]:
        np.testing.assert_array_equal(ctx.download(n), om.tensor(n), err_msg=n)
    assert ctx.scalar("lm_head.input_activation_scale") == 0.0
    name = "model.language_model.layers.3.mlp.up_proj.weight"
    w = ctx.download(name)
    w2 = w.copy()
    w2[:64] ^= 0x5A
    half = w2.size // 2
    ctx.upload(name, w2[:half], 0, w2.size)
    ctx.upload(name, w2[half:], half, w2.size)
    np.testing.assert_array_equal(ctx.download(name), w2)
    ctx.close()


@pytest.mark.parametrize("graphs", [True, False])
def test_checkpoint_family_generation_bit_exact(pkg, O, ckpt, graphs):
    """Consumer MLP 2-bit at twice the producer width, 2-bit embedding and uncalibrated f32 head:
    the first logits bit-identical and 8 greedy tokens equal to the oracle."""
    a, om = ckpt
    ctx = pkg.engine.Context(device=0, max_seqs=2, max_context=128, max_step_columns=16, arch=a,
                             use_graphs=graphs)
    ctx.init_random(SEED)
    prompt = O.synth_prompt(SEED + 4, 20, a.vocab_size)
    s = O.Sequence(om, 128)
    s.forward(prompt[:-1], 0, False, False)
    t0, l0, _ = s.forward(prompt[-1:], len(prompt) - 1, True, True, want_logits=True)
    got = [ctx.prefill(0, prompt, 0, True)]
    np.testing.assert_array_equal(ctx.logits(0).view(np.uint32), l0.view(np.uint32))
    for i in range(1, 8):
        got.append(ctx.decode(0, got[-1], len(prompt) + i - 1))
    want, _ = om.generate(prompt, 8, 128)
    assert got == list(want)
    ctx.close()


def test_checkpoint_family_batched_and_prefill_paths(pkg, O, ckpt):
    """A 24-sequence batch (consumer 2-bit MLP on the tensor-core GEMM, the f32 head in 8-column
    launches) equals each sequence decoded alone, and a 100-token prompt through tensor-core
    prefill chunks gives the oracle's tokens."""
    a, om = ckpt
    B = 24
    ctx = pkg.engine.Context(device=0, max_seqs=B, max_context=160, max_step_columns=32, arch=a)
    ctx.init_random(SEED)
    prompts = [O.synth_prompt(SEED + 90 + b, 5 + (b % 7), a.vocab_size) for b in range(B)]
    first = [ctx.prefill(b, prompts[b], 0, True) for b in range(B)]
    pos = [len(q) for q in prompts]
    batch = list(ctx.decode_batch(np.arange(B), first, pos))
    logits = [ctx.logits(b).copy() for b in (0, 9, B - 1)]
    for b in range(B):
        ctx.kv_truncate(b, pos[b])
        assert ctx.decode(b, first[b], pos[b]) == batch[b], b
        if b in (0, 9, B - 1):
            np.testing.assert_array_equal(ctx.logits(0).view(np.uint32),
                                          logits[(0, 9, B - 1).index(b)].view(np.uint32))
    long_prompt = O.synth_prompt(SEED + 77, 100, a.vocab_size)
    want, _ = om.generate(long_prompt, 3, 160)
    got = [ctx.prefill(0, long_prompt, 0, True)]
    for i in range(1, 3):
        got.append(ctx.decode_ahead(0, len(long_prompt) + i - 1))
    assert got == list(want)
    ctx.close()
