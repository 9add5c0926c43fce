"""The CPU oracle against the reference's literal known answers and against golden vectors from
the Python transliteration of the reference's own CPU oracles (tests/golden/ref_restate.py)."""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def K():
    return json.loads((GOLDEN / "reference_constants.json").read_text())


@pytest.fixture(scope="module")
def V():
    return json.loads((GOLDEN / "ref_vectors.json").read_text())


def test_srq_tie_case(O, K):
    """src/quant.ts:320-329: the f32 quotient is exactly -18.5 and ties-to-even gives -18; the
    f64 quotient would round to -19."""
    t = K["srq_tie"]["value"]
    x, s = np.float32(t["x"]), np.float32(t["scale"])
    assert float(x) == t["x"] and float(s) == t["scale"]  # both are f32 values in the checkpoint
    assert np.float32(x / s) == np.float32(-18.5)
    assert O.lib().g4o_srq_code(x, s) == t["code"] == -18
    assert round(t["x"] / t["scale"]) == t["f64_quotient_rounds_to"]


def test_srq_rounding_and_clamp(O):
    L = O.lib()
    assert L.g4o_srq_code(2.5, 1.0) == 2 and L.g4o_srq_code(3.5, 1.0) == 4
    assert L.g4o_srq_code(-2.5, 1.0) == -2 and L.g4o_srq_code(-0.4, 1.0) == 0
    assert L.g4o_srq_code(1e9, 1.0) == 127 and L.g4o_srq_code(-1e9, 1.0) == -128
    assert L.g4o_srq_out(1.26, 0.0) == np.float32(1.26)  # scale 0: uncalibrated, identity
    assert L.g4o_srq_out(1.26, 0.0625) == np.float32(1.25)


def test_constants(K):
    assert K["attention_scale"]["value"] == 1.0
    assert K["final_logit_softcap"]["value"] == 30.0
    assert K["ple_embed_scale"]["value"] == 16.0 == math.sqrt(256)
    assert K["global_layers"]["value"] == [4, 9, 14, 19, 24, 29, 34]
    assert K["k_span_per_iter"]["value"] == {"2": 512, "4": 256, "8": 128}
    assert K["per_layer_input_scale"]["value"] == math.sqrt(0.5)
    assert np.float32(K["per_layer_input_scale"]["value"]) == np.float32(2 ** -0.5)
    assert K["ple_table_bytes"]["value"] == 1174405120
    # Integer bound (src/kernels/exactSplit.ts:2-3): 8 * 128 * K < 2^24 for K <= 16384.
    assert 8 * 128 * 16384 <= 2 ** 24


def test_f16_conversion_matches_numpy(O):
    L = O.lib()
    vals = np.concatenate([np.linspace(-70000, 70000, 2001), np.geomspace(1e-9, 1e-3, 500),
                           -np.geomspace(1e-9, 1e-3, 500), [0.0, 65504.0, 65520.0]]).astype(np.float32)
    for v in vals:
        assert L.g4o_f32_to_f16(float(v)) == int(np.float16(v).view(np.uint16)), v
    for h in range(0, 65536, 7):
        f = np.uint16(h).view(np.float16)
        if np.isfinite(f):
            assert L.g4o_f16_to_f32(h) == np.float32(f)


def test_exp_tanh_accuracy(O):
    """The oracle's exp and tanh (the ones the kernels mirror) against f64 references."""
    L = O.lib()
    xs = np.concatenate([np.linspace(-87, 88, 20001), np.random.default_rng(1).normal(0, 4, 5000)])
    for x in xs.astype(np.float32):
        e = L.g4o_exp(float(x))
        ref = math.exp(float(x))
        if ref > 1.2e-38:
            assert abs(e - ref) <= 3e-7 * ref, x
        t = L.g4o_tanh(float(x))
        assert abs(t - math.tanh(float(x))) <= 2.5e-7, x


def test_qgemv_golden(O, V):
    for name, c in V.items():
        if not name.startswith("qgemv"):
            continue
        if c["bits"] == 2:
            # The fixtures hold the tile layout; the oracle reads the checkpoint's rows. On the f32
            # path the codes are integers and x sits on the 1/8 grid, so every partial sum is
            # exact in f32 whatever the order, and zero tolerance holds there too.
            packed = np.array(c["row_words"], np.uint32).view(np.uint8)
        else:
            packed = np.frombuffer(bytes.fromhex(c["packed"]), np.uint8)
        scales = np.array(c["scales_f16"], np.uint16)
        x = np.array(c["x"], np.float32)
        y, acc = O.qgemv(packed, scales, x, c["in_scale"], c["out_scale"], c["bits"], c["rows"], c["k"])
        # Zero tolerance on both axes (src/kernels/qgemv.ts:1365-1381 tolerance argument).
        np.testing.assert_array_equal(y[0], np.array(c["y"], np.float32), err_msg=name)
        if c["acc"] is not None:
            np.testing.assert_array_equal(acc[0], np.array(c["acc"], np.int64), err_msg=name)


def test_norms_golden(O, V):
    c = V["rms_norm"]
    src, gain = np.array(c["src"], np.float32), np.array(c["gain"], np.float32)
    ref = O.rms_norm(src, gain, c["rows"], c["width"], ref=True)
    np.testing.assert_allclose(ref, c["y"], rtol=0, atol=2e-7)
    mirror = O.rms_norm(src, gain, c["rows"], c["width"])
    assert np.max(np.abs(mirror - np.array(c["y"]))) < 3e-4  # 8 ULP or 3e-4
    c = V["norm_residual"]
    got = O.norm_residual(c["src"], c["gain"], c["residual"], c["rows"], c["width"])
    assert np.max(np.abs(got - np.array(c["y"]))) < 3e-4


def test_gelu_golden(O, V):
    c = V["gelu_mul"]
    got = O.gelu_mul(np.array(c["gate"], np.float32), np.array(c["up"], np.float32), 0.0)
    np.testing.assert_allclose(got, c["y"], rtol=2e-6, atol=2e-6)
    got_ref = O.gelu_mul(np.array(c["gate"], np.float32), np.array(c["up"], np.float32), 0.0, ref=True)
    np.testing.assert_allclose(got_ref, c["y"], rtol=0, atol=1e-7)
    snapped = O.gelu_mul(np.array(c["gate"], np.float32), np.array(c["up"], np.float32), 0.0625)
    assert np.mean(snapped == np.array(c["y_srq"], np.float32)) > 0.98


@pytest.mark.parametrize("case", ["attention_window16", "attention_global"])
def test_attention_golden(O, V, case):
    c = V[case]
    q, k, v = (np.array(c[n], np.float32) for n in ("q", "k", "v"))
    hd, kv = c["hd"], c["kv_len"]
    cache = np.zeros(2 * kv * hd, np.float32)
    cache[: kv * hd] = k
    cache[kv * hd:] = v
    got = O.attention(q, cache, c["heads"], hd, 1, c["q_start"], kv, c["window"], kv)
    want = np.array(c["y"], np.float32)
    cos = float(np.dot(got, want) / (np.linalg.norm(got) * np.linalg.norm(want)))
    assert cos >= 0.999 and np.max(np.abs(got - want)) < 1e-4
    ref = O.ref_attention(q, k, v, c["heads"], hd, 1, c["q_start"], kv, c["window"])
    np.testing.assert_allclose(ref, want, rtol=0, atol=1e-6)


def test_attention_scale_trap(O, V):
    """Flipping the scale to 1/sqrt(d) must break agreement (src/kernels/attention.ts:11-18)."""
    c = V["attention_global"]
    q, k, v = (np.array(c[n], np.float32) for n in ("q", "k", "v"))
    std = O.ref_attention(q, k, v, c["heads"], c["hd"], 1, c["q_start"], c["kv_len"], 0,
                          1 / math.sqrt(c["hd"]))
    assert np.max(np.abs(std - np.array(c["y"]))) > 1e-2


def test_gather_golden(O, V):
    c = V["ple_gather"]
    got = O.embed_gather(np.frombuffer(bytes.fromhex(c["codes"]), np.uint8),
                         np.array(c["scales_f16"], np.uint16), c["ids"], c["cols"], c["group"],
                         c["out_scale"])
    np.testing.assert_array_equal(got, np.array(c["y"], np.float32))


def test_softcap_argmax_golden(O, V):
    c = V["softcap_argmax"]
    capped, tok = O.softcap_argmax(np.array(c["logits"], np.float32))
    np.testing.assert_allclose(capped, c["capped"], rtol=0, atol=3e-6)
    assert tok == c["argmax"] == 17  # two equal maxima: the lowest index wins


@pytest.mark.parametrize("kind", ["sliding", "global"])
def test_rope_tables_golden(O, V, kind):
    c = V[f"rope_{kind}"]
    cos, sin = [], []
    for pos in c["positions"]:
        cc, ss = O.rope_tables(c["hd"], c["rot"], c["theta"], pos, 1)
        cos += list(cc)
        sin += list(ss)
    np.testing.assert_array_equal(np.array(cos, np.float32), np.array(c["cos"], np.float32))
    np.testing.assert_array_equal(np.array(sin, np.float32), np.array(c["sin"], np.float32))
    if kind == "global":
        # Partial rotary over the FULL head dimension (src/kernels/rope.ts:111-146): the last
        # rotating pair's inverse frequency is about 3.2e-2, and pairs 64.. do not rotate.
        assert abs(c["inv_freq_last_rotating"] - 1e6 ** (-126 / 512)) < 1e-12
        assert 3.0e-2 < c["inv_freq_last_rotating"] < 3.4e-2
        cc, ss = O.rope_tables(512, 64, 1e6, 77, 1)
        assert np.all(cc[64:] == 1.0) and np.all(ss[64:] == 0.0)


def test_oracle_mirror_close_to_reference(O):
    """The mirrored f32 norms sit within the reference's norm tolerance of its f64 oracle."""
    rng = np.random.default_rng(5)
    for width in (256, 512, 1536):
        src = rng.normal(0, 4, 3 * width).astype(np.float32)
        g = rng.uniform(0.5, 1.5, width).astype(np.float32)
        a = O.rms_norm(src, g, 3, width)
        b = O.rms_norm(src, g, 3, width, ref=True)
        assert np.max(np.abs(a - b)) < 3e-4


def test_tile16_layout_restatement(V):
    """The interleaved 2-bit layout (src/kernels/qlayout.ts:160-234) as restated: round trip, the
    code of (row, k) at bits 2 (row % 16) of word (row / 16) K + k, padded rows zero."""
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location(
        "ref_restate", Path(__file__).resolve().parent / "golden" / "ref_restate.py")
    R = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(R)
    c = V["qgemv2_512_thirds"]
    rows, k = c["rows"], c["k"]
    tw = np.array(c["tile_words"], np.uint32)
    rw = np.array(c["row_words"], np.uint32)
    assert tw.size == -(-rows // 16) * k
    for row in (0, 7, 15, 16, 20):
        for kk in (0, 1, 15, 16, 511):
            want = (int(rw[row * (k // 16) + kk // 16]) >> (2 * (kk % 16))) & 3
            assert (int(tw[(row // 16) * k + kk]) >> (2 * (row % 16))) & 3 == want
    # rows 21..31 of the last tile are zero codes
    assert all((int(w) >> 2 * r) & 3 == 0 for w in tw[k:] for r in range(5, 16))
    assert R.tile16_to_row_words(list(map(int, tw)), rows, k) == list(map(int, rw))
