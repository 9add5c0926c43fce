"""Regenerate the committed golden fixtures under tests/golden/.

  reference_constants.json  literal known answers read out of the reference's TypeScript source
                            (needs the reference tree; path from $G4_REFERENCE or the argument)
  ref_vectors.json          small seeded cases computed by ref_restate.py, the Python
                            transliteration of the reference's own CPU oracles
  config2_tokens.json       the C oracle's greedy tokens for BASELINE config 2 (seeded synthetic
                            Gemma-4-E2B shape, 128-token prompt, 128 new tokens)
  config3_prefill.json      the oracle's token and logits digest after a 2048-token prefill
  config4_ragged.json       prompt lengths of the 64 ragged sequences, and for three of them the
                            oracle's tokens and logits digests over prefill + 3 decode steps
  config5_box.json          the same for three of the box's 512 sequences (512-token prompts)

Usage: python tests/golden/make_golden.py [reference_root] [--vectors] [--config2] [--config3]
                                          [--config4] [--config5]
Test infrastructure only.
"""
from __future__ import annotations

import json
import os
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(ROOT))

import ref_restate as R  # noqa: E402

SEED = 0x6E6D6134


def find(ref: Path, rel: str, pattern: str):
    """Return (value text, 'rel:line') of the first line matching `pattern` (one group)."""
    lines = (ref / rel).read_text().splitlines()
    for i, line in enumerate(lines, 1):
        m = re.search(pattern, line)
        if m:
            return m.group(1), f"{rel}:{i}"
    raise KeyError(f"{pattern} not found in {rel}")


def reference_constants(ref: Path) -> dict:
    out = {}

    def num(key, rel, pattern, conv=float):
        v, where = find(ref, rel, pattern)
        out[key] = {"value": conv(v), "source": where}

    num("ple_embed_scale", "src/quant.ts", r"export const PLE_EMBED_SCALE = ([0-9.]+);")
    num("final_logit_softcap", "src/kernels/logitSoftcap.ts", r"export const FINAL_LOGIT_SOFTCAP = ([0-9.]+);")
    num("attention_scale", "src/kernels/attention.ts", r"export const ATTENTION_SCALE = ([0-9.]+);")
    num("gelu_coef", "src/kernels/geluMul.ts", r"export const GELU_TANH_COEF = ([0-9.]+);")
    num("gelu_cubic", "src/kernels/geluMul.ts", r"export const GELU_TANH_CUBIC = ([0-9.]+);")
    num("gelu_clamp", "src/kernels/geluMul.ts", r"export const GELU_TANH_CLAMP = ([0-9.]+);")
    num("srq_in_thirds", "src/kernels/qgemv.ts", r"const SRQ_IN_THIRDS = ([0-9.]+);")
    num("srq_in_clamping", "src/kernels/qgemv.ts", r"const SRQ_IN_CLAMPING = ([0-9.]+);")
    num("srq_out", "src/kernels/qgemv.ts", r"const SRQ_OUT = ([0-9.]+);")
    num("argmax_elems_per_wg", "src/kernels/argmax.ts", r"export const ARGMAX_ELEMS_PER_WORKGROUP = ([0-9]+);", int)
    num("sliding_window", "src/kernels/layerGeometry.ts", r"export const SLIDING_WINDOW = ([0-9]+);", int)
    num("kv_producer_layers", "src/kernels/layerGeometry.ts", r"export const KV_PRODUCER_LAYERS = ([0-9]+);", int)
    num("vocab_size", "src/kernels/layerGeometry.ts", r"export const VOCAB_SIZE = ([0-9]+);", int)
    num("default_max_context", "src/kv.ts", r"export const DEFAULT_MAX_CONTEXT = ([0-9]+);", int)
    num("default_prefill_chunk", "src/plan.ts", r"export const DEFAULT_PREFILL_CHUNK = ([0-9]+);", int)
    v, where = find(ref, "src/kernels/layerGeometry.ts", r"GLOBAL_LAYERS: readonly number\[\] = \[([0-9, ]+)\]")
    out["global_layers"] = {"value": [int(t) for t in v.split(",")], "source": where}
    v, where = find(ref, "src/kernels/qgemv.ts", r"export const K_SPAN_PER_ITER = (\{[^}]*\})")
    out["k_span_per_iter"] = {"value": {k: int(x) for k, x in re.findall(r"(\d+): (\d+)", v)}, "source": where}
    v, where = find(ref, "src/tableSplit.ts", r"export const DEFAULT_MAX_SLICE_BYTES = ([0-9 *]+);")
    out["default_max_slice_bytes"] = {"value": int(eval(v)), "source": where}  # "256 * 1024 * 1024"
    # The SRQ tie pinned in the srqCodes comment: f32 quotient exactly -18.5, ties to even -> -18.
    _, where = find(ref, "src/quant.ts", r"(-11\.435039520263672)")
    out["srq_tie"] = {"value": {"x": -11.435039520263672, "scale": 0.6181102395057678,
                                "f64_quotient_rounds_to": -19, "code": -18}, "source": where}
    _, where = find(ref, "src/plan.ts", r"export const (PER_LAYER_INPUT_SCALE) = Math.SQRT1_2")
    out["per_layer_input_scale"] = {"value": 0.7071067811865476, "source": where}
    _, where = find(ref, "src/kernels/subgroupReduce.ts", r"return (32 \* group) \+")
    out["subgroup_selftest"] = {"value": "out[i] = 32 * floor(i/32)*32 + 496", "source": where}
    _, where = find(ref, "src/execute.ts", r"(1,174,405,120)")
    out["ple_table_bytes"] = {"value": 262144 * 4480, "source": where}
    return out


def ref_vectors() -> dict:
    rng = np.random.default_rng(SEED)
    cases = {}
    # qgemv under the reference's fixture rules (src/kernels/qgemv.ts:1365-1388): codes on the
    # integer grid, x on the 1/8 grid, SRQ scales that keep quotients off half integers.
    for bits, k, rows in ((4, 512, 8), (4, 1024, 8), (8, 256, 10)):
        packed = rng.integers(0, 256, rows * k * bits // 8).astype(np.uint8)
        scales = np.float16(rng.uniform(1e-3, 1e-2, rows))
        x = (rng.integers(-64, 65, k) / 8.0).astype(np.float32)
        pk = [int(b) for b in packed]
        sc = [float(s) for s in scales]
        xs = [float(v) for v in x]
        for name, ins, outs in (("thirds", 0.1875, 0.0625), ("clamping", 0.015625, 0.0),
                                ("uncalibrated", 0.0, 0.0)):
            y = R.qgemv_oracle(bits, pk, sc, xs, rows, k, ins, outs)
            acc = R.qgemv_acc(bits, pk, xs, rows, k, ins) if ins else None
            cases[f"qgemv{bits}_{k}_{name}"] = {
                "bits": bits, "k": k, "rows": rows, "in_scale": ins, "out_scale": outs,
                "packed": packed.tobytes().hex(), "scales_f16": scales.view(np.uint16).tolist(),
                "x": xs, "y": y, "acc": acc}
    w = 256
    src = [float(v) for v in np.float32(rng.normal(0, 2, 2 * w))]
    gain = [float(v) for v in np.float32(rng.uniform(0.5, 1.5, w))]
    res = [float(v) for v in np.float32(rng.normal(0, 1, 2 * w))]
    cases["rms_norm"] = {"src": src, "gain": gain, "rows": 2, "width": w, "eps": 1e-6,
                         "y": R.rms_norm_oracle(src, gain, 2, w, 1e-6)}
    cases["norm_residual"] = {"src": src, "gain": gain, "residual": res, "rows": 2, "width": w,
                              "eps": 1e-6, "y": R.norm_residual_oracle(src, gain, res, 2, w, 1e-6)}
    gate = [float(v) for v in np.float32(np.concatenate([rng.normal(0, 3, 60), [12, -12, 5.6, -5.6]]))]
    up = [float(v) for v in np.float32(rng.normal(0, 2, 64))]
    cases["gelu_mul"] = {"gate": gate, "up": up, "y": R.gelu_mul_oracle(gate, up, 64, 0.0),
                         "y_srq": R.gelu_mul_oracle(gate, up, 64, 0.0625)}
    hd, heads, kv = 256, 8, 40
    q = [float(v) for v in np.float32(rng.normal(0, 0.3, heads * hd))]
    kk = [float(v) for v in np.float32(rng.normal(0, 0.3, kv * hd))]
    vv = [float(v) for v in np.float32(rng.normal(0, 1, kv * hd))]
    cases["attention_window16"] = {"q": q, "k": kk, "v": vv, "heads": heads, "hd": hd, "q_start": kv - 1,
                                   "kv_len": kv, "window": 16,
                                   "y": R.attention_oracle(q, kk, vv, heads, hd, 1, kv - 1, kv, 16)}
    cases["attention_global"] = {"q": q, "k": kk, "v": vv, "heads": heads, "hd": hd, "q_start": kv - 1,
                                 "kv_len": kv, "window": 0,
                                 "y": R.attention_oracle(q, kk, vv, heads, hd, 1, kv - 1, kv, 0)}
    codes = rng.integers(0, 256, 6 * 256).astype(np.uint8)
    escales = np.float16(rng.uniform(1e-3, 1e-2, 6 * 2))
    ids = [5, 0, 3, 3]
    cases["ple_gather"] = {"codes": codes.tobytes().hex(), "scales_f16": escales.view(np.uint16).tolist(),
                           "ids": ids, "cols": 512, "group": 256, "out_scale": 16.0,
                           "y": R.embed_gather_oracle([int(b) for b in codes], [float(s) for s in escales],
                                                      ids, 512, 256, 16.0)}
    logits = [float(v) for v in np.float32(rng.normal(0, 5, 300))]
    logits[17] = logits[250] = 41.0
    capped = R.softcap_oracle(logits)
    cases["softcap_argmax"] = {"logits": logits, "capped": capped, "argmax": R.argmax_oracle(capped)}
    for kind, hd_, rot, theta in (("sliding", 256, 128, 1e4), ("global", 512, 64, 1e6)):
        c, s = R.rope_tables(hd_, rot, theta, [0, 1, 77, 2047])
        cases[f"rope_{kind}"] = {"hd": hd_, "rot": rot, "theta": theta, "positions": [0, 1, 77, 2047],
                                 "cos": c, "sin": s,
                                 "inv_freq_last_rotating": R.rope_inverse_frequencies(hd_, rot, theta)[rot - 1]}
    # The 2-bit family (src/kernels/qgemv.ts:693-868): fixtures in the interleaved tile layout,
    # 21 rows (a partial last tile) at K 512, the reference's fixture scales.
    rng2 = np.random.default_rng(SEED + 2)
    rows2, k2 = 21, 512
    row_words = [int(w) for w in rng2.integers(0, 2 ** 32, rows2 * k2 // 16, dtype=np.uint64)]
    tile_words = R.row_words_to_tile16(row_words, rows2, k2)
    assert R.tile16_to_row_words(tile_words, rows2, k2) == row_words
    scales2 = np.float16(rng2.uniform(4e-3, 4e-2, rows2))
    x2 = (rng2.integers(-64, 65, k2) / 8.0).astype(np.float32)
    sc2 = [float(v) for v in scales2]
    xs2 = [float(v) for v in x2]
    for name, ins, outs in (("thirds", 0.1875, 0.0625), ("clamping", 0.015625, 0.0),
                            ("uncalibrated", 0.0, 0.0)):
        cases[f"qgemv2_{k2}_{name}"] = {
            "bits": 2, "k": k2, "rows": rows2, "in_scale": ins, "out_scale": outs,
            "row_words": row_words, "tile_words": tile_words,
            "scales_f16": scales2.view(np.uint16).tolist(), "x": xs2,
            "y": R.qgemv_oracle(2, tile_words, sc2, xs2, rows2, k2, ins, outs),
            "acc": R.qgemv_acc(2, tile_words, xs2, rows2, k2, ins) if ins else None}
    return cases


def config2_tokens() -> dict:
    from oracle import oracle as O
    O.build()
    prompt = O.synth_prompt(SEED, 128)
    m = O.Model(SEED)
    toks, gaps = m.generate(prompt, 128, 256)
    return {"seed": SEED, "prompt_len": 128, "new_tokens": 128, "prompt": prompt.tolist(),
            "tokens": toks.tolist(), "top2_gaps": [float(g) for g in gaps]}


def logits_digest(logits) -> dict:
    """SHA-256 of the f32 logits' bytes (little-endian) plus a few readable values."""
    import hashlib
    x = np.ascontiguousarray(logits, np.float32)
    return {"sha256": hashlib.sha256(x.tobytes()).hexdigest(), "first": [float(v) for v in x[:4]],
            "max": float(x.max())}


def oracle_steps(O, m, prompt, decode_steps: int) -> dict:
    """Prefill with the KV-sharing exit (producer layers for all but the last position), then
    greedy decode steps: the token and the logits digest of every step."""
    n = len(prompt)
    s = O.Sequence(m, n + decode_steps + 8)
    if n > 1:
        s.forward(prompt[:-1], 0, False, False)
    tok, logits, _ = s.forward(prompt[-1:], n - 1, True, True, want_logits=True)
    toks, digests = [tok], [logits_digest(logits)]
    for i in range(decode_steps):
        tok, logits, _ = s.forward(np.array([toks[-1]], np.int32), n + i, True, True, want_logits=True)
        toks.append(tok)
        digests.append(logits_digest(logits))
    return {"prompt_len": n, "tokens": toks, "logits": digests}


def config3_prefill() -> dict:
    """a 2048-token prefill (prompt = synth_prompt(SEED, 2048))."""
    from oracle import oracle as O
    O.build()
    m = O.Model(SEED)
    r = oracle_steps(O, m, O.synth_prompt(SEED, 2048), 1)
    return {"seed": SEED, "prompt_seed": SEED, **r}


B64_LO, B64_HI, B64 = 128, 4096, 64


def config4_lengths() -> list:
    """The ragged prompt lengths of BASELINE config 4: U[128, 4096] from numpy's default_rng(SEED)
    (the same draw bench.py makes)."""
    return [int(v) for v in np.random.default_rng(SEED).integers(B64_LO, B64_HI + 1, B64)]


def config4_ragged() -> dict:
    """64 sequences, prompt b = synth_prompt(SEED + b, lens[b]); the oracle's
    prefill and 3 decode steps for the shortest, the longest and sequence 0."""
    from oracle import oracle as O
    O.build()
    m = O.Model(SEED)
    lens = config4_lengths()
    picks = sorted({int(np.argmin(lens)), int(np.argmax(lens)), 0})
    seqs = {}
    for b in picks:
        seqs[str(b)] = oracle_steps(O, m, O.synth_prompt(SEED + b, lens[b]), 3)
        print(f"config4 sequence {b} (len {lens[b]}) done", flush=True)
    return {"seed": SEED, "lens": lens, "decode_steps": 3, "sequences": seqs}


BOX_SEQS, BOX_PROMPT = 512, 512


def config5_box() -> dict:
    """BASELINE config 5 on one replica: 512 sequences of 512 tokens (prompt b =
    synth_prompt(SEED + b, 512)); the oracle's prefill and 2 decode steps for three of them."""
    from oracle import oracle as O
    O.build()
    m = O.Model(SEED)
    seqs = {}
    for b in (0, 257, 511):
        seqs[str(b)] = oracle_steps(O, m, O.synth_prompt(SEED + b, BOX_PROMPT), 2)
        print(f"config5 sequence {b} done", flush=True)
    return {"seed": SEED, "sequences_total": BOX_SEQS, "prompt_len": BOX_PROMPT, "decode_steps": 2,
            "sequences": seqs}


def main():
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    ref = args[0] if args else os.environ.get("G4_REFERENCE")
    ref = Path(ref) if ref else None
    if ref is not None and ref.exists():
        (HERE / "reference_constants.json").write_text(json.dumps(reference_constants(ref), indent=1))
    if "--vectors" in sys.argv or not any(a.startswith("--config") for a in sys.argv):
        (HERE / "ref_vectors.json").write_text(json.dumps(ref_vectors()))
    if "--config2" in sys.argv:
        (HERE / "config2_tokens.json").write_text(json.dumps(config2_tokens(), indent=1))
    if "--config3" in sys.argv:
        (HERE / "config3_prefill.json").write_text(json.dumps(config3_prefill(), indent=1))
    if "--config4" in sys.argv:
        (HERE / "config4_ragged.json").write_text(json.dumps(config4_ragged(), indent=1))
    if "--config5" in sys.argv:
        (HERE / "config5_box.json").write_text(json.dumps(config5_box(), indent=1))


if __name__ == "__main__":
    main()
