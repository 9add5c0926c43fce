"""The checkpoint loader (loader.py, mirroring src/safetensors.ts, src/quant.ts and the upload of
src/engine.ts:530-603): header parsing and its refusals, the quantization rules, the ties, the
text tensor selection, and a round trip of a model through a safetensors file. CPU tests export
the oracle's synthetic model; the GPU test loads a file into a fresh context and generates the
same tokens as the context it came from."""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest

import __graft_entry__ as entry

SEED = 0x6E6D6134


@pytest.fixture(scope="module")
def L(pkg):
    return pkg.loader


def blob(header: dict, payload: bytes = b"") -> bytes:
    h = json.dumps(header).encode()
    return struct.pack("<Q", len(h)) + h + payload


def test_parse_header_entries_and_refusals(L):
    good = blob({"__metadata__": {"format": "pt"},
                 "b": {"dtype": "F32", "shape": [2], "data_offsets": [4, 12]},
                 "a": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]}}, bytes(12))
    d = L.parse_header(good)
    assert [t.name for t in d.tensors] == ["a", "b"]          # sorted by payload offset
    assert d.by_name["b"].file_start == d.payload_start + 4 and d.metadata == {"format": "pt"}
    assert L.coverage_gaps(d) == []
    gap = L.parse_header(blob({"a": {"dtype": "U8", "shape": [4], "data_offsets": [8, 12]}}))
    assert L.coverage_gaps(gap) == [(0, 8)]
    cases = {
        "short-prefix": b"\x01\x00",
        "bad-header-length": struct.pack("<Q", 0),
        "truncated-header": struct.pack("<Q", 100) + b"{}",
        "bad-json": blob({"a": 1})[:8] + b"{not json}"[:len(blob({"a": 1})) - 8],
        "bad-dtype": blob({"a": {"dtype": "F7", "shape": [1], "data_offsets": [0, 1]}}),
        "bad-shape": blob({"a": {"dtype": "U8", "shape": [-1], "data_offsets": [0, 1]}}),
        "bad-offsets": blob({"a": {"dtype": "U8", "shape": [1], "data_offsets": [3, 2]}}),
        "size-mismatch": blob({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 4]}}),
        "overlap": blob({"a": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]},
                         "b": {"dtype": "U8", "shape": [4], "data_offsets": [2, 6]}}),
        "bad-entry": blob({"__metadata__": [1]}),
    }
    for kind, data in cases.items():
        with pytest.raises(L.SafetensorsError) as e:
            L.parse_header(data)
        assert e.value.kind == kind, (kind, e.value)
    L.parse_header(cases["overlap"], reject_overlaps=False)


def test_quant_rules_leftmost_match(L):
    lm = "model.language_model."
    assert L.resolve_quant_bits("lm_head") == 2
    assert L.resolve_quant_bits(lm + "embed_tokens") == 2
    assert L.resolve_quant_bits(lm + "embed_tokens_per_layer") == 4
    for layer in (0, 9, 14):
        assert L.resolve_quant_bits(f"{lm}layers.{layer}.mlp.down_proj") == 4     # producers
    for layer in (15, 20, 34):
        assert L.resolve_quant_bits(f"{lm}layers.{layer}.mlp.gate_proj") == 2     # consumers
    assert L.resolve_quant_bits(f"{lm}layers.3.per_layer_input_gate") == 8
    assert L.resolve_quant_bits(f"{lm}layers.30.per_layer_projection") == 8
    assert L.resolve_quant_bits(f"{lm}layers.30.self_attn.o_proj") == 4
    assert L.resolve_quant_bits(lm + "per_layer_model_projection") is None
    assert L.resolve_quant_bits("model.vision_tower.encoder.x") == 8
    assert L.resolve_quant_bits("model.something_else") == L.DEFAULT_QUANT_BITS


def test_text_selection_and_ties(L):
    names = L.text_tensor_names(35, 20)
    # 9 top-level + per layer 9 + k_norm on producers + 4 suffixes x (7 linears, +2 on producers)
    assert len(names) == 9 + 35 * 9 + 15 + 4 * (35 * 7 + 15 * 2)
    assert "model.language_model.layers.20.self_attn.k_proj.weight" not in names
    assert "lm_head.weight" not in names
    header = {n: {"dtype": "U8", "shape": [1], "data_offsets": [i, i + 1]} for i, n in enumerate(names[:5])}
    header["lm_head.weight"] = {"dtype": "U8", "shape": [1], "data_offsets": [5, 6]}
    header["model.vision_tower.x"] = {"dtype": "U8", "shape": [1], "data_offsets": [6, 7]}
    header["model.language_model.embed_tokens.embedding_quantized"]["data_offsets"] = [2, 3]
    d = L.parse_header(blob(header, bytes(7)))
    sel = L.select_text_tensors(d, 35, 20)
    assert sel.skipped == ["model.vision_tower.x"]
    assert [t.alias for t in sel.tied] == ["lm_head.weight"]
    assert sel.resolved_directory.by_name["lm_head.weight"].name == \
        "model.language_model.embed_tokens.embedding_quantized"
    assert len(sel.missing) == len(names) - 5
    assert L.resolve_tied_tensor_name("lm_head.weight_scale") == "model.language_model.embed_tokens.embedding_scale"


class _OracleAsContext:
    """An oracle model seen through the Context methods export_checkpoint and load_checkpoint use;
    uploads and scalars are recorded."""

    def __init__(self, om):
        self.om, self.up, self.sc = om, {}, {}

    def download(self, name):
        return self.om.tensor(name)

    def scalar(self, name):
        return self.om.scalar(name)

    def upload(self, name, data, offset=0, total=None):
        buf = self.up.setdefault(name, bytearray(total))
        buf[offset:offset + data.nbytes] = np.ascontiguousarray(data).view(np.uint8).tobytes()

    def set_scalar(self, name, value):
        self.sc[name] = np.float32(value)


@pytest.mark.parametrize("checkpoint", [False, True])
def test_export_then_load_round_trip(L, pkg, O, tmp_path, checkpoint):
    a = entry.tiny_checkpoint_arch(pkg) if checkpoint else entry.tiny_arch(pkg)
    om = O.Model(SEED, entry.oracle_arch(O, a))
    src = _OracleAsContext(om)
    path = tmp_path / "model.safetensors"
    n = L.export_checkpoint(src, path, a.layer_count, a.layer_count - a.kv_producer_layers)
    assert path.stat().st_size == n
    d = L.parse_header(path.read_bytes())
    assert L.coverage_gaps(d) == []
    dst = _OracleAsContext(om)
    rep = L.load_checkpoint(dst, path, a.layer_count, a.layer_count - a.kv_producer_layers, scale_policy="exact")
    assert rep.missing == [] and rep.skipped == [] and rep.scales_rounded == 0
    assert len(rep.unused) == 2 * a.layer_count                 # k / v cache scales
    for name, got in dst.up.items():
        np.testing.assert_array_equal(np.frombuffer(bytes(got), np.uint8), om.tensor(name), err_msg=name)
    for name, v in dst.sc.items():
        assert v == np.float32(om.scalar(name)), name
    assert dst.sc["lm_head.input_activation_scale"] == (0.0 if checkpoint else np.float32(om.scalar("lm_head.input_activation_scale")))


@pytest.mark.gpu
@pytest.mark.parametrize("checkpoint", [False, True])
def test_loaded_context_generates_the_same_tokens(L, pkg, O, tmp_path, cuda, checkpoint):
    a = entry.tiny_checkpoint_arch(pkg) if checkpoint else entry.tiny_arch(pkg)
    shared = a.layer_count - a.kv_producer_layers
    src = pkg.engine.Context(device=0, max_seqs=1, max_context=64, max_step_columns=16, arch=a)
    src.init_random(SEED)
    path = tmp_path / "model.safetensors"
    L.export_checkpoint(src, path, a.layer_count, shared)
    prompt = O.synth_prompt(SEED + 8, 14, a.vocab_size)
    want = list(pkg.engine.Gemma4Mobile(src).generate(prompt, max_new_tokens=6))
    src.close()
    dst = pkg.engine.Context(device=0, max_seqs=1, max_context=64, max_step_columns=16, arch=a)
    rep = L.load_checkpoint(dst, path, a.layer_count, shared)
    assert rep.missing == [] and rep.scales_rounded == 0
    got = list(pkg.engine.Gemma4Mobile(dst).generate(prompt, max_new_tokens=6))
    dst.close()
    assert got == want
    om = O.Model(SEED, entry.oracle_arch(O, a))
    assert got == [int(t) for t in om.generate(prompt, 6, 64)[0]]
