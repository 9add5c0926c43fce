"""Checkpoint loading: the safetensors header, the checkpoint's quantization rules and ties, the
text tensor selection, and the upload of a checkpoint's tensors into a Context.

Mirrors the reference's src/safetensors.ts (parseHeader 163-289, coverageGaps 297-314, the ties
616-706, textTensorNames / selectTextTensors 930-1002), src/quant.ts (QUANT_RULES 430-466 with
the leftmost-match resolution, the storage families 550-663) and the upload step of
src/engine.ts:530-603 (BF16 gains widened to f32, scalars to the scalars map, everything else as
stored). The network fetch (range plans, the tie guard's revision pin) is the browser's and is not
mirrored: a checkpoint here is a local file.

Storage adaptation, stated: the checkpoint's row scales are F32 and this build stores f16 row
scales (BASELINE's storage). `scale_policy="exact"` refuses a scale that f16 cannot hold exactly;
"round" (the default) rounds to the nearest f16 and counts the rows it changed in the report.
"""
from __future__ import annotations

import json
import re
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

# ------------------------------------------------------------------ safetensors (safetensors.ts)

DTYPE_BYTES = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E4M3": 1, "F8_E5M2": 1, "U16": 2, "I16": 2, "F16": 2,
               "BF16": 2, "U32": 4, "I32": 4, "F32": 4, "U64": 8, "I64": 8, "F64": 8}
HEADER_PREFIX_BYTES = 8
MAX_HEADER_BYTES = 64 * 1024 * 1024


class SafetensorsError(ValueError):
    """A malformed or unusable checkpoint; `kind` names the check (the reference's error kinds)."""

    def __init__(self, kind: str, message: str):
        super().__init__(f"{kind}: {message}")
        self.kind = kind


@dataclass(frozen=True)
class TensorEntry:
    name: str
    dtype: str
    shape: tuple
    data_start: int
    data_end: int
    file_start: int
    file_end: int
    byte_length: int
    element_count: int


@dataclass
class SafetensorsDirectory:
    header_length: int
    payload_start: int
    payload_length: int
    file_length: int
    metadata: dict | None
    tensors: list
    by_name: dict


def read_header_length(prefix: bytes) -> int:
    """readHeaderLength (safetensors.ts:130-147): the little-endian u64 that opens the file."""
    if len(prefix) < HEADER_PREFIX_BYTES:
        raise SafetensorsError("short-prefix", f"need {HEADER_PREFIX_BYTES} bytes to read the header "
                                               f"length, got {len(prefix)}")
    raw = struct.unpack_from("<Q", prefix, 0)[0]
    if raw > MAX_HEADER_BYTES:
        raise SafetensorsError("bad-header-length", f"header length {raw} exceeds the {MAX_HEADER_BYTES} byte ceiling")
    if raw <= 0:
        raise SafetensorsError("bad-header-length", f"header length {raw} is not a positive integer")
    return raw


def _is_count(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and v >= 0


def parse_header(data: bytes, reject_overlaps: bool = True) -> SafetensorsDirectory:
    """parseHeader (safetensors.ts:163-289): the JSON header of a safetensors file, every entry
    checked (known dtype, a shape of counts, offsets that span exactly dtype x shape bytes), sorted
    by payload offset, overlapping entries refused."""
    header_length = read_header_length(data)
    needed = HEADER_PREFIX_BYTES + header_length
    if len(data) < needed:
        raise SafetensorsError("truncated-header", f"header claims {header_length} JSON bytes so {needed} "
                                                   f"are needed, got {len(data)}")
    try:
        parsed = json.loads(bytes(data[HEADER_PREFIX_BYTES:needed]).decode("utf-8", errors="replace"))
    except json.JSONDecodeError as e:
        raise SafetensorsError("bad-json", f"header JSON did not parse: {e}") from None
    if not isinstance(parsed, dict):
        raise SafetensorsError("bad-json", "header JSON is not an object")
    metadata = None
    if "__metadata__" in parsed:
        raw = parsed["__metadata__"]
        if not isinstance(raw, dict):
            raise SafetensorsError("bad-entry", "__metadata__ is present but is not an object")
        metadata = {k: v if isinstance(v, str) else str(v) for k, v in raw.items()}
    tensors = []
    for name, entry in parsed.items():
        if name == "__metadata__":
            continue
        if not isinstance(entry, dict):
            raise SafetensorsError("bad-entry", f"tensor {name} is not an object")
        dtype = entry.get("dtype")
        if not isinstance(dtype, str) or dtype not in DTYPE_BYTES:
            raise SafetensorsError("bad-dtype", f"tensor {name} has dtype {dtype}")
        shape = entry.get("shape")
        if not isinstance(shape, list) or not all(_is_count(d) for d in shape):
            raise SafetensorsError("bad-shape", f"tensor {name} has a shape that is not a list of counts")
        count = 1
        for d in shape:
            count *= d
        offs = entry.get("data_offsets")
        if not isinstance(offs, list) or len(offs) != 2 or not all(_is_count(o) for o in offs):
            raise SafetensorsError("bad-offsets", f"tensor {name} has data_offsets that are not a pair of counts")
        start, end = offs
        if end < start:
            raise SafetensorsError("bad-offsets", f"tensor {name} ends at {end} before it starts at {start}")
        if end - start != count * DTYPE_BYTES[dtype]:
            raise SafetensorsError("size-mismatch", f"tensor {name} spans {end - start} bytes but {dtype} "
                                                    f"{shape} needs {count * DTYPE_BYTES[dtype]}")
        tensors.append(TensorEntry(name, dtype, tuple(shape), start, end, needed + start, needed + end,
                                   end - start, count))
    tensors.sort(key=lambda t: (t.data_start, t.data_end, t.name))
    if reject_overlaps:
        for prev, cur in zip(tensors, tensors[1:]):
            if cur.byte_length > 0 and prev.byte_length > 0 and cur.data_start < prev.data_end:
                raise SafetensorsError("overlap", f"tensor {cur.name} starts at {cur.data_start} inside "
                                                  f"{prev.name} which ends at {prev.data_end}")
    payload = max((t.data_end for t in tensors), default=0)
    return SafetensorsDirectory(header_length, needed, payload, needed + payload, metadata, tensors,
                                {t.name: t for t in tensors})


def coverage_gaps(directory: SafetensorsDirectory) -> list:
    """coverageGaps (safetensors.ts:297-314): payload spans no tensor claims, as (start, end)."""
    gaps, cursor = [], 0
    for t in directory.tensors:
        if t.data_start > cursor:
            gaps.append((cursor, t.data_start))
        cursor = max(cursor, t.data_end)
    return gaps


# ------------------------------------------------------------------ ties (safetensors.ts:616-706)

@dataclass(frozen=True)
class TiedTensor:
    alias: str
    source: str
    byte_length: int


TIED_TENSORS = (
    TiedTensor("lm_head.weight", "model.language_model.embed_tokens.embedding_quantized", 100_663_296),
    TiedTensor("lm_head.weight_scale", "model.language_model.embed_tokens.embedding_scale", 1_048_576),
)
_ALIAS_TO_SOURCE = {t.alias: t.source for t in TIED_TENSORS}


def is_tied_alias(name: str) -> bool:
    return name in _ALIAS_TO_SOURCE


def resolve_tied_tensor_name(name: str) -> str:
    return _ALIAS_TO_SOURCE.get(name, name)


def lookup_tensor(directory: SafetensorsDirectory, name: str):
    return directory.by_name.get(resolve_tied_tensor_name(name)) or directory.by_name.get(name)


def apply_ties(directory: SafetensorsDirectory, ties=TIED_TENSORS) -> SafetensorsDirectory:
    """applyTies: the aliases resolve to their source entries; `tensors` stays the file's."""
    if not ties:
        return directory
    by_name = dict(directory.by_name)
    for tie in ties:
        src = directory.by_name.get(tie.source)
        if src is None:
            raise SafetensorsError("bad-entry", f"tie {tie.alias} points at {tie.source} and this "
                                                f"checkpoint does not carry it")
        by_name[tie.alias] = src
    return SafetensorsDirectory(directory.header_length, directory.payload_start, directory.payload_length,
                                directory.file_length, directory.metadata, directory.tensors, by_name)


# ------------------------------------------------------------------ quantization rules (quant.ts)

QUANT_RULES = (
    (r"^lm_head$", 2),
    (r"audio_tower(?!.*lconv1d\.linear_start)", 2),
    (r"audio_tower\.layers\.\d+\.lconv1d\.linear_start\.", 4),
    (r"language_model\.embed_tokens$", 2),
    (r"language_model\.embed_tokens_per_layer$", 4),
    (r"language_model\.layers\.(\d|1[0-4])\.mlp\.", 4),
    (r"language_model\.layers\.\d+\.mlp\.", 2),
    (r"language_model\.layers\.\d+\.per_layer_input_gate$", 8),
    (r"language_model\.layers\.\d+\.per_layer_projection$", 8),
    (r"language_model\.layers\.\d+\.self_attn\.", 4),
    (r"vision_tower", 8),
)
DEFAULT_QUANT_BITS = 4
MODULES_TO_NOT_CONVERT = ("model.vision_tower.patch_embedder", "model.audio_tower.subsample_conv_projection",
                          "model.audio_tower.output_proj", "relative_k_proj", "model.embed_audio",
                          "model.embed_vision", "per_layer_model_projection")


def resolve_quant_bits(module: str) -> int | None:
    """resolveQuantBits: the rules joined as one alternation, the leftmost match wins and an
    earlier rule wins a tie at the same position; None for modules left unquantized."""
    if any(m in module for m in MODULES_TO_NOT_CONVERT):
        return None
    best = None
    for i, (pattern, bits) in enumerate(QUANT_RULES):
        m = re.search(pattern, module)
        if m and (best is None or m.start() < best[0]):
            best = (m.start(), i, bits)
    return best[2] if best else DEFAULT_QUANT_BITS


# ------------------------------------------------------------------ text tensor selection

LINEAR_SUFFIXES = ("weight", "weight_scale", "input_activation_scale", "output_activation_scale")


def text_tensor_names(num_hidden_layers: int, num_kv_shared_layers: int, fetch_tied_pair: bool = False) -> list:
    """textTensorNames (safetensors.ts:930-980): the allow list built from the layer count."""
    layers, shared = max(0, int(num_hidden_layers)), max(0, int(num_kv_shared_layers))
    producers = max(0, layers - shared)
    lm = "model.language_model."
    names = ["lm_head.input_activation_scale", "lm_head.output_activation_scale",
             lm + "embed_tokens.embedding_quantized", lm + "embed_tokens.embedding_scale",
             lm + "embed_tokens_per_layer.embedding_quantized", lm + "embed_tokens_per_layer.embedding_scale",
             lm + "norm.weight", lm + "per_layer_model_projection.weight",
             lm + "per_layer_projection_norm.weight"]
    for layer in range(layers):
        base = f"{lm}layers.{layer}"
        names += [f"{base}.input_layernorm.weight", f"{base}.post_attention_layernorm.weight",
                  f"{base}.pre_feedforward_layernorm.weight", f"{base}.post_feedforward_layernorm.weight",
                  f"{base}.post_per_layer_input_norm.weight", f"{base}.layer_scalar",
                  f"{base}.self_attn.q_norm.weight", f"{base}.self_attn.k_cache_scale",
                  f"{base}.self_attn.v_cache_scale"]
        producer = layer < producers
        if producer:
            names.append(f"{base}.self_attn.k_norm.weight")
        linears = ["self_attn.q_proj", "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj",
                   "per_layer_input_gate", "per_layer_projection"]
        if producer:
            linears += ["self_attn.k_proj", "self_attn.v_proj"]
        for lin in linears:
            names += [f"{base}.{lin}.{s}" for s in LINEAR_SUFFIXES]
    if fetch_tied_pair:
        names += [t.alias for t in TIED_TENSORS]
    return names


@dataclass
class TextTensorSelection:
    names: list
    skipped: list
    missing: list
    tied: list
    resolved_directory: SafetensorsDirectory


def select_text_tensors(directory: SafetensorsDirectory, num_hidden_layers: int, num_kv_shared_layers: int,
                        fetch_tied_pair: bool = False) -> TextTensorSelection:
    """selectTextTensors (safetensors.ts:983-1002)."""
    wanted = text_tensor_names(num_hidden_layers, num_kv_shared_layers, fetch_tied_pair)
    wanted_set = set(wanted)
    tied = [] if fetch_tied_pair else [t for t in TIED_TENSORS if t.alias in directory.by_name]
    aliases = {t.alias for t in tied}
    names, skipped = [], []
    for t in directory.tensors:
        if t.name in wanted_set:
            names.append(t.name)
        elif t.name not in aliases:
            skipped.append(t.name)
    present = set(names)
    missing = [n for n in wanted if n not in present]
    return TextTensorSelection(names, skipped, missing, tied, apply_ties(directory, tied))


# ------------------------------------------------------------------ loading into a Context

def _bf16_to_f32(raw: bytes) -> np.ndarray:
    """bf16ToF32 (quant.ts:400-411): exact widening."""
    return (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even bf16 of f32 values (roundToBf16, quant.ts:418-428), as u16 bits."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    lower, upper = b & 0xFFFF, b >> 16
    up = (lower > 0x8000) | ((lower == 0x8000) & ((upper & 1) == 1))
    return (upper + up.astype(np.uint32)).astype(np.uint16)


def read_scalar_tensor(dtype: str, count: int, raw: bytes):
    """readScalarTensor: a one-element F32 / F16 / BF16 tensor as a float, else None."""
    if count != 1:
        return None
    if dtype == "F32":
        return float(np.frombuffer(raw, np.float32)[0])
    if dtype == "F16":
        return float(np.frombuffer(raw, np.float16)[0])
    if dtype == "BF16":
        return float(_bf16_to_f32(raw)[0])
    return None


@dataclass
class LoadReport:
    uploaded: list = field(default_factory=list)
    scalars: dict = field(default_factory=dict)
    skipped: list = field(default_factory=list)
    missing: list = field(default_factory=list)
    unused: list = field(default_factory=list)     # selected but not held by this build (k/v cache scales)
    scales_rounded: int = 0                        # f32 row scales f16 could not hold exactly


PIECE_BYTES = 64 << 20


def load_checkpoint(ctx, path, num_hidden_layers: int, num_kv_shared_layers: int,
                    scale_policy: str = "round", allow_missing: bool = False) -> LoadReport:
    """Upload a checkpoint's text tensors into `ctx` (src/engine.ts:530-603): quantized codes as
    stored (2-bit tensors in the checkpoint's row layout, repacked on the device), F32 row scales
    to the f16 storage (`scale_policy`), BF16 norm gains widened to f32, the per-layer model
    projection kept BF16, one-element tensors to the scalars. Tensors above PIECE_BYTES go up in
    pieces at their byte offsets (BufferManager.uploadWeight pieces)."""
    if scale_policy not in ("round", "exact"):
        raise ValueError("scale_policy is 'round' or 'exact'")
    path = Path(path)
    with path.open("rb") as f:
        prefix = f.read(HEADER_PREFIX_BYTES)
        hl = read_header_length(prefix)
        directory = parse_header(prefix + f.read(hl))
    sel = select_text_tensors(directory, num_hidden_layers, num_kv_shared_layers)
    rep = LoadReport(skipped=list(sel.skipped), missing=list(sel.missing))
    if sel.missing and not allow_missing:
        raise SafetensorsError("bad-entry", f"{len(sel.missing)} text tensors are not in this checkpoint, "
                                            f"first {sel.missing[0]}")
    with path.open("rb") as f:
        for name in sel.names:
            t = directory.by_name[name]
            f.seek(t.file_start)
            raw = f.read(t.byte_length)
            if len(raw) != t.byte_length:
                raise SafetensorsError("truncated-payload", f"tensor {name} is cut short")
            if name.endswith("k_cache_scale") or name.endswith("v_cache_scale"):
                rep.unused.append(name)       # this build keeps an f32 KV cache (parity mode)
                continue
            scalar = read_scalar_tensor(t.dtype, t.element_count, raw)
            if scalar is not None and not name.endswith(".weight"):
                ctx.set_scalar(name, scalar)
                rep.scalars[name] = scalar
                continue
            if name.endswith("weight_scale") or name.endswith("embedding_scale"):
                if t.dtype == "F32":
                    s32 = np.frombuffer(raw, np.float32)
                    s16 = s32.astype(np.float16)
                    changed = int(np.count_nonzero(s16.astype(np.float32) != s32))
                    if changed and scale_policy == "exact":
                        raise SafetensorsError("scale-precision", f"{name}: {changed} row scales are not "
                                                                  f"f16 values (f16 row-scale storage)")
                    rep.scales_rounded += changed
                    data = s16.view(np.uint8)
                elif t.dtype == "F16":
                    data = np.frombuffer(raw, np.uint8)
                else:
                    raise SafetensorsError("bad-dtype", f"{name}: row scales as {t.dtype}")
            elif t.dtype == "BF16" and "per_layer_model_projection" not in name:
                data = _bf16_to_f32(raw).view(np.uint8)        # norm gains widen to f32
            else:
                data = np.frombuffer(raw, np.uint8)
            total = data.nbytes
            for off in range(0, total, PIECE_BYTES):
                ctx.upload(name, data[off:off + PIECE_BYTES], off, total)
            rep.uploaded.append(name)
    return rep


def export_checkpoint(ctx, path, num_hidden_layers: int, num_kv_shared_layers: int,
                      scalar_names=None) -> int:
    """Write a context's text tensors as a safetensors file in the checkpoint's own storage (U8 /
    I8 codes, F32 row scales, BF16 norm gains and per-layer model projection, one-element F32
    scalars, the tied lm_head pair left out as the checkpoint's download leaves it). Returns the
    file's byte length. The inverse of load_checkpoint for this build's storage."""
    names = text_tensor_names(num_hidden_layers, num_kv_shared_layers)
    blobs = []
    for name in names:
        if name.endswith("k_cache_scale") or name.endswith("v_cache_scale"):
            blobs.append((name, "F32", [1], np.ones(1, np.float32).tobytes()))
            continue
        if (name.endswith("activation_scale") or name.endswith("layer_scalar")):
            blobs.append((name, "F32", [1], np.array([ctx.scalar(name)], np.float32).tobytes()))
            continue
        raw = ctx.download(name)
        if name.endswith("weight_scale") or name.endswith("embedding_scale"):
            v = raw.view(np.float16).astype(np.float32)
            blobs.append((name, "F32", [v.size], v.tobytes()))
        elif name.endswith("norm.weight") or name.endswith("layernorm.weight"):
            b = _f32_to_bf16(raw.view(np.float32))
            blobs.append((name, "BF16", [b.size], b.tobytes()))
        elif name.endswith("per_layer_model_projection.weight"):
            blobs.append((name, "BF16", [raw.size // 2], raw.tobytes()))
        elif "per_layer_input_gate" in name or "per_layer_projection" in name:
            blobs.append((name, "I8", [raw.size], raw.tobytes()))
        else:
            blobs.append((name, "U8", [raw.size], raw.tobytes()))
    header, off = {}, 0
    for name, dtype, shape, data in blobs:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(data)]}
        off += len(data)
    header["__metadata__"] = {"format": "pt", "writer": "gemma4_webgpu_engine_b200.loader"}
    hjson = json.dumps(header, separators=(",", ":")).encode()
    hjson += b" " * ((8 - len(hjson) % 8) % 8)
    with Path(path).open("wb") as f:
        f.write(struct.pack("<Q", len(hjson)))
        f.write(hjson)
        for _, _, _, data in blobs:
            f.write(data)
    return 8 + len(hjson) + off
