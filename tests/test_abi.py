"""The C-ABI library loads, exports every symbol include/g4.h declares, and reports errors on
the host paths that need no GPU."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_symbols():
    text = (ROOT / "include" / "g4.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(g4_[a-z0-9_]+)\s*\(", text)))


def test_header_lists_entry_points():
    syms = header_symbols()
    assert "g4_decode" in syms and "g4_op_qgemv" in syms and len(syms) >= 35


def test_library_exports_every_symbol(lib):
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_header(pkg):
    assert set(header_symbols()) <= set(pkg._abi.SIGNATURES)


def test_defaults_and_version(pkg, lib):
    cfg = pkg._abi.config_default()
    a = cfg.arch
    assert (a.layer_count, a.hidden_size, a.query_heads, a.vocab_size) == (35, 1536, 8, 262144)
    assert a.global_layer_mask == sum(1 << l for l in (4, 9, 14, 19, 24, 29, 34))
    assert cfg.max_context == 2048 and cfg.use_graphs == 1
    assert lib.g4_version().startswith(b"gemma4_cuda")


def test_errors_without_gpu(pkg, lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("host-only error paths")
    h = C.c_void_p()
    rc = lib.g4_ctx_create(0, None, C.byref(h))
    assert rc == -2 and not h.value
    assert "not available" in pkg._abi.last_error()
    assert lib.g4_ctx_create(0, None, None) == -1
    with pytest.raises(pkg.G4Error):
        pkg._abi.plan_table_split(10, 1000, 100, 100)
    # Invalid arguments to operators are refused before any device work.
    assert lib.g4_op_qgemv(None, None, None, 0.0, 0.0, 4, 8, 512, 1, None, None, None) == -1
    assert lib.g4_op_qgemv(1, 1, 1, 0.1, 0.0, 4, 8, 300, 1, 1, None, None) == -1
    assert "multiple of 256" in pkg._abi.last_error()
    assert lib.g4_op_attention(1, 1, 1, 8, 256, 1, 10, 5, 0, 64, None) == -1
    assert "store KV before attending" in pkg._abi.last_error()


def test_no_oracle_in_product():
    """The product sources never reference the oracle."""
    for p in list((ROOT / "gemma4-webgpu-engine_b200").rglob("*.py")) + \
            list((ROOT / "gemma4-webgpu-engine_b200" / "csrc").glob("*")):
        text = p.read_text()
        assert "oracle" not in text.replace("Oracle", ""), p
