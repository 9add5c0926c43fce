"""The critical-path trace tool's host logic (no GPU): record naming and per-kernel shares."""
from __future__ import annotations

import importlib.util
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
spec = importlib.util.spec_from_file_location("g4_trace_tool", ROOT / "gemma4-webgpu-engine_b200" / "trace.py")
T = importlib.util.module_from_spec(spec)
spec.loader.exec_module(T)


def test_kernel_names():
    assert T.kernel_name(1410) == "gemv int4 norm -> y [prologue]"
    assert T.kernel_name(101421) == "gemv int4 join -> gelu-codes [main loop]"
    assert T.kernel_name(201421) == "gemv int4 join -> gelu-codes [epilogue + release]"
    assert T.kernel_name(5411) == "gemm int4 64 tok, cluster split [block 0 main loop]"
    assert T.kernel_name(405801) == "gemm int8 64 tok [last CTA done -> next]"
    assert T.kernel_name(3001) == "embed"
    assert T.kernel_name(4002) == "quantize (join)"


def test_summarize_charges_each_interval_to_the_earlier_record():
    # Two steps, each: embed at t, a GEMV 2 us later whose main loop starts 3 us after that, the
    # next step's embed 10 us after t. Times are %globaltimer nanoseconds.
    rec = [(3001, 0), (1410, 2000), (101410, 5000), (3001, 10000), (1410, 12000), (101410, 15000),
           (3001, 20000)]
    agg = T.summarize(rec, steps=3)
    assert agg["embed"] == [2, 4.0]
    assert agg["gemv int4 norm -> y [prologue]"] == [2, 6.0]
    assert agg["gemv int4 norm -> y [main loop]"] == [2, 10.0]
