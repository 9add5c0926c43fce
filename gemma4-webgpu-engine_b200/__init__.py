"""gemma4-webgpu-engine for B200: the quantized decode/prefill hot path as sm_100a CUDA.

The product is libgemma4_cuda.so (csrc/, C ABI in include/g4.h). This package is its host side:
the ctypes binding (`_abi`), the reference's host interfaces (`engine`: Gemma4Mobile and the
ForwardExecutor seam; `plan`: prefill chunks, dispatch lists, KV reuse, table split;
`replicas`: the request split across one replica per GPU).
"""
from . import _abi, engine, loader, plan, replicas  # noqa: F401
from ._abi import G4Error, load  # noqa: F401

__all__ = ["G4Error", "load", "plan", "engine", "loader", "replicas"]
