"""ctypes binding of include/g4.h (libgemma4_cuda.so).

This is the Python twin of the N-API addon a TypeScript host would bind: every
declaration of g4.h, with status codes turned into exceptions that carry g4_last_error's text.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libgemma4_cuda.so"

G4_OK = 0
ERRORS = {
    -1: "G4_ERR_INVALID", -2: "G4_ERR_CUDA", -3: "G4_ERR_OOM", -4: "G4_ERR_STATE",
    -5: "G4_ERR_UNSUPPORTED", -6: "G4_ERR_NOT_FOUND", -7: "G4_ERR_TIMEOUT",
}


class G4Error(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERRORS.get(code, code)}: {message}")
        self.code = code


class Arch(C.Structure):
    _fields_ = [
        ("layer_count", C.c_int32), ("hidden_size", C.c_int32), ("query_heads", C.c_int32),
        ("kv_heads", C.c_int32), ("sliding_head_dim", C.c_int32), ("global_head_dim", C.c_int32),
        ("global_layer_mask", C.c_uint64), ("sliding_window", C.c_int32),
        ("kv_producer_layers", C.c_int32), ("producer_intermediate", C.c_int32),
        ("consumer_intermediate", C.c_int32), ("vocab_size", C.c_int32), ("ple_dim", C.c_int32),
        ("attn_bits", C.c_int32), ("mlp_bits", C.c_int32), ("ple_bits", C.c_int32),
        ("consumer_mlp_bits", C.c_int32), ("head_bits", C.c_int32), ("head_calibrated", C.c_int32),
        ("rms_eps", C.c_float), ("final_softcap", C.c_float), ("rope_theta_sliding", C.c_float),
        ("rope_theta_global", C.c_float), ("partial_rotary_factor", C.c_float),
    ]


class Config(C.Structure):
    _fields_ = [
        ("arch", Arch), ("max_seqs", C.c_int32), ("max_context", C.c_int32),
        ("max_step_columns", C.c_int32), ("use_graphs", C.c_int32),
        ("ple_slice_bytes", C.c_uint64), ("gemm_min_columns", C.c_int32),
        ("gemm_shadow_min_columns", C.c_int32), ("gemm_split_k", C.c_int32),
    ]


# Every exported symbol of include/g4.h with its ctypes signature (restype, argtypes).
_vp, _i32, _u64, _f = C.c_void_p, C.c_int32, C.c_uint64, C.c_float
_i32p, _u64p, _fp = C.POINTER(C.c_int32), C.POINTER(C.c_uint64), C.POINTER(C.c_float)
SIGNATURES = {
    "g4_last_error": (C.c_char_p, [_vp]),
    "g4_version": (C.c_char_p, []),
    "g4_arch_default": (C.c_int, [C.POINTER(Arch)]),
    "g4_config_default": (C.c_int, [C.POINTER(Config)]),
    "g4_ctx_create": (C.c_int, [C.c_int, C.POINTER(Config), C.POINTER(_vp)]),
    "g4_ctx_destroy": (None, [_vp]),
    "g4_ctx_memory": (C.c_int, [_vp, _u64p, _u64p, _u64p]),
    "g4_ctx_ple_slices": (C.c_int, [_vp, _i32p, _i32p, _i32p]),
    "g4_init_random": (C.c_int, [_vp, _u64]),
    "g4_upload_weight": (C.c_int, [_vp, C.c_char_p, _vp, _u64, _u64, _u64]),
    "g4_download_weight": (C.c_int, [_vp, C.c_char_p, _vp, _u64p]),
    "g4_set_scalar": (C.c_int, [_vp, C.c_char_p, _f]),
    "g4_get_scalar": (C.c_int, [_vp, C.c_char_p, _fp]),
    "g4_plan_table_split": (C.c_int, [_u64, _u64, _u64, _u64, _i32p, _i32p, _i32p]),
    "g4_prefill": (C.c_int, [_vp, _i32, _i32p, _i32, _i32, _i32, _i32p]),
    "g4_decode": (C.c_int, [_vp, _i32, _i32, _i32, _i32p]),
    "g4_decode_ahead": (C.c_int, [_vp, _i32, _i32, _i32p]),
    "g4_decode_batch": (C.c_int, [_vp, _i32, _i32p, _i32p, _i32p, _i32p]),
    "g4_verify": (C.c_int, [_vp, _i32, _i32p, _i32, _i32, _i32p]),
    "g4_op_wait_probe": (C.c_int, [_vp, _i32, _i32, _i32, _vp, _vp]),
    "g4_op_repack_tile16": (C.c_int, [_vp, _vp, _i32, _i32, _i32, _vp]),
    "g4_arch_checkpoint": (C.c_int, [C.POINTER(Arch)]),
    "g4_debug_fail_allocation": (C.c_int, [_i32]),
    "g4_debug_raise_error_flag": (C.c_int, [_vp, _i32]),
    "g4_step_stage": (C.c_int, [_vp, _i32, _i32p, _i32p, _i32p]),
    "g4_step_run_device": (C.c_int, [_vp, _i32, _i32]),
    "g4_step_read_tokens": (C.c_int, [_vp, _i32, _i32p]),
    "g4_kv_truncate": (C.c_int, [_vp, _i32, _i32]),
    "g4_kv_length": (C.c_int, [_vp, _i32, _i32p]),
    "g4_read_logits": (C.c_int, [_vp, _i32, _fp, _i32]),
    "g4_ctx_stream": (_vp, [_vp]),
    "g4_last_launches": (C.c_int, [_vp, _i32p]),
    "g4_last_launch_list": (C.c_int, [_vp, C.c_char_p, _u64, _u64p]),
    "g4_op_qgemv": (C.c_int, [_vp, _vp, _vp, _f, _f, _i32, _i32, _i32, _i32, _vp, _vp, _vp]),
    "g4_op_qgemv_codes": (C.c_int, [_vp, _vp, _vp, _f, _f, _i32, _i32, _i32, _i32, _vp, _vp, _vp]),
    "g4_op_qgemm": (C.c_int, [_vp, _vp, _vp, _f, _f, _i32, _i32, _i32, _i32, _vp, _vp]),
    "g4_op_qgemv_gelu": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _f, _f, _i32, _i32, _i32, _i32,
                                   _vp, _vp]),
    "g4_op_rms_norm": (C.c_int, [_vp, _vp, _vp, _i32, _i32, _f, _vp]),
    "g4_op_norm_residual": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _f, _vp]),
    "g4_op_norm_residual_norm": (C.c_int, [_vp, _vp, _vp, _vp, _f, _vp, _vp, _i32, _i32, _f,
                                           _vp]),
    "g4_op_gelu_mul": (C.c_int, [_vp, _vp, _vp, _i32, _f, _vp]),
    "g4_op_q_norm_rope": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _f, _vp]),
    "g4_op_kv_norm_rope_store": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                           _f, _vp]),
    "g4_op_attention": (C.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp]),
    "g4_op_attention_prefill": (C.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp]),
    "g4_op_attention_noalloc": (C.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                          _vp]),
    "g4_op_embed_gather": (C.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _f, _i32, _i32, _vp]),
    "g4_op_dense_bf16": (C.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _f, _vp]),
    "g4_op_softcap_argmax": (C.c_int, [_vp, _vp, _vp, _i32, _f, _vp]),
    "g4_op_math_probe": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _vp]),
}

_lib = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load libgemma4_cuda.so. There is no fallback: a missing library is an error."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(
            f"{p} is missing: build it with __graft_entry__.build() (nvcc, sm_100a). "
            "The engine has no CPU path.")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error(ctx=None) -> str:
    return load().g4_last_error(ctx).decode(errors="replace")


def check(rc: int, ctx=None) -> None:
    if rc != G4_OK:
        raise G4Error(rc, last_error(ctx))


def arch_default() -> Arch:
    a = Arch()
    check(load().g4_arch_default(C.byref(a)))
    return a


def config_default() -> Config:
    c = Config()
    check(load().g4_config_default(C.byref(c)))
    return c


def plan_table_split(rows: int, row_bytes: int, limit_bytes: int, slice_bytes: int):
    n, per, last = C.c_int32(), C.c_int32(), C.c_int32()
    check(load().g4_plan_table_split(rows, row_bytes, limit_bytes, slice_bytes, C.byref(n),
                                     C.byref(per), C.byref(last)))
    return n.value, per.value, last.value


def i32p(a):
    return a.ctypes.data_as(_i32p)


def ptr(x) -> int:
    """Device pointer of a torch tensor (or None)."""
    return None if x is None else x.data_ptr()
