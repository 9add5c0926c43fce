"""ctypes binding of the CPU oracle (oracle/_build/libg4oracle.so).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline. Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / reference arms import this module. The
product library never loads it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libg4oracle.so"

_lib = None


def build() -> Path:
    """Compile the oracle (gcc; see oracle/Makefile)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def _f(a):
    return a.ctypes.data_as(C.POINTER(C.c_float)) if a is not None else None


def _i(a):
    return a.ctypes.data_as(C.POINTER(C.c_int32)) if a is not None else None


def _u8(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint8))


def _u16(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint16))


class Arch(C.Structure):
    _fields_ = [
        ("layer_count", C.c_int32), ("hidden", C.c_int32), ("q_heads", C.c_int32),
        ("sliding_hd", C.c_int32), ("global_hd", C.c_int32), ("global_mask", C.c_uint64),
        ("window", C.c_int32), ("producers", C.c_int32), ("ffn", C.c_int32),
        ("vocab", C.c_int32), ("ple_dim", C.c_int32), ("eps", C.c_float),
        ("softcap", C.c_float), ("theta_sliding", C.c_float), ("theta_global", C.c_float),
        ("partial_rotary", C.c_float), ("consumer_ffn", C.c_int32),
        ("consumer_mlp_bits", C.c_int32), ("head_bits", C.c_int32), ("head_calibrated", C.c_int32),
    ]


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        fp, ip, vp = C.POINTER(C.c_float), C.POINTER(C.c_int32), C.c_void_p
        u8p, u16p = C.POINTER(C.c_uint8), C.POINTER(C.c_uint16)
        L.g4o_exp.restype = C.c_float
        L.g4o_exp.argtypes = [C.c_float]
        L.g4o_tanh.restype = C.c_float
        L.g4o_tanh.argtypes = [C.c_float]
        L.g4o_gelu.restype = C.c_float
        L.g4o_gelu.argtypes = [C.c_float]
        L.g4o_srq_code.restype = C.c_int
        L.g4o_srq_code.argtypes = [C.c_float, C.c_float]
        L.g4o_srq_out.restype = C.c_float
        L.g4o_srq_out.argtypes = [C.c_float, C.c_float]
        L.g4o_f32_to_f16.restype = C.c_uint16
        L.g4o_f32_to_f16.argtypes = [C.c_float]
        L.g4o_f16_to_f32.restype = C.c_float
        L.g4o_f16_to_f32.argtypes = [C.c_uint16]
        L.g4o_hash.restype = C.c_uint64
        L.g4o_hash.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
        L.g4o_qgemv.argtypes = [u8p, u16p, fp, C.c_float, C.c_float, C.c_int, C.c_int, C.c_int,
                                C.c_int, fp, ip]
        L.g4o_gelu_mul.argtypes = [fp, fp, fp, C.c_int, C.c_float]
        L.g4o_rms_inv.restype = C.c_float
        L.g4o_rms_inv.argtypes = [fp, C.c_int, C.c_float]
        L.g4o_rms_norm.argtypes = [fp, fp, fp, C.c_int, C.c_int, C.c_float]
        L.g4o_norm_residual.argtypes = [fp, fp, fp, fp, C.c_int, C.c_int, C.c_float]
        L.g4o_norm_residual_norm.argtypes = [fp, fp, fp, fp, C.c_float, fp, fp, C.c_int, C.c_int,
                                             C.c_float]
        L.g4o_rope_tables.argtypes = [C.c_int, C.c_int, C.c_double, C.c_int, C.c_int, fp, fp]
        L.g4o_q_norm_rope.argtypes = [fp, fp, fp, fp, fp, C.c_int, C.c_int, C.c_int, C.c_float]
        L.g4o_kv_norm_rope_store.argtypes = [fp, fp, fp, fp, fp, fp, C.c_int, C.c_int, C.c_int,
                                             C.c_int, C.c_float]
        L.g4o_attention.argtypes = [fp, fp, fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int]
        L.g4o_embed_gather.argtypes = [u8p, u16p, ip, fp, C.c_int, C.c_int, C.c_int, C.c_float,
                                       C.c_int, C.c_int]
        L.g4o_dense_bf16.argtypes = [u16p, fp, fp, C.c_int, C.c_int, C.c_int, C.c_float]
        L.g4o_softcap_argmax.argtypes = [fp, fp, ip, C.c_int, C.c_float]
        L.g4o_ref_rms_norm.argtypes = [fp, fp, fp, C.c_int, C.c_int, C.c_float]
        L.g4o_ref_norm_residual.argtypes = [fp, fp, fp, fp, C.c_int, C.c_int, C.c_float]
        L.g4o_ref_attention.argtypes = [fp, fp, fp, fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_double]
        L.g4o_ref_gelu_mul.argtypes = [fp, fp, fp, C.c_int, C.c_float]
        L.g4o_ref_dense.argtypes = [fp, fp, fp, C.c_int, C.c_int, C.c_int, C.c_float]
        L.g4o_plan_table_split.restype = C.c_int
        L.g4o_plan_table_split.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, ip, ip,
                                           ip]
        L.g4o_arch_default.argtypes = [C.POINTER(Arch)]
        L.g4o_model_synth.restype = vp
        L.g4o_model_synth.argtypes = [C.POINTER(Arch), C.c_uint64]
        L.g4o_model_free.argtypes = [vp]
        L.g4o_model_tensor.restype = vp
        L.g4o_model_tensor.argtypes = [vp, C.c_char_p, C.POINTER(C.c_uint64)]
        L.g4o_model_scalar.restype = C.c_float
        L.g4o_model_scalar.argtypes = [vp, C.c_char_p]
        L.g4o_seq_new.restype = vp
        L.g4o_seq_new.argtypes = [vp, C.c_int32]
        L.g4o_seq_free.argtypes = [vp]
        L.g4o_forward.restype = C.c_int
        L.g4o_forward.argtypes = [vp, vp, ip, C.c_int32, C.c_int32, C.c_int32, C.c_int32, ip, fp,
                                  fp]
        L.g4o_generate.restype = C.c_int
        L.g4o_generate.argtypes = [vp, ip, C.c_int32, C.c_int32, C.c_int32, ip, fp]
        L.g4o_synth_prompt.argtypes = [C.c_uint64, C.c_int32, C.c_int32, ip]
        L.g4o_site_stats.argtypes = [fp, fp, C.c_int32]
        L.g4o_threads.argtypes = [C.c_int32]
        _lib = L
    return _lib


def threads(n: int) -> None:
    lib().g4o_threads(int(n))


# ---------------------------------------------------------------- per-kernel helpers

def qgemv(wq: np.ndarray, scales_f16: np.ndarray, x: np.ndarray, in_scale: float,
          out_scale: float, bits: int, N: int, K: int, cols: int = 1):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(cols, K)
    y = np.zeros((cols, N), np.float32)
    acc = np.zeros((cols, N), np.int32)
    lib().g4o_qgemv(_u8(np.ascontiguousarray(wq, dtype=np.uint8)),
                    _u16(np.ascontiguousarray(scales_f16, dtype=np.uint16)), _f(x),
                    in_scale, out_scale, bits, N, K, cols, _f(y), _i(acc))
    return y, acc


def rms_norm(src, gain, rows, width, eps=1e-6, ref=False):
    src = np.ascontiguousarray(src, np.float32)
    dst = np.zeros(rows * width, np.float32)
    g = np.ascontiguousarray(gain, np.float32) if gain is not None else None
    fn = lib().g4o_ref_rms_norm if ref else lib().g4o_rms_norm
    fn(_f(src), _f(g), _f(dst), rows, width, eps)
    return dst


def norm_residual(src, gain, residual, rows, width, eps=1e-6, ref=False):
    dst = np.zeros(rows * width, np.float32)
    fn = lib().g4o_ref_norm_residual if ref else lib().g4o_norm_residual
    fn(_f(np.ascontiguousarray(src, np.float32)), _f(np.ascontiguousarray(gain, np.float32)),
       _f(np.ascontiguousarray(residual, np.float32)), _f(dst), rows, width, eps)
    return dst


def norm_residual_norm(src, gain, residual, gain2, alpha, rows, width, eps=1e-6):
    hidden = np.zeros(rows * width, np.float32)
    dst = np.zeros(rows * width, np.float32)
    lib().g4o_norm_residual_norm(
        _f(np.ascontiguousarray(src, np.float32)), _f(np.ascontiguousarray(gain, np.float32)),
        _f(np.ascontiguousarray(residual, np.float32)),
        _f(np.ascontiguousarray(gain2, np.float32)), alpha, _f(hidden), _f(dst), rows, width,
        eps)
    return hidden, dst


def gelu_mul(gate, up, srq_scale=0.0, ref=False):
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    dst = np.zeros_like(gate)
    fn = lib().g4o_ref_gelu_mul if ref else lib().g4o_gelu_mul
    fn(_f(gate), _f(up), _f(dst), gate.size, srq_scale)
    return dst


def rope_tables(head_dim, rotary_pairs, theta, pos0, npos):
    pairs = head_dim // 2
    c = np.zeros(npos * pairs, np.float32)
    s = np.zeros(npos * pairs, np.float32)
    lib().g4o_rope_tables(head_dim, rotary_pairs, theta, pos0, npos, _f(c), _f(s))
    return c, s


def q_norm_rope(src, gain, cos_t, sin_t, rows, width, rows_per_pos, eps=1e-6):
    dst = np.zeros(rows * width, np.float32)
    lib().g4o_q_norm_rope(_f(np.ascontiguousarray(src, np.float32)),
                          _f(np.ascontiguousarray(gain, np.float32)), _f(cos_t), _f(sin_t),
                          _f(dst), rows, width, rows_per_pos, eps)
    return dst


def kv_norm_rope_store(k, v, gain, cos_t, sin_t, cache, tokens, head_dim, start_pos,
                       max_context, eps=1e-6):
    lib().g4o_kv_norm_rope_store(_f(np.ascontiguousarray(k, np.float32)),
                                 _f(np.ascontiguousarray(v, np.float32)),
                                 _f(np.ascontiguousarray(gain, np.float32)), _f(cos_t),
                                 _f(sin_t), _f(cache), tokens, head_dim, start_pos, max_context,
                                 eps)
    return cache


def attention(q, cache, heads, head_dim, q_count, q_start, kv_len, window, max_context):
    out = np.zeros(q_count * heads * head_dim, np.float32)
    lib().g4o_attention(_f(np.ascontiguousarray(q, np.float32)),
                        _f(np.ascontiguousarray(cache, np.float32)), _f(out), heads, head_dim,
                        q_count, q_start, kv_len, window, max_context)
    return out


def ref_attention(q, k, v, heads, head_dim, q_count, q_start, kv_len, window, scale=1.0):
    out = np.zeros(q_count * heads * head_dim, np.float32)
    lib().g4o_ref_attention(_f(np.ascontiguousarray(q, np.float32)),
                            _f(np.ascontiguousarray(k, np.float32)),
                            _f(np.ascontiguousarray(v, np.float32)), _f(out), heads, head_dim,
                            q_count, q_start, kv_len, window, scale)
    return out


def embed_gather(codes, scales_f16, ids, cols, group_size, out_scale, slice_start=0,
                 slice_rows=0, dst=None):
    ids = np.ascontiguousarray(ids, np.int32)
    if dst is None:
        dst = np.zeros(ids.size * cols, np.float32)
    lib().g4o_embed_gather(_u8(np.ascontiguousarray(codes, np.uint8)),
                           _u16(np.ascontiguousarray(scales_f16, np.uint16)), _i(ids), _f(dst),
                           ids.size, cols, group_size, out_scale, slice_start, slice_rows)
    return dst


def dense_bf16(w_bf16, x, N, K, cols, alpha):
    y = np.zeros(cols * N, np.float32)
    lib().g4o_dense_bf16(_u16(np.ascontiguousarray(w_bf16, np.uint16)),
                         _f(np.ascontiguousarray(x, np.float32)), _f(y), N, K, cols, alpha)
    return y


def softcap_argmax(logits, cap=30.0):
    logits = np.ascontiguousarray(logits, np.float32)
    capped = np.zeros_like(logits)
    tok = np.zeros(2, np.int32)
    lib().g4o_softcap_argmax(_f(logits), _f(capped), _i(tok), logits.size, cap)
    return capped, int(tok[0])


def plan_table_split(rows, row_bytes, limit_bytes, slice_bytes):
    n = C.c_int32()
    per = C.c_int32()
    last = C.c_int32()
    rc = lib().g4o_plan_table_split(rows, row_bytes, limit_bytes, slice_bytes, C.byref(n),
                                    C.byref(per), C.byref(last))
    if rc != 0:
        return None
    return n.value, per.value, last.value


def arch_default() -> Arch:
    a = Arch()
    lib().g4o_arch_default(C.byref(a))
    return a


class Model:
    """The seeded synthetic model on the host (about 2.2 GB at the full architecture)."""

    def __init__(self, seed: int, arch: Arch | None = None):
        self.arch = arch or arch_default()
        self.ptr = lib().g4o_model_synth(C.byref(self.arch), seed)
        self.seed = seed

    def close(self):
        if self.ptr:
            lib().g4o_model_free(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()

    def tensor(self, name: str) -> np.ndarray:
        n = C.c_uint64()
        p = lib().g4o_model_tensor(self.ptr, name.encode(), C.byref(n))
        if not p:
            raise KeyError(name)
        return np.ctypeslib.as_array((C.c_uint8 * n.value).from_address(p)).copy()

    def scalar(self, name: str) -> float:
        return float(lib().g4o_model_scalar(self.ptr, name.encode()))

    def generate(self, prompt, max_new: int, max_context: int):
        prompt = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(max_new, np.int32)
        gaps = np.zeros(max_new, np.float32)
        rc = lib().g4o_generate(self.ptr, _i(prompt), prompt.size, max_new, max_context,
                                _i(toks), _f(gaps))
        if rc != 0:
            raise RuntimeError("g4o_generate failed")
        return toks, gaps


class Sequence:
    def __init__(self, model: Model, max_context: int):
        self.model = model
        self.ptr = lib().g4o_seq_new(model.ptr, max_context)

    def __del__(self):
        if getattr(self, "ptr", None):
            lib().g4o_seq_free(self.ptr)
            self.ptr = None

    def forward(self, ids, start_pos: int, all_layers: bool, want_head: bool,
                want_logits: bool = False):
        ids = np.ascontiguousarray(ids, np.int32)
        tok = np.zeros(1, np.int32)
        top2 = np.zeros(4, np.float32)
        logits = np.zeros(self.model.arch.vocab, np.float32) if want_logits else None
        rc = lib().g4o_forward(self.model.ptr, self.ptr, _i(ids), ids.size, start_pos,
                               int(all_layers), int(want_head), _i(tok), _f(logits), _f(top2))
        if rc != 0:
            raise RuntimeError("g4o_forward failed")
        return int(tok[0]), logits, top2


def synth_prompt(seed: int, n: int, vocab: int = 262144) -> np.ndarray:
    ids = np.zeros(n, np.int32)
    lib().g4o_synth_prompt(seed, n, vocab, _i(ids))
    return ids


def site_stats():
    mi = np.zeros(10, np.float32)
    mo = np.zeros(10, np.float32)
    lib().g4o_site_stats(_f(mi), _f(mo), 10)
    return mi, mo


SITES = ["q", "k", "v", "o", "gate", "up", "down", "ple_gate", "ple_proj", "lm_head"]


def n_threads_default() -> int:
    return len(os.sched_getaffinity(0))
