"""The host API over libgemma4_cuda.so, mirroring the reference's Gemma4Mobile and
ForwardExecutor (src/engine.ts:289-927, src/runtime.ts:73-88).

`CudaExecutor` is the ForwardExecutor seam: prefill / decode / decodeAhead each call one C-ABI
entry point. `Gemma4Mobile` keeps the reference's load / generate / reset / dispose shape, with a
seeded synthetic model standing in for the checkpoint download (no network here).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _abi
from .plan import (GEMMA4_E2B, KvCacheState, LookupDrafter, SpeculationStats, prefill_chunks,
                   run_greedy_loop, run_speculative_loop)


class Context:
    """One libgemma4_cuda context on one GPU (owns weights, KV caches, graphs)."""

    def __init__(self, device: int = 0, max_seqs: int = 1, max_context: int = 2048,
                 max_step_columns: int = 64, use_graphs: bool = True, ple_slice_bytes: int = 0,
                 arch: _abi.Arch | None = None, gemm_min_columns: int = 16,
                 gemm_split_k: int = 0, gemm_shadow_min_columns: int = 0):
        lib = _abi.load()
        cfg = _abi.config_default()
        if arch is not None:
            cfg.arch = arch
        cfg.max_seqs = max_seqs
        cfg.max_context = max_context
        cfg.max_step_columns = max_step_columns
        cfg.use_graphs = 1 if use_graphs else 0
        cfg.ple_slice_bytes = ple_slice_bytes
        cfg.gemm_min_columns = gemm_min_columns
        cfg.gemm_split_k = gemm_split_k
        cfg.gemm_shadow_min_columns = gemm_shadow_min_columns
        h = C.c_void_p()
        _abi.check(lib.g4_ctx_create(device, C.byref(cfg), C.byref(h)))
        self.lib = lib
        self.h = h
        self.cfg = cfg
        self.vocab = cfg.arch.vocab_size

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.g4_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _check(self, rc: int) -> None:
        _abi.check(rc, self.h)

    # weights
    def init_random(self, seed: int) -> None:
        self._check(self.lib.g4_init_random(self.h, seed))

    def upload(self, name: str, data: bytes | np.ndarray, offset: int = 0, total: int | None = None):
        buf = np.ascontiguousarray(np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray)) else data.view(np.uint8).reshape(-1))
        total = buf.nbytes + offset if total is None else total
        self._check(self.lib.g4_upload_weight(self.h, name.encode(), buf.ctypes.data, offset,
                                              buf.nbytes, total))

    def download(self, name: str) -> np.ndarray:
        n = C.c_uint64(0)
        self._check(self.lib.g4_download_weight(self.h, name.encode(), None, C.byref(n)))
        out = np.zeros(n.value, np.uint8)
        self._check(self.lib.g4_download_weight(self.h, name.encode(), out.ctypes.data, C.byref(n)))
        return out

    def set_scalar(self, name: str, value: float) -> None:
        self._check(self.lib.g4_set_scalar(self.h, name.encode(), value))

    def scalar(self, name: str) -> float:
        v = C.c_float()
        self._check(self.lib.g4_get_scalar(self.h, name.encode(), C.byref(v)))
        return v.value

    def memory(self):
        w, k, o = C.c_uint64(), C.c_uint64(), C.c_uint64()
        self._check(self.lib.g4_ctx_memory(self.h, C.byref(w), C.byref(k), C.byref(o)))
        return w.value, k.value, o.value

    def ple_slices(self) -> tuple[int, int, int]:
        """(slices, rows per slice, rows of the last slice) of the PLE code table."""
        n, rps, last = C.c_int32(), C.c_int32(), C.c_int32()
        self._check(self.lib.g4_ctx_ple_slices(self.h, C.byref(n), C.byref(rps), C.byref(last)))
        return n.value, rps.value, last.value

    # forward
    def prefill(self, seq: int, ids, start: int, is_last: bool) -> int:
        ids = np.ascontiguousarray(ids, np.int32)
        tok = C.c_int32(-1)
        self._check(self.lib.g4_prefill(self.h, seq, _abi.i32p(ids), ids.size, start,
                                        1 if is_last else 0, C.byref(tok)))
        return tok.value

    def decode(self, seq: int, prev: int, pos: int) -> int:
        tok = C.c_int32(-1)
        self._check(self.lib.g4_decode(self.h, seq, prev, pos, C.byref(tok)))
        return tok.value

    def decode_ahead(self, seq: int, pos: int) -> int:
        tok = C.c_int32(-1)
        self._check(self.lib.g4_decode_ahead(self.h, seq, pos, C.byref(tok)))
        return tok.value

    def verify(self, seq: int, tokens, pos: int) -> list:
        tokens = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(tokens.size, np.int32)
        self._check(self.lib.g4_verify(self.h, seq, _abi.i32p(tokens), tokens.size, pos, _abi.i32p(out)))
        return [int(t) for t in out]

    def decode_batch(self, seqs, tokens, positions) -> np.ndarray:
        seqs = np.ascontiguousarray(seqs, np.int32)
        tokens = np.ascontiguousarray(tokens, np.int32)
        positions = np.ascontiguousarray(positions, np.int32)
        out = np.zeros(seqs.size, np.int32)
        self._check(self.lib.g4_decode_batch(self.h, seqs.size, _abi.i32p(seqs), _abi.i32p(tokens),
                                             _abi.i32p(positions), _abi.i32p(out)))
        return out

    def step_stage(self, seqs, tokens, positions) -> None:
        seqs = np.ascontiguousarray(seqs, np.int32)
        tokens = np.ascontiguousarray(tokens, np.int32)
        positions = np.ascontiguousarray(positions, np.int32)
        self._check(self.lib.g4_step_stage(self.h, seqs.size, _abi.i32p(seqs), _abi.i32p(tokens),
                                           _abi.i32p(positions)))

    def step_run_device(self, B: int) -> None:
        self._check(self.lib.g4_step_run_device(self.h, B, 1))

    def step_read_tokens(self, B: int) -> np.ndarray:
        out = np.zeros(B, np.int32)
        self._check(self.lib.g4_step_read_tokens(self.h, B, _abi.i32p(out)))
        return out

    def kv_truncate(self, seq: int, n: int) -> None:
        self._check(self.lib.g4_kv_truncate(self.h, seq, n))

    def kv_length(self, seq: int) -> int:
        n = C.c_int32()
        self._check(self.lib.g4_kv_length(self.h, seq, C.byref(n)))
        return n.value

    def logits(self, col: int = 0, n: int | None = None) -> np.ndarray:
        n = self.vocab if n is None else n
        out = np.zeros(n, np.float32)
        self._check(self.lib.g4_read_logits(self.h, col, out.ctypes.data_as(C.POINTER(C.c_float)), n))
        return out

    def launches(self) -> int:
        n = C.c_int32()
        self._check(self.lib.g4_last_launches(self.h, C.byref(n)))
        return n.value

    def launch_list(self) -> list:
        """(kernel, roles) of every launch of the last forward call, in launch order."""
        need = C.c_uint64(0)
        self._check(self.lib.g4_last_launch_list(self.h, None, 0, C.byref(need)))
        buf = C.create_string_buffer(need.value)
        self._check(self.lib.g4_last_launch_list(self.h, buf, need.value, C.byref(need)))
        return [tuple(line.split("\t", 1)) for line in buf.value.decode().splitlines()]

    def stream(self) -> int:
        return self.lib.g4_ctx_stream(self.h)


class CudaExecutor:
    """ForwardExecutor (src/runtime.ts:73-88) for one sequence slot of a Context."""

    def __init__(self, ctx: Context, seq: int = 0, max_chunk_tokens: int = 2048):
        self.ctx = ctx
        self.seq = seq
        self.max_chunk_tokens = max_chunk_tokens

    def prefill(self, tokens, start_position: int, is_last: bool) -> int:
        if len(tokens) == 0:
            return -1
        if len(tokens) > self.max_chunk_tokens:
            raise ValueError(f"gemma4 engine: a prefill chunk of {len(tokens)} exceeds the "
                             f"{self.max_chunk_tokens} this executor sized its slots for")
        return self.ctx.prefill(self.seq, tokens, start_position, is_last)

    def decode(self, prev_token: int, position: int) -> int:
        return self.ctx.decode(self.seq, prev_token, position)

    def decode_ahead(self, position: int) -> int:
        return self.ctx.decode_ahead(self.seq, position)

    def verify(self, tokens, position: int) -> list:
        """The verify pass (src/runtime.ts:993-1014): tokens[0] is the last chosen token,
        tokens[1:] a drafted continuation at `position` onward; answer[i] is the model's argmax
        after tokens[i], exactly the plain greedy decode's choice there."""
        if len(tokens) < 1:
            raise ValueError("gemma4 engine: a verify pass takes at least 1 token, got 0")
        return self.ctx.verify(self.seq, tokens, position)


class Gemma4Mobile:
    """Gemma4Mobile.load / generate / reset / dispose (src/engine.ts:289-927) over the CUDA
    executor. Token ids are the interface (the tokenizer is out of scope)."""

    def __init__(self, ctx: Context, seq: int = 0):
        self.ctx = ctx
        self.executor = CudaExecutor(ctx, seq)
        self.kv_state = KvCacheState()
        self.eos_ids = frozenset()

    @classmethod
    def load(cls, seed: int = 0x6E6D6134, device: int = 0, max_context: int = 2048,
             **ctx_kwargs) -> "Gemma4Mobile":
        ctx = Context(device=device, max_context=max_context, **ctx_kwargs)
        ctx.init_random(seed)
        return cls(ctx)

    def generate(self, prompt_ids, max_new_tokens: int = 16, eos_ids=None, lookahead: bool = True,
                 is_aborted=lambda: False, speculate: bool = False, max_columns: int = 2,
                 drafter=None, stats: SpeculationStats | None = None):
        """Greedy generation; yields token ids. Reuses the KV prefix of the previous call. With
        `speculate`, passes verify a prompt-lookup draft of up to max_columns - 1 tokens
        (src/engine.ts:660-707, src/draft.ts): the ids are the same, only the pass count
        changes."""
        prompt = [int(t) for t in prompt_ids]
        eos = frozenset(eos_ids) if eos_ids is not None else self.eos_ids
        plan = self.kv_state.accept_prompt(prompt)
        self.ctx.kv_truncate(self.executor.seq, plan.reuse)
        chunks = prefill_chunks(plan.prefill_from, len(prompt), chunk_size=min(
            2048, self.ctx.cfg.max_step_columns))
        first = -1
        for i, ch in enumerate(chunks):
            last = i == len(chunks) - 1
            first = self.executor.prefill(prompt[ch.start:ch.end], ch.start, last)
            self.kv_state.append(prompt[ch.start:ch.end])
        start = len(prompt)
        if speculate:
            for token, index in run_speculative_loop(
                    first, max_new_tokens, eos, start, prompt, max_columns,
                    drafter or LookupDrafter(), self.executor.decode, self.executor.verify,
                    is_aborted, on_advance=lambda t, p: self.kv_state.append([t]), stats=stats):
                yield token
            self.ctx.kv_truncate(self.executor.seq, self.kv_state.length)
            return
        for token, index in run_greedy_loop(
                first, max_new_tokens, eos, start, self.executor.decode, is_aborted,
                decode_ahead=self.executor.decode_ahead if lookahead else None):
            if index > 0:
                self.kv_state.append([prev])
            prev = token
            yield token

    def reset(self) -> None:
        self.kv_state.reset()
        self.ctx.kv_truncate(self.executor.seq, 0)

    def dispose(self) -> None:
        self.ctx.close()
