"""Pure host-side planning, mirroring the reference's src/plan.ts, src/kv.ts and src/tableSplit.ts.

Nothing here touches a GPU. The C++ executor in libgemma4_cuda.so runs the same step order that
`plan_decode_step` lists; `census` lets a caller check a recorded step count against it.
"""
from __future__ import annotations

from dataclasses import dataclass, field

# ---------------------------------------------------------------- architecture (plan.ts:29-82)


@dataclass(frozen=True)
class Gemma4Arch:
    layer_count: int = 35
    hidden_size: int = 1536
    query_heads: int = 8
    kv_heads: int = 1
    sliding_head_dim: int = 256
    global_head_dim: int = 512
    global_layers: tuple = (4, 9, 14, 19, 24, 29, 34)
    sliding_window: int = 512
    kv_producer_layers: int = 15
    producer_intermediate: int = 6144
    consumer_intermediate: int = 6144  # the checkpoint's 12288 belongs to the 2-bit family
    vocab_size: int = 262144
    ple_dim: int = 256
    rms_eps: float = 1e-6
    final_softcap: float = 30.0
    rope_theta_sliding: float = 1e4
    rope_theta_global: float = 1e6
    partial_rotary_factor: float = 0.25


GEMMA4_E2B = Gemma4Arch()


def is_global_layer(arch: Gemma4Arch, layer: int) -> bool:
    return layer in arch.global_layers


def is_kv_producer(arch: Gemma4Arch, layer: int) -> bool:
    return 0 <= layer < arch.kv_producer_layers


def head_dim_for_layer(arch: Gemma4Arch, layer: int) -> int:
    return arch.global_head_dim if is_global_layer(arch, layer) else arch.sliding_head_dim


def kv_role_for_layer(arch: Gemma4Arch, layer: int) -> dict:
    """kvRoleForLayer (src/kv.ts:76-88): producers read their own cache, consumers the last
    producer of the same attention type."""
    if not (0 <= layer < arch.layer_count):
        raise ValueError(f"kvRoleForLayer: layer {layer} outside 0..{arch.layer_count - 1}")
    if is_kv_producer(arch, layer):
        return {"kind": "producer", "layer": layer}
    want = is_global_layer(arch, layer)
    last = -1
    for p in range(arch.kv_producer_layers):
        if is_global_layer(arch, p) == want:
            last = p
    if last < 0:
        raise ValueError(f"kvRoleForLayer: no producer of the same type as layer {layer}")
    return {"kind": "consumer", "layer": layer, "readsFrom": last}


# ---------------------------------------------------------------- prefill chunks (plan.ts:160-192)

DEFAULT_PREFILL_CHUNK = 64


@dataclass(frozen=True)
class PrefillChunk:
    start: int
    end: int
    length: int


def prefill_chunks(start: int, prompt_length: int, chunk_size: int = DEFAULT_PREFILL_CHUNK):
    """Positions [start, prompt_length) in chunks of at most chunk_size; the last chunk is exactly
    the final position, so every earlier chunk stops at the KV producers."""
    if not isinstance(start, int) or start < 0:
        raise ValueError(f"prefillChunks: bad from {start}")
    if not isinstance(prompt_length, int) or prompt_length < start:
        raise ValueError(f"prefillChunks: promptLength {prompt_length} below from {start}")
    if not isinstance(chunk_size, int) or chunk_size <= 0:
        raise ValueError(f"prefillChunks: chunkSize must be a positive integer, got {chunk_size}")
    chunks = []
    last = prompt_length - 1
    s = start
    while s < last:
        e = min(s + chunk_size, last)
        chunks.append(PrefillChunk(s, e, e - s))
        s += chunk_size
    if prompt_length > start:
        chunks.append(PrefillChunk(last, prompt_length, 1))
    return chunks


# ---------------------------------------------------------------- dispatch lists (plan.ts:487-784)


@dataclass(frozen=True)
class DispatchStep:
    kernel: str    # the executor's kernel family (g4_last_launch_list's first field)
    phase: str     # embed, attn, mlp, ple, head
    layer: int
    modules: str   # the checkpoint modules or roles the launch covers (its second field)
    covers: str = ""   # the reference dispatch roles the fused launch replaces


GEMV_MAX_COLUMNS = 8   # the streaming GEMV takes up to 8 columns per launch
PLE_BLOCK_MAX_COLUMNS = 16   # the fused per-layer-input tail takes up to 16 columns per launch


def ple_block_eligible(arch: Gemma4Arch, cols: int) -> bool:
    """Whether the executor runs a layer's per-layer-input tail (post-FFN norm-residual,
    per_layer_input_gate, gelu times the per-layer row, per_layer_projection) as one cluster
    launch: a PD of 256, a hidden size that is a multiple of 256 and at most 2048, and 1..16
    columns on the GEMV path."""
    return (arch.ple_dim == 256 and arch.hidden_size % 256 == 0 and arch.hidden_size <= 2048
            and 1 <= cols <= PLE_BLOCK_MAX_COLUMNS)


def plan_layer(arch: Gemma4Arch, layer: int, mode: str = "decode", cols: int = 1) -> list:
    """One layer as the executor launches it on the GEMV path (steps narrower than the
    tensor-core threshold), each launch named by its kernel and the modules it covers. A decode
    step fuses the attention prologue, blocks and merge into one launch per layer; a prefill chunk
    runs the prologue, then the query-tiled attention (blocks and merge for a single column)."""
    producer = is_kv_producer(arch, layer)
    p = f"layers.{layer}."
    s = []
    reps = (cols + GEMV_MAX_COLUMNS - 1) // GEMV_MAX_COLUMNS

    def add(kernel, phase, modules, covers="", n=1):
        for _ in range(n):
            s.append(DispatchStep(kernel, phase, layer, modules, covers))

    pre = "input_layernorm" if layer == 0 else "previous tail join"
    qkv = p + "self_attn.q_proj" + (f",{p}self_attn.k_proj,{p}self_attn.v_proj" if producer else "")
    add("qgemv-4bit", "attn", qkv, f"{pre}; q_proj" + (", k_proj, v_proj" if producer else ""), reps)
    att = p + "self_attn" + (",kv_store" if producer else "")
    pro = "q_norm per head, rope q" + ("; k_norm, v_norm weightless, rope k, kv store" if producer else "")
    if mode == "decode":
        add("attention-decode", "attn", att, pro + "; attention; attention split fold")
    else:
        add("attn-prologue", "attn", att, pro)
        if cols > 1:
            add("attention-prefill", "attn", p + "self_attn", "attention; attention split fold")
        else:
            add("attention-blocks", "attn", p + "self_attn", "attention")
            add("attention-merge", "attn", p + "self_attn", "attention split fold")
    add("qgemv-4bit", "attn", p + "self_attn.o_proj", "o_proj", reps)
    add("qgemv-4bit", "mlp", f"{p}mlp.gate_proj,{p}mlp.up_proj",
        "post_attention_layernorm plus residual, pre_feedforward_layernorm; gate_proj, up_proj", reps)
    add("qgemv-4bit", "mlp", p + "mlp.down_proj", "gelu times up, down_proj", reps)
    if ple_block_eligible(arch, cols):
        add("ple-block", "ple", f"{p}per_layer_input_gate,{p}per_layer_projection",
            "post_feedforward_layernorm plus residual; per_layer_input_gate; "
            "gate times per layer row, per_layer_projection")
    else:
        add("qgemv-8bit", "ple", p + "per_layer_input_gate",
            "post_feedforward_layernorm plus residual; per_layer_input_gate", reps)
        add("qgemv-8bit", "ple", p + "per_layer_projection",
            "gate times per layer row, per_layer_projection", reps)
    return s


def plan_embed(arch: Gemma4Arch) -> list:
    return [
        DispatchStep("embed-gather", "embed", -1, "embed_tokens,embed_tokens_per_layer",
                     "embed_tokens gather, per layer embedding gather"),
        DispatchStep("dense-bf16", "embed", -1, "per_layer_model_projection",
                     "per_layer_model_projection"),
        DispatchStep("ple-combine", "embed", -1, "per_layer_projection_norm",
                     "per_layer_projection_norm, per layer inputs add, per layer inputs scale"),
    ]


def plan_head(arch: Gemma4Arch, cols: int = 1, advance: bool = False) -> list:
    reps = (cols + GEMV_MAX_COLUMNS - 1) // GEMV_MAX_COLUMNS
    s = [DispatchStep("qgemv-4bit-head", "head", -1, "lm_head",
                      "post_per_layer_input_norm plus residual, layer_scalar, final norm; lm_head; "
                      "tanh(logits / 30) * 30; argmax partials")] * reps
    s.append(DispatchStep("argmax-final", "head", -1, "argmax", "argmax final"))
    if advance:
        s.append(DispatchStep("advance", "head", -1, "position advance", "next step's position"))
    return s


def plan_decode_step(arch: Gemma4Arch = GEMMA4_E2B, cols: int = 1, advance: bool = False) -> list:
    """planDecodeStep (src/plan.ts:487-784) as this executor launches it: the embed, every layer,
    the head. `cols` sequences of one position each on the GEMV path."""
    steps = list(plan_embed(arch))
    for layer in range(arch.layer_count):
        steps += plan_layer(arch, layer, "decode", cols)
    steps += plan_head(arch, cols, advance)
    return steps


def plan_prefill_chunk(arch: Gemma4Arch, is_last: bool, cols: int = 1) -> list:
    """A prefill chunk of `cols` positions (src/plan.ts:790-824): the producer layers over every
    position but the last chunk's final one, which then runs as a one-column decode step through
    all layers and the head (the KV-sharing exit)."""
    body = cols - 1 if is_last else cols
    steps = []
    if body > 0:
        steps += plan_embed(arch)
        for layer in range(arch.kv_producer_layers):
            steps += plan_layer(arch, layer, "prefill", body)
    if is_last:
        steps += plan_decode_step(arch, 1)
    return steps


def census(steps) -> dict:
    out: dict = {}
    for s in steps:
        out[s.kernel] = out.get(s.kernel, 0) + 1
    return out


# ---------------------------------------------------------------- KV reuse (kv.ts:150-286)


@dataclass
class KvReusePlan:
    action: str
    reuse: int
    prefill_from: int
    prefill_count: int


def plan_kv_reuse(cached, nxt) -> KvReusePlan:
    """planKvReuse (src/kv.ts:194-218): extend, rewind, or reset."""
    if len(nxt) == 0:
        raise ValueError("planKvReuse: next must hold at least one token")
    o = 0
    while o < len(cached) and o < len(nxt) and cached[o] == nxt[o]:
        o += 1
    if o == len(nxt) or o == 0:
        return KvReusePlan("reset", 0, 0, len(nxt))
    if o == len(cached):
        return KvReusePlan("extend", o, o, len(nxt) - o)
    return KvReusePlan("rewind", o, o, len(nxt) - o)


@dataclass
class KvCacheState:
    """KvCacheState (src/kv.ts:230-286): which token ids the caches hold, host bookkeeping."""
    tokens: list = field(default_factory=list)

    @property
    def length(self) -> int:
        return len(self.tokens)

    def truncate(self, n: int) -> None:
        if not isinstance(n, int) or n < 0 or n > len(self.tokens):
            raise ValueError(f"KvCacheState.truncate: {n} outside 0..{len(self.tokens)}")
        del self.tokens[n:]

    def reset(self) -> None:
        self.tokens.clear()

    def append(self, ids) -> None:
        for i in ids:
            if not isinstance(i, int) or i < 0:
                raise ValueError(f"KvCacheState.append: bad token id {i}")
        self.tokens.extend(ids)

    def accept_prompt(self, nxt) -> KvReusePlan:
        plan = plan_kv_reuse(self.tokens, nxt)
        if plan.action == "reset":
            self.reset()
        elif plan.action == "rewind":
            self.truncate(plan.reuse)
        return plan


# ---------------------------------------------------------------- table split (tableSplit.ts)

DEFAULT_MAX_SLICE_BYTES = 256 * 1024 * 1024


@dataclass(frozen=True)
class TableSplitPlan:
    rows: int
    row_bytes: int
    rows_per_slice: int
    slices: tuple  # (index, start_row, row_count)
    single: bool


def plan_table_split(rows: int, row_bytes: int, max_binding: int, max_buffer: int,
                     max_slice_bytes: int = DEFAULT_MAX_SLICE_BYTES):
    """planTableSplit (src/tableSplit.ts:125-215): one buffer when the table fits the limit,
    otherwise vocab-row slices of at most the cap, 16-row aligned. None when a row cannot fit."""
    rows = max(0, int(rows))
    row_bytes = max(1, int(row_bytes))
    total = rows * row_bytes
    limit = max(0, min(int(max_binding), int(max_buffer)))
    fits = 0 < total <= limit
    cap = max(1, min(limit, int(max_slice_bytes)))
    per = (limit if fits else cap) // row_bytes
    if per < 1:
        return None
    aligned = per - per % 16 if per >= 16 else per
    per_slice = min(rows, aligned)
    slices = []
    s = 0
    while s < rows:
        slices.append((len(slices), s, min(per_slice, rows - s)))
        s += per_slice
    if not slices:
        slices.append((0, 0, 0))
    return TableSplitPlan(rows, row_bytes, per_slice, tuple(slices), len(slices) == 1)


# ---------------------------------------------------------------- synthetic prompts

_M64 = (1 << 64) - 1


def _mix64(z: int) -> int:
    z ^= z >> 30
    z = (z * 0xBF58476D1CE4E5B9) & _M64
    z ^= z >> 27
    z = (z * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def synth_prompt(seed: int, n: int, vocab: int = 262144) -> list:
    """Seeded prompt ids uniform over the vocabulary: the counter hash of (seed, stream 50, i),
    the same generator the library uses for the synthetic weights."""
    key = _mix64((seed ^ (50 * 0x9E3779B97F4A7C15)) & _M64)
    return [_mix64((key + i * 0xD1B54A32D192ED03) & _M64) % vocab for i in range(n)]


# ---------------------------------------------------------------- greedy loop (plan.ts:905-999)


def run_greedy_loop(first_token: int, max_new_tokens: int, eos_ids, start_position: int,
                    decode, is_aborted=lambda: False, decode_ahead=None):
    """The greedy schedule: yields (token, index). The first token comes from the prefill; a stop
    token ends the loop and is not yielded. With `decode_ahead`, the next step reads its input
    token from the device (the tokens are the same)."""
    budget = max(0, int(max_new_tokens))
    if budget == 0 or is_aborted():
        return
    if first_token in eos_ids:
        return
    yield first_token, 0
    prev = first_token
    for index in range(1, budget):
        if is_aborted():
            return
        pos = start_position + index - 1
        token = decode_ahead(pos) if decode_ahead else decode(prev, pos)
        if token in eos_ids:
            return
        yield token, index
        prev = token


# ---------------------------------------------------------------- speculative decode (draft.ts)

LOOKUP_MAX_NGRAM = 8
LOOKUP_MIN_NGRAM = 2


class LookupDrafter:
    """Prompt-lookup drafting (createLookupDrafter, src/draft.ts:60-98): take the last n tokens,
    find their most recent earlier occurrence, propose what followed it; the longest n first
    (max_ngram down to min_ngram), never padding past the end of what exists."""

    def __init__(self, max_ngram: int = LOOKUP_MAX_NGRAM, min_ngram: int = LOOKUP_MIN_NGRAM):
        self.hi = max(1, int(max_ngram))
        self.lo = max(1, min(self.hi, int(min_ngram)))
        self.name = f"lookup-{self.lo}-{self.hi}"

    def propose(self, tokens, want: int) -> list:
        wanted = max(0, int(want))
        n_tok = len(tokens)
        if wanted == 0 or n_tok < self.lo + 1:
            return []
        for n in range(min(self.hi, n_tok - 1), self.lo - 1, -1):
            frm = n_tok - n
            suffix = list(tokens[frm:])
            for start in range(frm - 1, -1, -1):
                if list(tokens[start:start + n]) != suffix:
                    continue
                out = list(tokens[start + n:start + n + wanted])
                if out:
                    return out
        return []


@dataclass
class SpeculationStats:
    """What a speculative run did (SpeculationStats, src/draft.ts:104-134)."""
    passes: int = 0
    proposed_drafts: int = 0
    drafted_tokens: int = 0
    accepted_drafts: int = 0
    tokens: int = 0

    def tokens_per_pass(self) -> float:
        return 0.0 if self.passes == 0 else self.tokens / self.passes

    def acceptance_rate(self) -> float:
        return 0.0 if self.drafted_tokens == 0 else self.accepted_drafts / self.drafted_tokens


def run_speculative_loop(first_token: int, max_new_tokens: int, eos_ids, start_position: int,
                         history, max_columns: int, drafter, decode, verify,
                         is_aborted=lambda: False, on_advance=None, stats=None):
    """runSpeculativeLoop (src/draft.ts:233-330): the greedy loop with one pass per group of
    tokens. A pass verifies [prev, *draft] when the drafter proposes and decodes prev otherwise;
    the longest prefix of the draft the model agrees with is accepted, plus the model's own next
    token. Yields (token, index) exactly as run_greedy_loop does for the same model."""
    budget = max(0, int(max_new_tokens))
    if budget == 0 or is_aborted():
        return
    if first_token in eos_ids:
        return
    yield first_token, 0
    stats = stats if stats is not None else SpeculationStats()
    hist = list(history) + [first_token]
    max_draft = max(0, int(max_columns) - 1)
    prev, position, index = first_token, start_position, 1
    while index < budget:
        if is_aborted():
            return
        want = min(max_draft, budget - index - 1)
        draft = drafter.propose(hist, want) if want > 0 else []
        stats.passes += 1
        if draft:
            stats.proposed_drafts += 1
            stats.drafted_tokens += len(draft)
            answer = list(verify([prev, *draft], position))
            if not answer:
                return
            if len(answer) != len(draft) + 1:
                raise RuntimeError(f"gemma4 engine: a verify pass over {len(draft) + 1} positions "
                                   f"answered {len(answer)}")
        else:
            answer = [decode(prev, position)]
        matched = 0
        while matched < len(draft) and answer[matched] == draft[matched]:
            matched += 1
        stats.accepted_drafts += matched
        if on_advance:
            on_advance(prev, position)
        for j in range(matched + 1):
            token = answer[j]
            if token in eos_ids:
                return
            yield token, index
            index += 1
            stats.tokens += 1
            hist.append(token)
            if j < matched and on_advance:
                on_advance(token, position + 1 + j)
        prev = answer[matched]
        position += 1 + matched
