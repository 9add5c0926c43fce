"""A line-by-line Python transliteration of the reference's own CPU oracles (TypeScript), used to
generate golden vectors that pin the C oracle. Independent of oracle/g4_oracle.c: written from the
TypeScript text, with JavaScript's f64 arithmetic as Python floats and `Math.fround` as a
round-trip through numpy float32. Pure-Python loops: small cases only.

Test infrastructure; the product never imports it.
"""
from __future__ import annotations

import math

import numpy as np


def fround(x: float) -> float:
    return float(np.float32(x))


# src/quant.ts:350-357 roundTiesToEven
def round_ties_to_even(x: float) -> float:
    if not math.isfinite(x):
        return x
    truncated = math.trunc(x)
    fraction = x - truncated
    if fraction != 0.5 and fraction != -0.5:
        return float(math.floor(x + 0.5))  # Math.round
    return float(truncated if truncated % 2 == 0 else truncated + math.copysign(1, fraction))


# src/quant.ts:309-334 srqCodes
def srq_codes(values, scale, bits=8):
    if scale == 0:
        return [0.0] * len(values)
    mx = 2 ** (bits - 1) - 1
    mn = -mx - 1
    out = []
    for v in values:
        r = round_ties_to_even(fround(fround(v) / fround(scale)))
        out.append(float(mn if r < mn else mx if r > mx else r))
    return out


# src/quant.ts:278-288 applySrq
def apply_srq(values, scale):
    if scale == 0:
        return [fround(v) for v in values]
    codes = srq_codes(values, scale)
    return [fround(c * scale) for c in codes]


# src/quant.ts:87-96 unpackInt4, 121-129 unpackInt8
def unpack_int4(packed, width):
    out = []
    for i in range(width):
        b = packed[i >> 1] if (i >> 1) < len(packed) else 0
        nib = (b & 0x0F) if (i & 1) == 0 else (b >> 4) & 0x0F
        out.append(nib - 8)
    return out


def unpack_int8(packed, width):
    return [(b - 256 if b > 127 else b) for b in packed[:width]]


# src/kernels/qlayout.ts:28-54 unpackWordsLikeShader at 2 bits: code k at bits 2 (k % 16) of
# word k / 16, zero point 2.
def unpack_2bit_words(words, width):
    return [((words[i >> 4] >> (2 * (i & 15))) & 3) - 2 for i in range(width)]


# src/kernels/qlayout.ts:172-175 tile16Words
def tile16_words(rows, k):
    if k % 16:
        raise ValueError(f"tile16Words: k must be a multiple of 16, got {k}")
    return -(-rows // 16) * k


# src/kernels/qlayout.ts:186-206 rowWordsToTile16
def row_words_to_tile16(row_words, rows, k):
    k_words = k // 16
    out = [0] * tile16_words(rows, k)
    for row in range(rows):
        tile, shift = row // 16, 2 * (row % 16)
        dst, src = tile * k, row * k_words
        for w in range(k_words):
            word = row_words[src + w]
            for i in range(16):
                code = (word >> (2 * i)) & 3
                out[dst + w * 16 + i] |= code << shift
    return out


# src/kernels/qlayout.ts:209-227 tile16ToRowWords
def tile16_to_row_words(tile_words, rows, k):
    k_words = k // 16
    out = [0] * (rows * k_words)
    for row in range(rows):
        tile, shift = row // 16, 2 * (row % 16)
        src, dst = tile * k, row * k_words
        for kk in range(k):
            code = (tile_words[src + kk] >> shift) & 3
            out[dst + (kk >> 4)] |= code << (2 * (kk & 15))
    return out


def _row_codes(bits, packed, r, k, num_rows):
    if bits == 2:
        # The 2-bit family's buffers are in the interleaved layout; read back to row words.
        return unpack_2bit_words(packed[r * (k // 16):(r + 1) * (k // 16)], k)
    row_bytes = k * bits // 8
    row = packed[r * row_bytes:(r + 1) * row_bytes]
    return unpack_int4(row, k) if bits == 4 else unpack_int8(row, k)


def _as_rows(bits, packed, num_rows, k):
    """2-bit: `packed` is the tile layout as u32 words; returns row words."""
    return tile16_to_row_words(packed, num_rows, k) if bits == 2 else packed


# src/kernels/qgemv.ts:1131-1176 qgemvOracle
def qgemv_oracle(bits, packed, scales, x, num_rows, k, in_scale=0.0, out_scale=0.0):
    calibrated = in_scale != 0
    x_codes = srq_codes(x[:k], in_scale) if calibrated else None
    packed = _as_rows(bits, packed, num_rows, k)
    out = []
    for r in range(num_rows):
        codes = _row_codes(bits, packed, r, k, num_rows)
        scale = fround(scales[r])
        s = 0.0
        if x_codes is not None:
            for i in range(k):
                s += codes[i] * x_codes[i]
        else:
            for i in range(k):
                s += codes[i] * x[i]
        xs = fround(in_scale) if calibrated else 1.0
        out.append(fround(fround(xs * scale) * fround(s)))
    return apply_srq(out, out_scale)


def qgemv_acc(bits, packed, x, num_rows, k, in_scale):
    """The exact integer accumulators of the calibrated path."""
    x_codes = srq_codes(x[:k], in_scale)
    packed = _as_rows(bits, packed, num_rows, k)
    accs = []
    for r in range(num_rows):
        codes = _row_codes(bits, packed, r, k, num_rows)
        accs.append(int(sum(c * int(q) for c, q in zip(codes, x_codes))))
    return accs


# src/kernels/rmsNorm.ts:208-245 rmsNormOracle
def rms_norm_oracle(src, gain, rows, width, eps):
    out = []
    for r in range(rows):
        base = r * width
        s = 0.0
        for i in range(width):
            v = src[base + i]
            s += v * v
        inv = 1 / math.sqrt(s / width + eps)
        for i in range(width):
            out.append(fround(src[base + i] * inv * (gain[i] if gain is not None else 1)))
    return out


# src/kernels/mlpEpilogue.ts:196-220 normResidualOracle
def norm_residual_oracle(src, gain, residual, rows, width, eps):
    out = []
    for r in range(rows):
        base = r * width
        s = 0.0
        for i in range(width):
            s += src[base + i] * src[base + i]
        inv = 1 / math.sqrt(s / width + eps)
        for i in range(width):
            out.append(fround(residual[base + i] + src[base + i] * inv * gain[i]))
    return out


# src/kernels/geluMul.ts:172-240 geluTanhScalar, geluMulOracle
def gelu_tanh_scalar(x):
    inner0 = 0.7978845608028654 * (x + 0.044715 * x * x * x)
    inner = 10 if inner0 > 10 else -10 if inner0 < -10 else inner0
    return 0.5 * x * (1 + math.tanh(inner))


def gelu_mul_oracle(gate, up, count, srq_scale=0.0):
    out = [fround(gelu_tanh_scalar(gate[i]) * up[i]) for i in range(count)]
    return apply_srq(out, srq_scale)


# src/kernels/attention.ts:858-903 attentionOracle
def attention_oracle(q, k, v, heads, head_dim, q_count, q_start, kv_len, window, scale=1.0):
    out = [0.0] * (q_count * heads * head_dim)
    for qi in range(q_count):
        p = q_start + qi
        lo = max(0, p - window + 1) if window > 0 else 0
        for h in range(heads):
            qb = (qi * heads + h) * head_dim
            scores = {}
            m = -math.inf
            for j in range(lo, p + 1):
                d = 0.0
                for i in range(head_dim):
                    d += q[qb + i] * k[j * head_dim + i]
                s = d * scale
                scores[j] = s
                m = max(m, s)
            l = 0.0
            for j in range(lo, p + 1):
                scores[j] = math.exp(scores[j] - m)
                l += scores[j]
            for i in range(head_dim):
                a = 0.0
                for j in range(lo, p + 1):
                    a += scores[j] * v[j * head_dim + i]
                out[qb + i] = fround(a / l)
    return out


# src/kernels/embedGather.ts:319-344 embedGatherOracle (row layout, 4-bit)
def embed_gather_oracle(codes_bytes, scales, ids, cols, group_size, output_scale):
    groups = cols // group_size
    out_scale = fround(output_scale)
    out = []
    for row in ids:
        rb = codes_bytes[row * cols // 2:(row + 1) * cols // 2]
        codes = [c + 8 for c in unpack_int4(rb, cols)]
        for col in range(cols):
            scale = fround(out_scale * scales[row * groups + col // group_size])
            out.append(fround((codes[col] - 8) * scale))
    return out


# src/kernels/logitSoftcap.ts:104-120 softcapOracle and src/kernels/argmax.ts:267-310
def softcap_oracle(logits, cap=30.0):
    return [fround(math.tanh(l / cap) * cap) for l in logits]


def argmax_oracle(values):
    index, value = -1, -math.inf
    for i, v in enumerate(values):
        if v > value:
            value, index = v, i
    return index


# src/kernels/rope.ts:149-191 ropeInverseFrequencies / ropeTables
def rope_inverse_frequencies(head_dim, rotary_pairs, theta):
    return [math.pow(theta, (-2 * i) / head_dim) if i < rotary_pairs else 0.0
            for i in range(head_dim // 2)]


def rope_tables(head_dim, rotary_pairs, theta, positions):
    inv = rope_inverse_frequencies(head_dim, rotary_pairs, theta)
    cos, sin = [], []
    for pos in positions:
        for i in range(head_dim // 2):
            cos.append(fround(math.cos(pos * inv[i])))
            sin.append(fround(math.sin(pos * inv[i])))
    return cos, sin
