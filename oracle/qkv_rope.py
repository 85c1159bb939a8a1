"""oracle.qkv_rope -- TEST INFRASTRUCTURE ONLY: the CPU checker for the QKV producer
(attn_qkv_rope_stream / attn_qkv_rope_paged_stream / attn_rope_table_stream).

numpy restatement of the published formulas the producer implements: RMSNorm (Zhang &
Sennrich, 2019) and rotary position embedding (Su et al., RoFormer, 2021) in its rotate-half
(NeoX) and interleaved (GPT-J) pairings. The reference has no counterpart -- its projections
never reach the attention kernel (flash.c:1301-1304) -- so parity is pinned to golden vectors
made with transformers' own Qwen3 and GPT-J functions (tests/golden/make_rope_golden.py), and
bf16 rounding follows flash.c:78-92 (the oracle package's f32_to_bf16).

Two forms:
  * rope_f32: the producer's exact fp32 arithmetic (x*cos and y*sin each rounded to fp32, then
    one fp32 add/subtract) -- bit-exact expectations when no RMSNorm is applied;
  * produce(): float64 throughout (norm and rotation), the value the bf16 output must round
    to within one bf16 ulp (rsqrt on the GPU is not correctly rounded).
Only tests/ and bench.py's checks may use this module, never the product.
"""
from __future__ import annotations

import numpy as np

from oracle import bf16_to_f32, f32_to_bf16

NEOX = 1
GPTJ = 0


def rope_table(max_pos: int, rot: int, theta: float) -> np.ndarray:
    """fp32 [max_pos][rot]: cos(p * theta^(-2i/rot)) in column i < rot/2, the sine in rot/2 + i;
    angle and trig in float64, one rounding to fp32."""
    half = rot // 2
    f = np.power(float(theta), -2.0 * np.arange(half, dtype=np.float64) / rot)
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * f[None, :]
    return np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32)


def _pairs(rot: int, style: int):
    """Index arrays (a, b, freq): element a pairs with element b at frequency freq; a takes
    x_a cos - x_b sin, b takes x_b cos + x_a sin."""
    half = rot // 2
    if style == NEOX:
        a = np.arange(half)
        return a, a + half, a
    a = np.arange(0, rot, 2)
    return a, a + 1, a // 2


def rope_f32(x: np.ndarray, cs_rows: np.ndarray, rot: int, style: int) -> np.ndarray:
    """x fp32 [..., D], cs_rows fp32 [..., rot] (each vector's table row): the producer's fp32
    arithmetic, element for element."""
    out = np.array(x, dtype=np.float32, copy=True)
    if rot == 0:
        return out
    half = rot // 2
    a, b, f = _pairs(rot, style)
    c = cs_rows[..., :half][..., f].astype(np.float32)
    s = cs_rows[..., half:][..., f].astype(np.float32)
    xa, xb = x[..., a].astype(np.float32), x[..., b].astype(np.float32)
    out[..., a] = (xa * c).astype(np.float32) - (xb * s).astype(np.float32)
    out[..., b] = (xb * c).astype(np.float32) + (xa * s).astype(np.float32)
    return out


def rope_f64(x: np.ndarray, cs_rows: np.ndarray, rot: int, style: int) -> np.ndarray:
    out = np.array(x, dtype=np.float64, copy=True)
    if rot == 0:
        return out
    half = rot // 2
    a, b, f = _pairs(rot, style)
    c = cs_rows[..., :half][..., f].astype(np.float64)
    s = cs_rows[..., half:][..., f].astype(np.float64)
    xa, xb = x[..., a].astype(np.float64), x[..., b].astype(np.float64)
    out[..., a] = xa * c - xb * s
    out[..., b] = xb * c + xa * s
    return out


def rms_norm_f64(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(np.float64)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + float(np.float32(eps)))
    return x * r * w.astype(np.float64)


def produce(qkv_bits, positions, cs, q_norm_bits, k_norm_bits, eps, B, S, Hq, Hkv, D, rot, style):
    """The producer's outputs before the cache write: (Q, K, V), Q [B*Hq][S][D] and K, V
    [B][S][Hkv][D] (token order). q/k heads come back float64 when a norm applies (compare
    within one bf16 ulp) and as exact bf16 bits otherwise; V is always the input bits."""
    T = B * S
    x = qkv_bits.reshape(T, Hq + 2 * Hkv, D)
    rows = cs[positions] if rot > 0 else np.zeros((T, 0), np.float32)

    def heads(lo, n, w_bits):
        h = bf16_to_f32(np.ascontiguousarray(x[:, lo:lo + n]))
        r = rows[:, None, :]
        if w_bits is not None:
            return rope_f64(rms_norm_f64(h, bf16_to_f32(w_bits), eps), r, rot, style)
        return f32_to_bf16(rope_f32(h, r, rot, style))

    q = heads(0, Hq, q_norm_bits)
    k = heads(Hq, Hkv, k_norm_bits)
    v = np.ascontiguousarray(x[:, Hq + Hkv:])
    Q = q.reshape(B, S, Hq, D).transpose(0, 2, 1, 3).reshape(B * Hq, S, D)
    return Q, k.reshape(B, S, Hkv, D), v.reshape(B, S, Hkv, D)


def bf16_ulp(v: np.ndarray) -> np.ndarray:
    """One bf16 ulp at |v| (8 significant bits); the smallest normal's ulp below it."""
    a = np.maximum(np.abs(v.astype(np.float64)), np.finfo(np.float32).tiny)
    return np.exp2(np.floor(np.log2(a)) - 7)


def within_one_ulp(got_bits: np.ndarray, ref: np.ndarray, atol: float = 0.0) -> np.ndarray:
    """Elementwise: the bf16 value `got_bits` lies within one bf16 ulp (plus `atol`) of the
    float64 `ref`. `atol` covers fp32 rounding of the terms when a rotation cancels them to a
    value far below their size."""
    got = bf16_to_f32(got_bits).astype(np.float64)
    return np.abs(got - ref) <= bf16_ulp(ref) + atol
