"""Numpy restatement of the reference's decoder-attention correctness path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

BF16 tensors are carried as ``uint16`` bit patterns.  Every stage rounds to
BF16 (round-to-nearest-even) exactly where the reference stores BF16.  FP32
arithmetic is ``numpy.float32``; sums are taken in float64 and rounded once to
FP32 (the correctly rounded value of the reference's FP32 sum), and the
transcendentals (pow, cos, sin, exp) are evaluated in float64 and rounded once
to FP32.  The reference's torch CPU path reduces in its own vectorised order
and uses SLEEF, so the two can differ by an FP32 ulp before the BF16 boundary;
the golden-vector tests state that tolerance.

* RMSNorm ............ reference/decoder_attention.py:117-140
* head reshape ....... reference/decoder_attention.py:181-202
* adjacent-pair RoPE . reference/decoder_attention.py:205-270
* causal GQA ......... reference/decoder_attention.py:273-381
* W4A16 projection ... reference/w4a16.py:11-59
* composition ........ reference/decoder_attention_nvfp4.py:45-141
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from .nvfp4 import NVFP4Storage, dequantize


# ---------------------------------------------------------------- BF16 bits
def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """FP32 -> BF16 bits, round to nearest even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    nan = np.isnan(x)
    if np.any(nan):
        out = np.where(nan, ((bits >> 16) | 0x40).astype(np.uint16), out)
    return out


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def _sum_f32(values: np.ndarray, axis: int) -> np.ndarray:
    """Correctly rounded FP32 value of an FP32 sum (float64 accumulation)."""
    return np.sum(values.astype(np.float64), axis=axis).astype(np.float32)


# ------------------------------------------------------------------ stages
def rms_norm(x_bits: np.ndarray, w_bits: np.ndarray, eps: float) -> np.ndarray:
    """``BF16(x * rsqrt(mean(x^2) + eps) * w)`` over the last axis.

    reference/decoder_attention.py:117-140: the mean is an FP32 sum divided by
    the length, rsqrt is ``1 / sqrt`` in FP32, then two FP32 products.
    """
    x = bf16_to_f32(x_bits)
    w = bf16_to_f32(w_bits)
    n = np.float32(x.shape[-1])
    sq = (x * x).astype(np.float32)
    mean = (_sum_f32(sq, -1) / n).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt((mean + np.float32(eps)).astype(np.float32))).astype(np.float32)
    y = ((x * inv[..., None]).astype(np.float32) * w).astype(np.float32)
    return f32_to_bf16(y)


def rope_cos_sin(positions: np.ndarray, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """FP32 cos/sin tables ``[len(positions), head_dim/2]``.

    reference/decoder_attention.py:237-257: exponent ``2m/D`` in FP32, the
    denominator ``theta ** exponent`` in FP32, ``angle = p / denominator`` in
    FP32, then FP32 cos and sin.
    """
    exps = (np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)).astype(np.float32)
    theta32 = np.float32(theta)
    denom = np.power(np.float64(theta32), exps.astype(np.float64)).astype(np.float32)
    pos = np.asarray(positions, dtype=np.int64).astype(np.float32)
    angle = (pos[:, None] / denom[None, :]).astype(np.float32)
    a64 = angle.astype(np.float64)
    return np.cos(a64).astype(np.float32), np.sin(a64).astype(np.float32)


def apply_rope(x_bits: np.ndarray, past_lengths, theta: float) -> np.ndarray:
    """Adjacent-pair RoPE on ``[B, T, H, D]`` BF16 bits at positions ``P_b + t``.

    reference/decoder_attention.py:205-270.  ``past_lengths`` is a scalar
    (the reference API) or one value per batch row (variable-length decode).
    """
    b_, t_, _, d_ = x_bits.shape
    p = np.broadcast_to(np.asarray(past_lengths, dtype=np.int64), (b_,))
    x = bf16_to_f32(x_bits)
    out = np.empty_like(x)
    for b in range(b_):
        cos, sin = rope_cos_sin(p[b] + np.arange(t_), d_, theta)
        c = cos[:, None, :]
        s = sin[:, None, :]
        xe = x[b, ..., 0::2]
        xo = x[b, ..., 1::2]
        out[b, ..., 0::2] = ((xe * c).astype(np.float32) - (xo * s).astype(np.float32)).astype(np.float32)
        out[b, ..., 1::2] = ((xe * s).astype(np.float32) + (xo * c).astype(np.float32)).astype(np.float32)
    return f32_to_bf16(out)


def w4a16_linear(x_bits: np.ndarray, weight: NVFP4Storage) -> np.ndarray:
    """``BF16(sum_k FP32(x_k * W_hat[n, k]))`` (reference/w4a16.py:11-59).

    ``W_hat`` is the FP32 dequantized matrix; each product is FP32, the sum is
    correctly rounded to FP32.
    """
    rows, k = weight.logical_shape
    w = dequantize(weight)
    x = bf16_to_f32(x_bits).reshape(-1, k)
    out = np.empty((x.shape[0], rows), dtype=np.float32)
    chunk = max(1, (1 << 24) // max(1, rows * k))
    for m0 in range(0, x.shape[0], chunk):
        prod = (x[m0:m0 + chunk, None, :] * w[None, :, :]).astype(np.float32)
        out[m0:m0 + chunk] = _sum_f32(prod, -1)
    return f32_to_bf16(out).reshape(*x_bits.shape[:-1], rows)


def gqa_attention(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray,
                  past_lengths, cache_len=None) -> np.ndarray:
    """Causal GQA over caches ``[B, Hkv, C, D]`` (reference/decoder_attention.py:273-381).

    ``q`` is ``[B, T, Hq, D]``; query head ``h`` reads KV head ``h // (Hq/Hkv)``.
    Key ``j`` is visible to token ``i`` iff ``j <= P_b + i``; only the first
    ``P_b + T`` cache slots are read, so a physical capacity ``C`` larger than
    the logical length behaves like the reference's compact present cache.
    Scores are ``FP32(q.k) * FP32(1/sqrt(D))``; softmax is ``exp(s - max)``
    times the FP32 reciprocal of the FP32 sum; context is ``BF16(sum p*v)``.
    """
    b_, t_, hq, d_ = q_bits.shape
    hkv = k_bits.shape[1]
    group = hq // hkv
    p = np.broadcast_to(np.asarray(past_lengths, dtype=np.int64), (b_,))
    scale = np.float32(1.0 / math.sqrt(d_))
    q = bf16_to_f32(q_bits)
    out = np.empty((b_, t_, hq, d_), dtype=np.float32)
    for b in range(b_):
        s_len = int(p[b]) + t_
        visible = np.arange(s_len)[None, :] <= (int(p[b]) + np.arange(t_))[:, None]
        for h in range(hq):
            kv = h // group
            k = bf16_to_f32(k_bits[b, kv, :s_len]).astype(np.float64)  # [S, D]
            qh = q[b, :, h, :].astype(np.float64)  # [T, D]
            # BF16 x BF16 products are exact in FP32, so the float64 matmul is
            # the correctly rounded FP32 sum of the reference's FP32 products.
            scores = ((qh @ k.T).astype(np.float32) * scale).astype(np.float32)
            scores = np.where(visible, scores, np.float32(-np.inf))
            mx = np.max(scores, axis=-1, keepdims=True)
            e = np.exp((scores - mx).astype(np.float32).astype(np.float64)).astype(np.float32)
            denom = _sum_f32(e, -1)
            probs = (e * (np.float32(1.0) / denom)[:, None]).astype(np.float32)  # [T, S]
            v = bf16_to_f32(v_bits[b, kv, :s_len])  # [S, D]
            acc = np.zeros((t_, d_), dtype=np.float64)
            step = max(1, (1 << 22) // max(1, t_ * d_))
            for j0 in range(0, s_len, step):
                # each FP32 product p*v is rounded to FP32, then summed
                pv = (probs[:, j0:j0 + step, None] * v[None, j0:j0 + step, :]).astype(np.float32)
                acc += pv.astype(np.float64).sum(axis=1)
            out[b, :, h, :] = acc.astype(np.float32)
    return f32_to_bf16(out)


@dataclass
class DecodeStages:
    """Stored BF16 stages (reference/decoder_attention_nvfp4.py:20-31)."""

    input_normalized: np.ndarray
    q_projected: np.ndarray
    k_projected: np.ndarray
    v_projected: np.ndarray
    q_normalized: np.ndarray
    k_normalized: np.ndarray
    q_rope: np.ndarray
    k_rope: np.ndarray
    context: np.ndarray
    output: np.ndarray


def decoder_attention_nvfp4(x_bits, input_norm_w, q_w: NVFP4Storage, k_w: NVFP4Storage,
                            v_w: NVFP4Storage, q_norm_w, k_norm_w, o_w: NVFP4Storage,
                            k_cache, v_cache, past_lengths, *, rms_eps=1e-6,
                            rope_theta=10000.0):
    """One forward step over physical caches ``[B, Hkv, C, D]`` (BF16 bits).

    Follows reference/decoder_attention_nvfp4.py:45-141.  The caches are
    updated in place at slots ``P_b .. P_b+T-1`` (the reference appends by
    ``torch.cat``; the physical-cache equivalent is the in-place write of
    reference decoder_attention_cuda.py:389-395).  Returns ``DecodeStages``.
    """
    b_, t_, h = x_bits.shape
    hkv, d_ = k_cache.shape[1], k_cache.shape[3]
    hq = h // d_
    p = np.broadcast_to(np.asarray(past_lengths, dtype=np.int64), (b_,))
    xn = rms_norm(x_bits, input_norm_w, rms_eps)
    qp = w4a16_linear(xn, q_w)
    kp = w4a16_linear(xn, k_w)
    vp = w4a16_linear(xn, v_w)
    qh = qp.reshape(b_, t_, hq, d_)
    kh = kp.reshape(b_, t_, hkv, d_)
    vh = vp.reshape(b_, t_, hkv, d_)
    qn = rms_norm(qh, q_norm_w, rms_eps)
    kn = rms_norm(kh, k_norm_w, rms_eps)
    qr = apply_rope(qn, p, rope_theta)
    kr = apply_rope(kn, p, rope_theta)
    for b in range(b_):
        pb = int(p[b])
        k_cache[b, :, pb:pb + t_] = kr[b].transpose(1, 0, 2)
        v_cache[b, :, pb:pb + t_] = vh[b].transpose(1, 0, 2)
    ctx = gqa_attention(qr, k_cache, v_cache, p)
    out = w4a16_linear(ctx.reshape(b_, t_, h), o_w)
    return DecodeStages(xn, qp, kp, vp, qn, kn, qr, kr, ctx, out)
