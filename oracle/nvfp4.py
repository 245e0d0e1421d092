"""Numpy restatement of the reference's portable NVFP4 storage format.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Every function follows ``reference/nvfp4.py`` of the reference repository
step for step, with FP32 arithmetic done in ``numpy.float32`` so that each
rounding happens where the reference's FP32 torch ops round:

* E2M1 decode table ............ reference/nvfp4.py:23-40, 269-284
* UE4M3 decode ................. reference/nvfp4.py:43-53, 341-361
* E2M1 RNE encoder ............. reference/nvfp4.py:287-338
* UE4M3 RNE encoder ............ reference/nvfp4.py:364-392
* pack / unpack ................ reference/nvfp4.py:395-436
* global encode/decode scales .. reference/nvfp4.py:443-460
* conversion factors ........... reference/nvfp4.py:470-482
* block scale state ............ reference/nvfp4.py:485-497
* quantize ..................... reference/nvfp4.py:500-536
* dequantize ................... reference/nvfp4.py:539-554
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

BLOCK = 16
E2M1_MAX = 6.0
UE4M3_MAX = 448.0
GLOBAL_RANGE = E2M1_MAX * UE4M3_MAX  # 2688
F32_MAX = np.float32(np.finfo(np.float32).max)

# Nibble -> value; code 0x8 is negative zero (reference/nvfp4.py:23-40).
E2M1_TABLE = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)


def _ue4m3_value(code: int) -> float:
    # e == 0: m * 2^-9 ; else (1 + m/8) * 2^(e-7)  (reference/nvfp4.py:43-50)
    e = (code >> 3) & 0xF
    m = code & 0x7
    if e == 0:
        return math.ldexp(float(m), -9)
    return math.ldexp(1.0 + m / 8.0, e - 7)


# Canonical finite bytes 0x00..0x7e; 0x7f and >=0x80 are invalid.
UE4M3_TABLE = np.array([_ue4m3_value(c) for c in range(0x7F)], dtype=np.float32)


@dataclass(frozen=True)
class NVFP4Storage:
    """The three fields of the reference's ``NVFP4Tensor`` (reference/nvfp4.py:56-71)."""

    packed_values: np.ndarray  # uint8 [N, K/2], even k in the low nibble
    block_scales: np.ndarray  # uint8 [N, K/16], canonical UE4M3
    global_decode_scale: np.float32  # FP32 scalar
    logical_shape: tuple[int, int]


def decode_e2m1(codes: np.ndarray) -> np.ndarray:
    codes = np.asarray(codes, dtype=np.uint8)
    if np.any(codes > 0x0F):
        raise ValueError("E2M1 codes must be nibbles in 0x0..0xf")
    return E2M1_TABLE[codes.astype(np.int64)]


def decode_ue4m3(scale_bytes: np.ndarray) -> np.ndarray:
    scale_bytes = np.asarray(scale_bytes, dtype=np.uint8)
    if np.any(scale_bytes > 0x7E):
        raise ValueError("UE4M3 scale bytes must be canonical finite bytes in 0x00..0x7e")
    return UE4M3_TABLE[scale_bytes.astype(np.int64)]


def encode_e2m1(values: np.ndarray) -> np.ndarray:
    """E2M1 round-to-nearest-even with finite saturation (reference/nvfp4.py:287-338).

    Inclusive bounds are the midpoints whose even neighbour is the lower code.
    """
    v = np.asarray(values, dtype=np.float32)
    if not np.all(np.isfinite(v)):
        raise ValueError("values must contain only finite values")
    mag = np.abs(v)
    code = np.full(mag.shape, 0x7, dtype=np.uint8)
    code = np.where(mag <= 5.0, np.uint8(0x6), code)
    code = np.where(mag < 3.5, np.uint8(0x5), code)
    code = np.where(mag <= 2.5, np.uint8(0x4), code)
    code = np.where(mag < 1.75, np.uint8(0x3), code)
    code = np.where(mag <= 1.25, np.uint8(0x2), code)
    code = np.where(mag < 0.75, np.uint8(0x1), code)
    code = np.where(mag <= 0.25, np.uint8(0x0), code)
    sign = np.where(np.signbit(v), np.uint8(0x8), np.uint8(0x0))
    return (code | sign).astype(np.uint8)


def encode_ue4m3(candidates: np.ndarray) -> np.ndarray:
    """UE4M3 round-to-nearest-even with saturation to 0x7e (reference/nvfp4.py:364-392)."""
    c = np.asarray(candidates, dtype=np.float32)
    if not np.all(np.isfinite(c)) or np.any(c < 0.0):
        raise ValueError("UE4M3 candidates must be finite and nonnegative")
    flat = c.reshape(-1)
    ins = np.searchsorted(UE4M3_TABLE, flat, side="left")
    upper = np.clip(ins, 0, 0x7E)
    lower = np.clip(ins - 1, 0, 0x7E)
    up_v = UE4M3_TABLE[upper]
    lo_v = UE4M3_TABLE[lower]
    up_d = np.abs(up_v - flat)
    lo_d = np.abs(flat - lo_v)
    tie_even_up = (up_d == lo_d) & ((upper & 1) == 0)
    choose_up = (up_d < lo_d) | tie_even_up
    return np.where(choose_up, upper, lower).astype(np.uint8).reshape(c.shape)


def pack_e2m1(codes: np.ndarray) -> np.ndarray:
    """Even K element in the low nibble, odd in the high nibble (reference/nvfp4.py:395-413)."""
    codes = np.asarray(codes, dtype=np.uint8)
    return (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)


def unpack_e2m1(packed: np.ndarray) -> np.ndarray:
    """Inverse of :func:`pack_e2m1` (reference/nvfp4.py:416-436)."""
    packed = np.asarray(packed, dtype=np.uint8)
    lo = packed & 0x0F
    hi = packed >> 4
    return np.stack((lo, hi), axis=-1).reshape(packed.shape[0], -1)


def global_scales(source_f32: np.ndarray) -> tuple[np.float32, np.float32]:
    """``(global_encode_scale, global_decode_scale)`` (reference/nvfp4.py:443-460)."""
    amax = np.float32(np.max(np.abs(source_f32)))
    if amax == 0.0:
        enc = np.float32(1.0)
    else:
        with np.errstate(over="ignore", divide="ignore"):
            enc = np.minimum(np.float32(GLOBAL_RANGE) / amax, F32_MAX)
    dec = np.float32(amax * np.float32(1.0 / GLOBAL_RANGE))
    return np.float32(enc), dec


def _conversion_factors(enc: np.float32, beta: np.ndarray) -> np.ndarray:
    # 1 / (beta * (1/enc)), capped at FLT_MAX; zero where beta == 0
    # (reference/nvfp4.py:470-482).
    out = np.zeros_like(beta, dtype=np.float32)
    pos = beta > 0.0
    if np.any(pos):
        ginv = np.float32(1.0) / enc
        denom = (beta[pos] * ginv).astype(np.float32)
        with np.errstate(divide="ignore", over="ignore"):
            recip = (np.float32(1.0) / denom).astype(np.float32)
        out[pos] = np.minimum(recip, F32_MAX)
    return out


def quantize(source: np.ndarray) -> NVFP4Storage:
    """Quantize an FP32 matrix ``[N, K]`` (K % 16 == 0) (reference/nvfp4.py:500-536)."""
    src = np.ascontiguousarray(source, dtype=np.float32)
    if src.ndim != 2 or src.shape[1] % BLOCK != 0 or src.shape[1] < BLOCK:
        raise ValueError("source must be [N, K] with K a positive multiple of 16")
    if not np.all(np.isfinite(src)):
        raise ValueError("source must contain only finite values")
    rows, cols = src.shape
    enc, dec = global_scales(src)
    blocks = src.reshape(rows, cols // BLOCK, BLOCK)
    block_amax = np.max(np.abs(blocks), axis=-1).astype(np.float32)
    mult = np.float32(enc * np.float32(1.0 / E2M1_MAX))
    candidates = (block_amax * mult).astype(np.float32)
    scale_bytes = encode_ue4m3(candidates)
    beta = decode_ue4m3(scale_bytes)
    factors = _conversion_factors(enc, beta)
    codes = np.zeros(blocks.shape, dtype=np.uint8)
    pos = beta > 0.0
    if np.any(pos):
        pre = (blocks[pos] * factors[pos][:, None]).astype(np.float32)
        codes[pos] = encode_e2m1(pre)
    packed = pack_e2m1(codes.reshape(rows, cols))
    return NVFP4Storage(packed, scale_bytes, np.float32(dec), (rows, cols))


def dequantize(q: NVFP4Storage) -> np.ndarray:
    """FP32 ``(decode(q) * beta) * gamma`` (reference/nvfp4.py:539-554)."""
    rows, cols = q.logical_shape
    vals = decode_e2m1(unpack_e2m1(q.packed_values)).reshape(rows, cols // BLOCK, BLOCK)
    beta = decode_ue4m3(q.block_scales)
    block_scaled = (vals * beta[:, :, None]).astype(np.float32)
    return (block_scaled * np.float32(q.global_decode_scale)).astype(np.float32).reshape(rows, cols)
