"""BF16 comparison metrics shared by the parity tests.

The adjacency distance is the number of representable BF16 values between two
results (0 = bit-identical value, 1 = neighbours), on the ordered-key mapping
the reference's own integration tests use (reference
tests/test_cuda_decoder_attention.py:43-64).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

# Tolerances, stated once.  Reference tests/test_cuda_decoder_attention.py:40 and
# tests/test_cuda_gqa_attention_cached.py:34-36.
ADJACENCY_FLOOR = 2.0 ** -20
ATTENTION_MAX_ABS = 2.0 ** -7
ATTENTION_MEAN_ABS = 2.0 ** -16
# End-to-end forward.  Any reordering of an FP32 sum can flip one BF16 rounding
# in an early stage (the reference's own torch CPU sum is not correctly
# rounded), and that flip propagates through the per-head norm, RoPE, the
# softmax and the O projection, so per-element adjacency is meaningless after
# the first stage.  Stated tolerance, relative to the expected tensor's own
# scale: max-abs <= 2^-6 * max|expected| (two BF16 ulps at the largest
# element), mean-abs <= 2^-8 * rms(expected), relative RMS error <= 2^-6.
E2E_MAX_REL = 2.0 ** -6
E2E_MEAN_REL = 2.0 ** -8
E2E_REL_RMS = 2.0 ** -6


def to_bits(a) -> np.ndarray:
    """Accept numpy uint16 bits or a torch bf16 tensor; return uint16 bits."""
    if hasattr(a, "dtype") and str(a.dtype) == "torch.bfloat16":
        import torch

        return a.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    return np.asarray(a, dtype=np.uint16)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def ordered_key(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16).astype(np.int64)
    neg = (b & 0x8000) != 0
    mag = b & 0x7FFF
    return np.where(neg, 0x8000 - mag, 0x8000 + mag)


@dataclass
class Bf16Metrics:
    max_abs: float
    mean_abs: float
    exact_fraction: float
    max_adjacency: int
    within_one_fraction: float

    def __str__(self) -> str:
        return (f"max_abs={self.max_abs:.3g} mean_abs={self.mean_abs:.3g} "
                f"exact={self.exact_fraction:.5f} max_adj={self.max_adjacency} "
                f"within1={self.within_one_fraction:.5f}")


def metrics(actual, expected) -> Bf16Metrics:
    a = to_bits(actual).reshape(-1)
    e = to_bits(expected).reshape(-1)
    assert a.shape == e.shape, (a.shape, e.shape)
    af, ef = bits_to_f32(a), bits_to_f32(e)
    assert np.all(np.isfinite(af)) and np.all(np.isfinite(ef))
    err = np.abs(af.astype(np.float64) - ef.astype(np.float64))
    adj = np.abs(ordered_key(a) - ordered_key(e))
    return Bf16Metrics(float(err.max(initial=0.0)), float(err.mean()) if err.size else 0.0,
                       float(np.mean(af == ef)) if a.size else 1.0,
                       int(adj.max(initial=0)), float(np.mean(adj <= 1)) if a.size else 1.0)


def assert_bitwise(actual, expected) -> None:
    a, e = to_bits(actual), to_bits(expected)
    assert a.shape == e.shape
    bad = np.flatnonzero(a.reshape(-1) != e.reshape(-1))
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}: {a.reshape(-1)[bad[:5]]} vs {e.reshape(-1)[bad[:5]]}"


def assert_stage_policy(actual, expected) -> Bf16Metrics:
    """Every element within one BF16 step, or within 2^-20 absolute."""
    m = metrics(actual, expected)
    a, e = to_bits(actual).reshape(-1), to_bits(expected).reshape(-1)
    err = np.abs(bits_to_f32(a).astype(np.float64) - bits_to_f32(e).astype(np.float64))
    adj = np.abs(ordered_key(a) - ordered_key(e))
    assert np.all((adj <= 1) | (err <= ADJACENCY_FLOOR)), str(m)
    return m


def assert_attention_policy(actual, expected) -> Bf16Metrics:
    m = assert_stage_policy(actual, expected)
    assert m.max_abs <= ATTENTION_MAX_ABS and m.mean_abs <= ATTENTION_MEAN_ABS, str(m)
    return m


def assert_e2e_policy(actual, expected) -> Bf16Metrics:
    m = metrics(actual, expected)
    a, e = to_bits(actual).reshape(-1), to_bits(expected).reshape(-1)
    ef = bits_to_f32(e).astype(np.float64)
    diff = bits_to_f32(a).astype(np.float64) - ef
    rel = float(np.sqrt(np.mean(diff * diff)) / max(np.sqrt(np.mean(ef * ef)), 1e-30)) if ef.size else 0.0
    scale_max = float(np.max(np.abs(ef), initial=0.0))
    scale_rms = float(np.sqrt(np.mean(ef * ef))) if ef.size else 0.0
    assert m.max_abs <= E2E_MAX_REL * scale_max, f"max-abs vs {scale_max:.3g}: {m}"
    assert m.mean_abs <= E2E_MEAN_REL * scale_rms, f"mean-abs vs rms {scale_rms:.3g}: {m}"
    assert rel <= E2E_REL_RMS, f"relative rms error {rel:.3g}: {m}"
    return m
