"""Python boundary of the B200 operator library (drop-in for the reference's
``cuda_primitives.py``, reference cuda_primitives.py:1-222).

Loads ``lib/cuda_primitives.so`` (or ``$CUDA_PRIMITIVES_LIBRARY``) with
``torch.ops.load_library``; a missing library raises ``ImportError`` — there is
no fallback implementation.  The wrappers have the reference's names,
arguments and error behaviour.  Weight arguments accept this package's
``NVFP4Tensor`` or the reference's (same four fields).
"""

from __future__ import annotations

import os
from pathlib import Path

import torch

from nvfp4_tensor import NVFP4Tensor, is_nvfp4_tensor, quantize_nvfp4  # noqa: F401

_PACKAGE_DIR = Path(__file__).resolve().parent
_LIBRARY_PATH = Path(os.environ.get("CUDA_PRIMITIVES_LIBRARY", _PACKAGE_DIR / "lib" / "cuda_primitives.so"))

if not _LIBRARY_PATH.is_file():
    raise ImportError(
        f"CUDA primitives library not found at {_LIBRARY_PATH}; "
        "run `python cuda-nvfp4-decoder-attention_b200/build.py` from the repository root"
    )

torch.ops.load_library(str(_LIBRARY_PATH))
_ops = torch.ops.cuda_nvfp4_decoder_attention
LIBRARY_PATH = _LIBRARY_PATH


def _require_weight(name: str, weight: object) -> None:
    if not is_nvfp4_tensor(weight):
        raise TypeError(f"{name} must be an NVFP4Tensor")
    derived = (weight.packed_values.shape[0], weight.packed_values.shape[1] * 2)
    if tuple(weight.logical_shape) != derived:
        raise ValueError(f"{name}.logical_shape must match packed_values-derived shape "
                         f"({tuple(weight.logical_shape)} != {derived})")


def _require_int(name: str, value: object) -> None:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError(f"{name} must be an integer")


def cuda_unpack_e2m1_codes(packed_values: torch.Tensor) -> torch.Tensor:
    """Unpack even-low, odd-high E2M1 bytes (reference cuda_primitives.py:30-36)."""
    return _ops.cuda_unpack_e2m1_codes(packed_values)


def cuda_dequantize_nvfp4(quantized) -> torch.Tensor:
    """Decode NVFP4 storage to FP32 ``(q * beta) * gamma`` (reference cuda_primitives.py:39-62)."""
    _require_weight("quantized", quantized)
    return _ops.cuda_dequantize_nvfp4(quantized.packed_values, quantized.block_scales,
                                      quantized.global_decode_scale)


def cuda_w4a16_linear(x: torch.Tensor, weight) -> torch.Tensor:
    """BF16 ``x @ W_hat.T`` with in-kernel NVFP4 decode (reference cuda_primitives.py:65-91)."""
    _require_weight("weight", weight)
    return _ops.cuda_w4a16_linear(x, weight.packed_values, weight.block_scales, weight.global_decode_scale)


def cuda_w4a16_linear_grouped_decode(x: torch.Tensor, weight) -> torch.Tensor:
    """Same projection under the reference's grouped-decode name (reference cuda_primitives.py:94-120)."""
    _require_weight("weight", weight)
    return _ops.cuda_w4a16_linear_grouped_decode(x, weight.packed_values, weight.block_scales,
                                                 weight.global_decode_scale)


def cuda_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last dimension (reference cuda_primitives.py:123-130)."""
    return _ops.cuda_rms_norm(x, weight, eps)


def cuda_apply_rope(x: torch.Tensor, past_length: int, rope_theta: float = 10000.0) -> torch.Tensor:
    """Adjacent-pair RoPE at positions ``past_length + t`` (reference cuda_primitives.py:133-144)."""
    return _ops.cuda_apply_rope(x, past_length, rope_theta)


def cuda_gqa_attention(q: torch.Tensor, present_k: torch.Tensor, present_v: torch.Tensor,
                       past_length: int) -> torch.Tensor:
    """Causal GQA over compact ``[B, Hkv, P+T, D]`` caches (reference cuda_primitives.py:147-161)."""
    _require_int("past_length", past_length)
    return _ops.cuda_gqa_attention(q, present_k, present_v, past_length)


def cuda_gqa_attention_cached(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                              past_length: int) -> torch.Tensor:
    """Causal GQA over physical ``[B, Hkv, C, D]`` caches (reference cuda_primitives.py:164-183)."""
    _require_int("past_length", past_length)
    return _ops.cuda_gqa_attention_cached(q, k_cache, v_cache, past_length)


def cuda_kv_cache_append_(k_cache: torch.Tensor, v_cache: torch.Tensor, new_k: torch.Tensor,
                          new_v: torch.Tensor, past_length: int) -> None:
    """Write token-major K/V into slots ``past_length ..`` in place (reference cuda_primitives.py:186-207)."""
    _require_int("past_length", past_length)
    _ops.cuda_kv_cache_append_(k_cache, v_cache, new_k, new_v, past_length)


__all__ = [
    "cuda_apply_rope",
    "cuda_dequantize_nvfp4",
    "cuda_gqa_attention",
    "cuda_gqa_attention_cached",
    "cuda_kv_cache_append_",
    "cuda_rms_norm",
    "cuda_unpack_e2m1_codes",
    "cuda_w4a16_linear",
    "cuda_w4a16_linear_grouped_decode",
    "quantize_nvfp4",
    "NVFP4Tensor",
]
