"""Portable NVFP4 weight storage and the device quantizer.

``NVFP4Tensor`` has the fields, shapes and validation of the reference's
``reference.nvfp4.NVFP4Tensor`` (reference/nvfp4.py:56-71, 163-232), so the
operators here accept either class: they read only the four fields.
``quantize_nvfp4`` runs the CUDA quantizer of ``lib/cuda_primitives.so``,
byte-exact with ``quantize_nvfp4_reference`` (reference/nvfp4.py:500-536).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

NVFP4_BLOCK_SIZE = 16


def _check_fields(packed_values, block_scales, global_decode_scale, logical_shape) -> None:
    if not isinstance(logical_shape, tuple) or len(logical_shape) != 2 or any(
            isinstance(v, bool) or not isinstance(v, int) for v in logical_shape):
        raise TypeError("logical_shape must be a tuple of two integers")
    rows, cols = logical_shape
    if rows < 1:
        raise ValueError(f"logical_shape N must be at least 1, got {rows}")
    if cols < NVFP4_BLOCK_SIZE or cols % NVFP4_BLOCK_SIZE:
        raise ValueError(f"logical_shape K must be a positive multiple of {NVFP4_BLOCK_SIZE}, got {cols}")
    for name, t in (("packed_values", packed_values), ("block_scales", block_scales),
                    ("global_decode_scale", global_decode_scale)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
    if block_scales.device != packed_values.device or global_decode_scale.device != packed_values.device:
        raise ValueError("NVFP4 fields must be on the same device")
    if packed_values.dtype != torch.uint8:
        raise TypeError(f"packed_values must have dtype torch.uint8, got {packed_values.dtype}")
    if block_scales.dtype != torch.uint8:
        raise TypeError(f"block_scales must have dtype torch.uint8, got {block_scales.dtype}")
    if global_decode_scale.dtype != torch.float32:
        raise TypeError(f"global_decode_scale must have dtype torch.float32, got {global_decode_scale.dtype}")
    if tuple(packed_values.shape) != (rows, cols // 2):
        raise ValueError(f"packed_values must have shape {(rows, cols // 2)}, got {tuple(packed_values.shape)}")
    if tuple(block_scales.shape) != (rows, cols // NVFP4_BLOCK_SIZE):
        raise ValueError(f"block_scales must have shape {(rows, cols // NVFP4_BLOCK_SIZE)}, "
                         f"got {tuple(block_scales.shape)}")
    if tuple(global_decode_scale.shape) != ():
        raise ValueError("global_decode_scale must be a scalar tensor with shape ()")
    if not packed_values.is_contiguous() or not block_scales.is_contiguous():
        raise ValueError("packed_values and block_scales must be contiguous")
    if bool((block_scales > 0x7E).any().item()):
        raise ValueError("block_scales must contain only canonical finite UE4M3 bytes in 0x00..0x7e")
    g = float(global_decode_scale.item())
    if not math.isfinite(g) or g < 0.0:
        raise ValueError(f"global_decode_scale must be finite and nonnegative, got {g}")


@dataclass(frozen=True)
class NVFP4Tensor:
    """One validated portable NVFP4 matrix ``W[N, K]``.

    ``packed_values`` uint8 ``[N, K/2]`` (even k in the low nibble),
    ``block_scales`` uint8 ``[N, K/16]`` (canonical UE4M3), ``global_decode_scale``
    float32 scalar, ``logical_shape`` ``(N, K)``.  Construction validates the
    contents once (host reads); the operators never re-scan device storage.
    """

    packed_values: torch.Tensor
    block_scales: torch.Tensor
    global_decode_scale: torch.Tensor
    logical_shape: tuple[int, int]

    def __post_init__(self) -> None:
        _check_fields(self.packed_values, self.block_scales, self.global_decode_scale, self.logical_shape)

    def to(self, device) -> "NVFP4Tensor":
        return NVFP4Tensor(self.packed_values.to(device), self.block_scales.to(device),
                           self.global_decode_scale.to(device), self.logical_shape)


def is_nvfp4_tensor(value: object) -> bool:
    """True for this class or any object with the reference NVFP4Tensor fields."""
    return isinstance(value, NVFP4Tensor) or all(
        hasattr(value, f) for f in ("packed_values", "block_scales", "global_decode_scale", "logical_shape"))


def quantize_nvfp4(source: torch.Tensor) -> NVFP4Tensor:
    """Quantize a CUDA FP32/BF16 matrix ``[N, K]`` on the device.

    Byte-exact with reference/nvfp4.py:500-536 (global amax scale, UE4M3 RNE
    block scales, E2M1 RNE codes).  The source must be finite.
    """
    import cuda_primitives  # noqa: F401  (loads the operator library)

    if not isinstance(source, torch.Tensor):
        raise TypeError("source must be a torch.Tensor")
    if source.device.type != "cuda":
        raise ValueError("source must be a CUDA tensor")
    packed, scales, gamma = torch.ops.cuda_nvfp4_decoder_attention.cuda_quantize_nvfp4(source)
    return NVFP4Tensor(packed, scales, gamma, (int(source.shape[0]), int(source.shape[1])))
