"""Helpers for the GPU parity tests: move golden/oracle arrays (BF16 as uint16
bits, NVFP4 fields as uint8) onto the device and back."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from oracle.nvfp4 import NVFP4Storage

CUDA = torch.cuda.is_available()
requires_cuda = pytest.mark.skipif(not CUDA, reason="needs a CUDA device")


def dev_bf16(bits: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)
    return torch.from_numpy(a.copy()).view(torch.bfloat16).cuda()


def host_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def dev_weight(s: NVFP4Storage):
    from nvfp4_tensor import NVFP4Tensor

    return NVFP4Tensor(torch.from_numpy(np.ascontiguousarray(s.packed_values)).cuda(),
                       torch.from_numpy(np.ascontiguousarray(s.block_scales)).cuda(),
                       torch.tensor(np.float32(s.global_decode_scale), dtype=torch.float32).cuda(),
                       tuple(int(v) for v in s.logical_shape))


def host_storage(w) -> NVFP4Storage:
    return NVFP4Storage(w.packed_values.cpu().numpy(), w.block_scales.cpu().numpy(),
                        np.float32(w.global_decode_scale.item()), tuple(int(v) for v in w.logical_shape))


def storage_sha(s: NVFP4Storage) -> str:
    h = hashlib.sha256()
    for a in (s.packed_values, s.block_scales, np.float32(s.global_decode_scale)):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def golden_storage(g: dict, prefix: str) -> NVFP4Storage:
    packed = g[prefix + "packed"]
    return NVFP4Storage(packed, g[prefix + "scales"], np.float32(g[prefix + "gamma"]),
                        (packed.shape[0], packed.shape[1] * 2))
