"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

The reference publishes no dataset: every config is seeded synthetic data.
Distributions (per config): hidden states BF16 ~N(0,1); RMSNorm gains
1+N(0,0.05); Q/K/V/O weights FP32 ~N(0,0.02) (quantised to NVFP4 by the
caller); BF16 K/V caches ~N(0,1) in the physical ``[B, Hkv, C, D]`` layout.

All host-side draws use one ``torch.Generator('cpu')`` per case so the same
seed gives the same bytes on every machine running this torch build.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class DecodeShape:
    batch: int = 1
    tokens: int = 1
    hidden: int = 3072
    kv_heads: int = 6
    head_dim: int = 128
    capacity: int = 1024
    past_lengths: tuple[int, ...] = (511,)

    @property
    def q_heads(self) -> int:
        return self.hidden // self.head_dim

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim

    def past(self, b: int) -> int:
        return self.past_lengths[b] if len(self.past_lengths) > 1 else self.past_lengths[0]


# configs[0] of the benchmark: canonical single-token decode.
CANONICAL = DecodeShape()


def batched_shape(batch: int = 64, seed: int = 2024, lo: int = 1024, hi: int = 8191,
                  capacity: int = 8192) -> DecodeShape:
    """B sequences with P_b ~ U[lo, hi] (integers, seeded)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    p = torch.randint(lo, hi + 1, (batch,), generator=g).tolist()
    return DecodeShape(batch=batch, capacity=capacity, past_lengths=tuple(int(v) for v in p))


LONG_CONTEXT = DecodeShape(batch=8, capacity=32768, past_lengths=(32767,))
PREFILL = DecodeShape(batch=4, tokens=2048, capacity=4096, past_lengths=(0,))


@dataclass
class DecodeInputs:
    shape: DecodeShape
    x: torch.Tensor  # bf16 [B, T, H]
    input_norm_weight: torch.Tensor  # bf16 [H]
    q_norm_weight: torch.Tensor  # bf16 [D]
    k_norm_weight: torch.Tensor  # bf16 [D]
    weights_fp32: dict[str, torch.Tensor] = field(default_factory=dict)  # q,k,v,o
    k_cache: torch.Tensor | None = None  # bf16 [B, Hkv, C, D]
    v_cache: torch.Tensor | None = None


def make_decode_inputs(shape: DecodeShape, seed: int = 0, *, cache_device: str = "cpu",
                       with_caches: bool = True) -> DecodeInputs:
    g = torch.Generator(device="cpu").manual_seed(seed)
    h, d = shape.hidden, shape.head_dim
    x = torch.randn((shape.batch, shape.tokens, h), generator=g).to(torch.bfloat16)
    g_in = (1.0 + 0.05 * torch.randn((h,), generator=g)).to(torch.bfloat16)
    g_q = (1.0 + 0.05 * torch.randn((d,), generator=g)).to(torch.bfloat16)
    g_k = (1.0 + 0.05 * torch.randn((d,), generator=g)).to(torch.bfloat16)
    w = {
        "q": 0.02 * torch.randn((h, h), generator=g),
        "k": 0.02 * torch.randn((shape.kv_width, h), generator=g),
        "v": 0.02 * torch.randn((shape.kv_width, h), generator=g),
        "o": 0.02 * torch.randn((h, h), generator=g),
    }
    inputs = DecodeInputs(shape, x, g_in, g_q, g_k, w)
    if with_caches:
        cshape = (shape.batch, shape.kv_heads, shape.capacity, d)
        if cache_device == "cpu":
            inputs.k_cache = torch.randn(cshape, generator=g).to(torch.bfloat16)
            inputs.v_cache = torch.randn(cshape, generator=g).to(torch.bfloat16)
        else:
            gd = torch.Generator(device=cache_device).manual_seed(seed + 1)
            inputs.k_cache = torch.randn(cshape, generator=gd, device=cache_device,
                                         dtype=torch.bfloat16)
            inputs.v_cache = torch.randn(cshape, generator=gd, device=cache_device,
                                         dtype=torch.bfloat16)
    return inputs
