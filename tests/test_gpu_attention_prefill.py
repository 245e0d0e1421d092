"""GPU parity of the tcgen05 causal prefill attention (attn_prefill_tc_kernel,
taken for T >= 64 at head_dim 128) against the oracle.

Bar: the reference's attention policy (one BF16 step or 2^-20 per element,
max-abs <= 2^-7, mean-abs <= 2^-16; reference
tests/test_cuda_gqa_attention_cached.py:34-36).  Cases: whole and partial
128-row query tiles, a prompt prefix (P > 0), per-sequence lengths, a cache
with NaN in every slot past P_b + T (the kernel loads whole 64-key tiles),
and GQA groups of 1, 3 and 4.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from bf16_metrics import assert_attention_policy, assert_bitwise
from gpu_util import host_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def capi():
    import nvfp4da_capi

    nvfp4da_capi.load()
    return nvfp4da_capi


def device_case(b, t, hq, hkv, c, seed, d=128):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((b, t, hq, d), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((b, hkv, c, d), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((b, hkv, c, d), generator=g, device="cuda").to(torch.bfloat16)
    return q, k, v


def check(q, k, v, ctx, pl, seqs=None):
    t = q.shape[1]
    for i in (range(q.shape[0]) if seqs is None else seqs):
        p = int(pl[i])
        exp = oracle.gqa_attention(host_bits(q[i:i + 1]), host_bits(k[i:i + 1, :, :p + t]),
                                   host_bits(v[i:i + 1, :, :p + t]), p)
        assert_attention_policy(host_bits(ctx[i:i + 1]), exp)


@pytest.mark.parametrize("b,t,hq,hkv,p,c", [
    (1, 128, 8, 2, 0, 128),     # one whole query tile, C = T
    (1, 64, 4, 4, 0, 100),      # half a tile, one query head per KV head
    (2, 200, 6, 2, 37, 300),    # partial second tile, prompt prefix, group of 3
    (1, 513, 24, 6, 0, 640),    # configs[4] head configuration, ragged tail
])
def test_prefill_attention_matches_oracle(capi, b, t, hq, hkv, p, c):
    q, k, v = device_case(b, t, hq, hkv, c, seed=b * 100 + t + p)
    ctx = capi.gqa_attention_cached(q, k, v, p)
    check(q, k, v, ctx, [p] * b)


def test_prefill_slots_past_the_causal_bound_are_never_used(capi):
    pl = np.array([0, 70, 5], dtype=np.int64)
    b, t, c = 3, 130, 260
    q, k, v = device_case(b, t, 8, 2, c, seed=12)
    for i, p in enumerate(pl):
        k[i, :, p + t:] = float("nan")
        v[i, :, p + t:] = float("nan")
    ctx = capi.gqa_attention_cached(q, k, v, 0, past_lengths=torch.from_numpy(pl).cuda(),
                                    max_past_length=int(pl.max()))
    assert torch.isfinite(ctx.float()).all()
    check(q, k, v, ctx, pl)


def test_prefill_config4_full_size_sampled(capi):
    """configs[4] shape (B=4, T=2048, Hq=24, Hkv=6, C=4096), two sequences checked."""
    q, k, v = device_case(4, 2048, 24, 6, 4096, seed=4)
    ctx = capi.gqa_attention_cached(q, k, v, 0)
    check(q, k, v, ctx, [0] * 4, seqs=(0, 3))


def test_prefill_attention_is_deterministic(capi):
    q, k, v = device_case(2, 300, 8, 2, 512, seed=3)
    first = host_bits(capi.gqa_attention_cached(q, k, v, 10))
    assert_bitwise(host_bits(capi.gqa_attention_cached(q, k, v, 10)), first)
