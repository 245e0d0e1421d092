"""GPU parity of the long-context decode attention (attn_stream_kernel: the
persistent TMA-fed tensor-core kernel the library takes once a sequence's
visible length reaches 2,048 positions) against the oracle.

Bar: the reference's attention policy (one BF16 step or 2^-20 per element,
max-abs <= 2^-7, mean-abs <= 2^-16; reference
tests/test_cuda_gqa_attention_cached.py:34-36).  Full-size configs[2] and
configs[3] caches are generated on the device and checked on sampled
sequences so that the oracle finishes in seconds.
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


def device_case(b, t, hq, hkv, d, c, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((b, t, hq, d), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((b, hkv, c, d), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((b, hkv, c, d), generator=g, device="cuda").to(torch.bfloat16)
    return q, k, v


def check_sequences(q, k, v, ctx, pl, seqs):
    for i in seqs:
        p = int(pl[i])
        s = p + q.shape[1]
        exp = oracle.gqa_attention(host_bits(q[i:i + 1]), host_bits(k[i:i + 1, :, :s]), host_bits(v[i:i + 1, :, :s]), p)
        assert_attention_policy(host_bits(ctx[i:i + 1]), exp)


def test_config3_long_context_full_size(capi):
    """B=8, T=1, P=32767, C=32768 on one GPU (sampled sequences)."""
    q, k, v = device_case(8, 1, 24, 6, 128, 32768, seed=33)
    ctx = capi.gqa_attention_cached(q, k, v, 32767)
    check_sequences(q, k, v, ctx, [32767] * 8, (0, 5, 7))


def test_config2_batched_ragged_full_size(capi):
    """B=64, P_b ~ U[1024, 8191] (seeded), C=8192 (sampled sequences)."""
    rng = np.random.default_rng(2)
    pl = rng.integers(1024, 8192, size=64).astype(np.int64)
    q, k, v = device_case(64, 1, 24, 6, 128, 8192, seed=22)
    ctx = capi.gqa_attention_cached(q, k, v, 0, past_lengths=torch.from_numpy(pl).cuda(),
                                    max_past_length=int(pl.max()))
    check_sequences(q, k, v, ctx, pl, (0, int(np.argmin(pl)), int(np.argmax(pl)), 31, 63))


def test_slots_past_the_causal_bound_are_never_used(capi):
    """NaN in every slot at or past P_b + T: the kernel reads whole 64-row
    tiles, so rows past the bound must not reach the softmax or the PV sum."""
    pl = np.array([2047, 2100, 4095, 3001], dtype=np.int64)
    b, t, hq, hkv, d, c = 4, 2, 8, 2, 128, 4160
    q, k, v = device_case(b, t, hq, hkv, d, c, seed=5)
    for i, p in enumerate(pl):
        k[i, :, p + t:] = float("nan")
        v[i, :, p + t:] = float("nan")
    ctx = capi.gqa_attention_cached(q, k, v, 0, past_lengths=torch.from_numpy(pl).cuda(),
                                    max_past_length=int(pl.max()))
    assert torch.isfinite(ctx.float()).all()
    check_sequences(q, k, v, ctx, pl, range(b))


@pytest.mark.parametrize("b,t,hq,hkv,d,p,c", [
    (2, 1, 8, 8, 64, 2500, 2600),      # D = 64, one query head per KV head
    (1, 1, 16, 2, 256, 3000, 3001),    # D = 256, 8 query heads per KV head, C = P + 1
    (1, 2, 8, 2, 128, 2111, 2113),     # T = 2: 8 query rows, per-token causal bound
    (3, 1, 24, 6, 128, 4095, 4096),    # a whole number of 64-position tiles
    (1, 1, 4, 1, 128, 65535, 65536),   # one pair, every SM on one sequence
])
def test_stream_shapes(capi, b, t, hq, hkv, d, p, c):
    q, k, v = device_case(b, t, hq, hkv, d, c, seed=b * 7 + p)
    ctx = capi.gqa_attention_cached(q, k, v, p)
    check_sequences(q, k, v, ctx, [p] * b, range(b))


def test_ragged_lengths_with_short_and_empty_sequences(capi):
    """Per-sequence lengths spanning 1 .. C on one launch: sequences shorter
    than one tile, exact tile multiples, and ones that straddle CTA ranges."""
    pl = np.array([0, 63, 64, 5000, 1, 4999, 127, 2048], dtype=np.int64)
    q, k, v = device_case(8, 1, 12, 3, 128, 5001, seed=9)
    ctx = capi.gqa_attention_cached(q, k, v, 0, past_lengths=torch.from_numpy(pl).cuda(), max_past_length=5000)
    check_sequences(q, k, v, ctx, pl, range(8))


def test_repeated_calls_are_bitwise_identical(capi):
    """The per-pair counters are left zero: every call combines the same way."""
    q, k, v = device_case(4, 1, 24, 6, 128, 9000, seed=4)
    first = host_bits(capi.gqa_attention_cached(q, k, v, 8999))
    for _ in range(3):
        assert_bitwise(host_bits(capi.gqa_attention_cached(q, k, v, 8999)), first)


def test_shard_partials_combine_to_the_unsharded_context(capi):
    """KV-length sharding: the partials of 4 shards of a 16,384-slot cache
    (each shard long enough for the streaming kernel), combined in shard
    order, match the oracle over the whole cache."""
    b, hq, hkv, d, c, p = 2, 24, 6, 128, 16384, 16000
    q, k, v = device_case(b, 1, hq, hkv, d, c, seed=44)
    from kv_sharding import CudaStages, shard_ranges

    st = CudaStages()
    parts = []
    for s in shard_ranges(c, 4):
        ks, vs = k[:, :, s.start:s.stop].contiguous(), v[:, :, s.start:s.stop].contiguous()
        parts.append(st.partials(q, ks, vs, s, p))
    ctx = st.combine(torch.stack(parts), q.shape)
    check_sequences(q, k, v, ctx, [p] * b, range(b))
