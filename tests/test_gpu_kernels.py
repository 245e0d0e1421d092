"""GPU parity of every kernel behind the C ABI against the oracle and the
reference's golden vectors.

Bars: storage decode, quantizer and cache append bit-exact; RMSNorm and RoPE
bit-exact against the oracle (both evaluate the correctly rounded FP32 sums and
trig) and within one BF16 step of the reference; W4A16 within one BF16 step (or
2^-20); attention per the reference's attention policy (one step or 2^-20,
max-abs <= 2^-7, mean-abs <= 2^-16).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from bf16_metrics import assert_attention_policy, assert_bitwise, assert_stage_policy
from gpu_util import dev_bf16, dev_weight, golden_storage, host_bits, storage_sha

pytestmark = pytest.mark.gpu

QUANT_CASES = ["q_rand", "q_zero", "q_zero_block", "q_local_underflow", "q_global_tiny", "q_bf16", "q_wide"]


@pytest.fixture(scope="module")
def capi():
    import nvfp4da_capi

    nvfp4da_capi.load()
    return nvfp4da_capi


# ------------------------------------------------------------------ storage format
@pytest.mark.parametrize("case", QUANT_CASES)
def test_unpack_and_dequantize_are_bit_exact(capi, golden_format, case):
    s = golden_storage(golden_format, case + "_")
    w = dev_weight(s)
    codes = capi.unpack(w.packed_values).cpu().numpy()
    assert np.array_equal(codes, oracle.unpack_e2m1(s.packed_values))
    deq = capi.dequantize(w).cpu().numpy()
    assert np.array_equal(deq.view(np.uint32), oracle.dequantize(s).view(np.uint32))


def test_every_byte_and_every_scale_code_decodes_exactly(capi):
    """All 256 packed bytes under all 127 canonical scale codes, gamma = 6/2688."""
    rows = 127
    packed = np.tile(np.arange(256, dtype=np.uint8), (rows, 1))  # K = 512
    scales = np.repeat(np.arange(127, dtype=np.uint8)[:, None], 512 // 16, axis=1)
    s = oracle.NVFP4Storage(packed, scales, np.float32(6.0 / 2688.0), (rows, 512))
    deq = capi.dequantize(dev_weight(s)).cpu().numpy()
    ref = oracle.dequantize(s)
    assert np.array_equal(deq.view(np.uint32), ref.view(np.uint32))
    # byte 0x80 (column 0x80) holds code 0x8 in its high nibble: -0.0
    assert np.signbit(deq[0, 2 * 0x80 + 1]) and deq[0, 2 * 0x80 + 1] == 0.0


@pytest.mark.parametrize("case", QUANT_CASES)
def test_quantizer_is_byte_exact_with_reference(capi, golden_format, case):
    g = golden_format
    if case + "_src_bf16" in g:
        src = dev_bf16(g[case + "_src_bf16"])
    else:
        src = torch.from_numpy(g[case + "_src"]).cuda()
    packed, scales, gamma = capi.quantize(src)
    assert np.array_equal(packed.cpu().numpy(), g[case + "_packed"])
    assert np.array_equal(scales.cpu().numpy(), g[case + "_scales"])
    assert np.float32(gamma.item()).view(np.uint32) == np.float32(g[case + "_gamma"]).view(np.uint32)


def test_quantizer_reproduces_canonical_weights(capi, golden_canonical):
    import synthetic

    inp = synthetic.make_decode_inputs(synthetic.CANONICAL, seed=0, with_caches=False)
    for key, w in inp.weights_fp32.items():
        packed, scales, gamma = capi.quantize(w.cuda())
        s = oracle.NVFP4Storage(packed.cpu().numpy(), scales.cpu().numpy(), np.float32(gamma.item()),
                                tuple(w.shape))
        assert storage_sha(s) == str(golden_canonical[f"c0_w{key}_sha256"]), key


# ------------------------------------------------------------------ W4A16
@pytest.mark.parametrize("i", range(4))
def test_w4a16_matches_reference_golden(capi, golden_stages, i):
    g = golden_stages
    s = golden_storage(g, f"lin{i}_")
    y = host_bits(capi.w4a16_linear(dev_bf16(g[f"lin{i}_x"]), dev_weight(s)))
    assert_stage_policy(y, g[f"lin{i}_y"])
    assert_stage_policy(y, oracle.w4a16_linear(g[f"lin{i}_x"], s))


SWEEP = [(m, n, k) for m in (1, 4, 16) for (n, k) in ((4608, 3072), (3072, 3072), (768, 3072), (3072, 128))]


@pytest.mark.parametrize("m,n,k", SWEEP)
def test_w4a16_projection_sweep_matches_oracle(capi, m, n, k):
    """M in {1,4,16} x the decoder's projection shapes."""
    gen = torch.Generator().manual_seed(1000 + m * 7 + n + k)
    x = torch.randn((m, k), generator=gen).to(torch.bfloat16)
    s = oracle.quantize((0.02 * torch.randn((n, k), generator=gen)).numpy())
    xb = host_bits(x)
    y = host_bits(capi.w4a16_linear(x.cuda(), dev_weight(s)))
    m_ = assert_stage_policy(y, oracle.w4a16_linear(xb, s))
    assert m_.exact_fraction > 0.95, str(m_)


@pytest.mark.parametrize("m,n,k", [(9, 4608, 3072), (24, 768, 3072), (33, 3072, 3072), (64, 3072, 3072),
                                   (64, 4608, 1024), (17, 256, 2048)])
def test_w4a16_batched_rows_match_oracle(capi, m, n, k):
    """8 < M <= 64 (the batched kernel: each weight fragment decoded once for
    all rows), including row counts that leave part of the last n-tile empty."""
    gen = torch.Generator().manual_seed(2000 + m + n + k)
    x = torch.randn((m, k), generator=gen).to(torch.bfloat16)
    s = oracle.quantize((0.02 * torch.randn((n, k), generator=gen)).numpy())
    xb = host_bits(x)
    y = capi.w4a16_linear(x.cuda(), dev_weight(s))
    again = capi.w4a16_linear(x.cuda(), dev_weight(s))
    assert torch.equal(y.view(torch.int16), again.view(torch.int16))  # deterministic
    m_ = assert_stage_policy(host_bits(y), oracle.w4a16_linear(xb, s))
    assert m_.exact_fraction > 0.95, str(m_)


def test_w4a16_one_hot_weights_are_exact(capi):
    """Code 0x2 (1.0) at one input per output row, scale 0x38 (1.0), gamma 1:
    y[m, n] == x[m, (n + 3) % K] bit-for-bit (orientation and nibble order)."""
    n, k, m = 96, 256, 5
    codes = np.zeros((n, k), dtype=np.uint8)
    codes[np.arange(n), (np.arange(n) + 3) % k] = 0x2
    s = oracle.NVFP4Storage(oracle.pack_e2m1(codes), np.full((n, k // 16), 0x38, np.uint8), np.float32(1.0),
                            (n, k))
    x = (torch.randn((m, k), generator=torch.Generator().manual_seed(5)) * 3).to(torch.bfloat16)
    y = host_bits(capi.w4a16_linear(x.cuda(), dev_weight(s)))
    assert_bitwise(y, host_bits(x)[:, (np.arange(n) + 3) % k])


def test_w4a16_every_code_and_scale_inside_projection(capi):
    """Row r has a single nonzero weight with code r % 16 and scale r % 127, so
    the output is exactly BF16(x_j * q * beta * gamma)."""
    n, k = 127 * 2, 64
    codes = np.zeros((n, k), dtype=np.uint8)
    col = np.arange(n) % k
    codes[np.arange(n), col] = np.arange(n) % 16
    scales = np.tile((np.arange(n) % 127).astype(np.uint8)[:, None], (1, k // 16))
    s = oracle.NVFP4Storage(oracle.pack_e2m1(codes), scales, np.float32(1.0), (n, k))
    x = torch.full((1, k), 1.5, dtype=torch.bfloat16)
    y = host_bits(capi.w4a16_linear(x.cuda(), dev_weight(s)))
    assert_bitwise(y, oracle.w4a16_linear(host_bits(x), s))


def test_w4a16_zero_inputs_zero_weights_and_zero_blocks(capi):
    n, k = 32, 128
    s = oracle.quantize((torch.randn((n, k), generator=torch.Generator().manual_seed(9)) * 0.02).numpy())
    zero = oracle.NVFP4Storage(np.zeros_like(s.packed_values), np.zeros_like(s.block_scales), np.float32(0.0),
                               (n, k))
    x = torch.randn((2, k), generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
    y0 = host_bits(capi.w4a16_linear(torch.zeros_like(x).cuda(), dev_weight(s)))
    assert np.all(oracle.bf16_to_f32(y0) == 0.0)
    y = host_bits(capi.w4a16_linear(x.cuda(), dev_weight(zero)))
    assert np.all(oracle.bf16_to_f32(y) == 0.0)


# ------------------------------------------------------------------ RMSNorm / RoPE
@pytest.mark.parametrize("i", range(5))
def test_rms_norm_matches_oracle_bitwise_and_reference(capi, golden_stages, i):
    g = golden_stages
    x, w = g[f"rms{i}_x"], g[f"rms{i}_w"]
    y = host_bits(capi.rms_norm(dev_bf16(x), dev_bf16(w), 1e-6))
    assert_bitwise(y, oracle.rms_norm(x, w, 1e-6))
    assert_stage_policy(y, g[f"rms{i}_y"])


@pytest.mark.parametrize("i", range(6))
def test_rope_matches_oracle_bitwise_and_reference(capi, golden_stages, i):
    g = golden_stages
    x, p, th = g[f"rope{i}_x"], int(g[f"rope{i}_p"]), float(g[f"rope{i}_theta"])
    y = host_bits(capi.apply_rope(dev_bf16(x), p, th))
    assert_bitwise(y, oracle.apply_rope(x, p, th))
    assert_stage_policy(y, g[f"rope{i}_y"])


def test_rope_position_zero_is_a_storage_copy(capi):
    x = (torch.randn((2, 1, 5, 8), generator=torch.Generator().manual_seed(3)) * 0.75).to(torch.bfloat16)
    x[0, 0, 0, 0] = 0.0
    x[0, 0, 0, 1] = -0.0
    assert_bitwise(host_bits(capi.apply_rope(x.cuda(), 0, 1e4)), host_bits(x))


# ------------------------------------------------------------------ KV append
def test_kv_append_layout_prefix_suffix_and_signed_zero(capi):
    b, hkv, c, d, t, p = 2, 3, 19, 8, 4, 5
    kc = torch.full((b, hkv, c, d), -31.0, dtype=torch.bfloat16)
    vc = torch.full((b, hkv, c, d), 47.0, dtype=torch.bfloat16)
    nk = torch.randn((b, t, hkv, d), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    nv = torch.randn((b, t, hkv, d), generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    nk[0, 0, 0, 0] = -0.0
    kd, vd = kc.cuda(), vc.cuda()
    ptr = kd.data_ptr()
    capi.kv_cache_append(kd, vd, nk.cuda(), nv.cuda(), p)
    assert kd.data_ptr() == ptr
    ek, ev = kc.clone(), vc.clone()
    ek[:, :, p:p + t] = nk.permute(0, 2, 1, 3)
    ev[:, :, p:p + t] = nv.permute(0, 2, 1, 3)
    assert_bitwise(host_bits(kd), host_bits(ek))
    assert_bitwise(host_bits(vd), host_bits(ev))


def test_kv_append_per_sequence_slots(capi):
    b, hkv, c, d = 3, 2, 16, 8
    kc = torch.zeros((b, hkv, c, d), dtype=torch.bfloat16).cuda()
    vc = torch.zeros_like(kc)
    nk = torch.randn((b, 1, hkv, d), generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    pl = torch.tensor([0, 7, 15], dtype=torch.int64)
    capi.kv_cache_append(kc, vc, nk.cuda(), nk.cuda(), 0, past_lengths=pl.cuda())
    host = kc.cpu()
    for i in range(b):
        assert torch.equal(host[i, :, int(pl[i])], nk[i, 0])
        assert int(torch.count_nonzero(host[i].float())) == int(torch.count_nonzero(nk[i].float()))


# ------------------------------------------------------------------ attention
@pytest.mark.parametrize("i", range(5))
def test_attention_matches_reference_golden(capi, golden_stages, i):
    g = golden_stages
    q, k, v, p = g[f"att{i}_q"], g[f"att{i}_k"], g[f"att{i}_v"], int(g[f"att{i}_p"])
    ctx = host_bits(capi.gqa_attention_cached(dev_bf16(q), dev_bf16(k), dev_bf16(v), p))
    assert_attention_policy(ctx, g[f"att{i}_ctx"])
    assert_attention_policy(ctx, oracle.gqa_attention(q, k, v, p))


def attention_case(b, t, hq, hkv, d, p, c, seed, sentinel=True):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn((b, t, hq, d), generator=gen).to(torch.bfloat16)
    k = torch.randn((b, hkv, c, d), generator=gen).to(torch.bfloat16)
    v = torch.randn((b, hkv, c, d), generator=gen).to(torch.bfloat16)
    if sentinel:  # slots beyond P+T must never be read
        k[:, :, p + t:] = 9000.0
        v[:, :, p + t:] = -7000.0
    return host_bits(q), host_bits(k), host_bits(v)


@pytest.mark.parametrize("b,t,hq,hkv,d,p,c", [
    (1, 1, 24, 6, 128, 511, 1024),   # configs[0]
    (2, 1, 24, 6, 128, 4000, 4097),  # many splits
    (1, 4, 8, 2, 64, 10, 20),        # T > 1, future slots hidden
    (2, 3, 6, 3, 16, 0, 5),          # P = 0
    (1, 1, 16, 2, 256, 300, 310),    # D = 256, 8 heads per KV head
    (1, 2, 3, 1, 2, 6, 9),           # tiny head dimension, odd group
])
def test_attention_capacity_stride_and_causality(capi, b, t, hq, hkv, d, p, c):
    q, k, v = attention_case(b, t, hq, hkv, d, p, c, seed=b * 131 + p)
    ctx = host_bits(capi.gqa_attention_cached(dev_bf16(q), dev_bf16(k), dev_bf16(v), p))
    assert_attention_policy(ctx, oracle.gqa_attention(q, k, v, p))


def test_attention_per_sequence_lengths(capi):
    b, hq, hkv, d, c = 4, 8, 2, 128, 3000
    pl = np.array([5, 2999, 1024, 0], dtype=np.int64)
    q, k, v = attention_case(b, 1, hq, hkv, d, 0, c, seed=77, sentinel=False)
    ctx = host_bits(capi.gqa_attention_cached(dev_bf16(q), dev_bf16(k), dev_bf16(v), 0,
                                              past_lengths=torch.from_numpy(pl).cuda(), max_past_length=2999))
    for i in range(b):
        exp = oracle.gqa_attention(q[i:i + 1], k[i:i + 1], v[i:i + 1], int(pl[i]))
        assert_attention_policy(ctx[i:i + 1], exp)


def test_attention_long_context_config3_slice(capi):
    """configs[3] shape (P = 32767, C = 32768) on one sequence."""
    q, k, v = attention_case(1, 1, 24, 6, 128, 32767, 32768, seed=3, sentinel=False)
    ctx = host_bits(capi.gqa_attention_cached(dev_bf16(q), dev_bf16(k), dev_bf16(v), 32767))
    assert_attention_policy(ctx, oracle.gqa_attention(q, k, v, 32767))


def test_attention_repeated_calls_reuse_cleared_counters(capi):
    q, k, v = attention_case(1, 1, 24, 6, 128, 2047, 2048, seed=12, sentinel=False)
    qd, kd, vd = dev_bf16(q), dev_bf16(k), dev_bf16(v)
    first = host_bits(capi.gqa_attention_cached(qd, kd, vd, 2047))
    for _ in range(3):
        assert_bitwise(host_bits(capi.gqa_attention_cached(qd, kd, vd, 2047)), first)
