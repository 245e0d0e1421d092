"""The reference-facing Python API on the GPU: ``cuda_primitives`` wrappers and
``decoder_attention_cuda.cuda_decoder_attention_forward_`` behave like the
reference's (same names, shapes, in-place semantics, error messages), and
agree with the C-ABI kernels they wrap."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from bf16_metrics import assert_attention_policy, assert_bitwise, assert_e2e_policy, assert_stage_policy
from gpu_util import dev_bf16, dev_weight, golden_storage, host_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cp():
    import cuda_primitives

    return cuda_primitives


def test_wrappers_match_oracle(cp, golden_stages):
    g = golden_stages
    s = golden_storage(g, "lin0_")
    w = dev_weight(s)
    x = dev_bf16(g["lin0_x"])
    y = cp.cuda_w4a16_linear(x, w)
    assert y.shape == (1, 96) and y.dtype == torch.bfloat16 and y.is_contiguous()
    assert_stage_policy(host_bits(y), g["lin0_y"])
    assert_bitwise(host_bits(cp.cuda_w4a16_linear_grouped_decode(x, w)), host_bits(y))
    assert np.array_equal(cp.cuda_unpack_e2m1_codes(w.packed_values).cpu().numpy(),
                          oracle.unpack_e2m1(s.packed_values))
    assert np.array_equal(cp.cuda_dequantize_nvfp4(w).cpu().numpy().view(np.uint32),
                          oracle.dequantize(s).view(np.uint32))
    xr, wr = g["rms3_x"], g["rms3_w"]
    assert_bitwise(host_bits(cp.cuda_rms_norm(dev_bf16(xr), dev_bf16(wr), 1e-6)), oracle.rms_norm(xr, wr, 1e-6))
    xq = g["rope3_x"]
    assert_bitwise(host_bits(cp.cuda_apply_rope(dev_bf16(xq), 511, 10000.0)), oracle.apply_rope(xq, 511, 1e4))


def test_compact_and_cached_attention(cp, golden_stages):
    g = golden_stages
    q, k, v, p = g["att3_q"], g["att3_k"], g["att3_v"], int(g["att3_p"])
    t = q.shape[1]
    ctx = cp.cuda_gqa_attention_cached(dev_bf16(q), dev_bf16(k), dev_bf16(v), p)
    assert_attention_policy(host_bits(ctx), g["att3_ctx"])
    kc = np.ascontiguousarray(k[:, :, :p + t])
    vc = np.ascontiguousarray(v[:, :, :p + t])
    ctx2 = cp.cuda_gqa_attention(dev_bf16(q), dev_bf16(kc), dev_bf16(vc), p)
    assert_bitwise(host_bits(ctx2), host_bits(ctx))
    with pytest.raises(RuntimeError, match="cache context length must equal"):
        cp.cuda_gqa_attention(dev_bf16(q), dev_bf16(k), dev_bf16(v), p)
    with pytest.raises(RuntimeError, match="exceeds cache capacity"):
        cp.cuda_gqa_attention_cached(dev_bf16(q), dev_bf16(k), dev_bf16(v), k.shape[2])


def test_kv_append_is_in_place_and_returns_none(cp):
    kc = torch.zeros((1, 2, 8, 4), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    nk = torch.ones((1, 1, 2, 4), dtype=torch.bfloat16, device="cuda")
    ptr = kc.data_ptr()
    assert cp.cuda_kv_cache_append_(kc, vc, nk, nk * 2, 3) is None
    assert kc.data_ptr() == ptr
    assert torch.equal(kc[0, :, 3], nk[0, 0]) and torch.equal(vc[0, :, 3], 2 * nk[0, 0])
    assert float(kc.float().sum()) == 8.0
    with pytest.raises(RuntimeError, match="exceeds cache capacity"):
        cp.cuda_kv_cache_append_(kc, vc, nk, nk, 8)
    with pytest.raises(RuntimeError, match="past_length must be nonnegative"):
        cp.cuda_kv_cache_append_(kc, vc, nk, nk, -1)


@pytest.mark.parametrize("call,match", [
    (lambda cp, x, w: cp.cuda_rms_norm(x.float(), w, 1e-6), "x must have dtype torch.bfloat16"),
    (lambda cp, x, w: cp.cuda_rms_norm(x, w[:4], 1e-6), "weight length must match"),
    (lambda cp, x, w: cp.cuda_rms_norm(x, w, float("inf")), "eps must be finite and positive"),
    (lambda cp, x, w: cp.cuda_rms_norm(x, w, 1e-300), "eps must be representable as a finite positive FP32 value"),
    (lambda cp, x, w: cp.cuda_apply_rope(x, 0), "x must have rank 4"),
    (lambda cp, x, w: cp.cuda_apply_rope(x.reshape(1, 1, 1, 8), -1), "past_length must be nonnegative"),
    (lambda cp, x, w: cp.cuda_apply_rope(x.reshape(1, 1, 1, 8), 1, 0.0), "rope_theta must be finite and positive"),
    (lambda cp, x, w: cp.cuda_rms_norm(x[..., ::2], w[::2], 1e-6), "x must be contiguous"),
])
def test_validation_messages_match_reference(cp, call, match):
    x = torch.ones((1, 1, 8), dtype=torch.bfloat16, device="cuda")
    w = torch.ones(8, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match=match):
        call(cp, x, w)


def test_quantize_nvfp4_returns_validated_tensor(golden_format):
    from nvfp4_tensor import NVFP4Tensor, quantize_nvfp4

    q = quantize_nvfp4(torch.from_numpy(golden_format["q_rand_src"]).cuda())
    assert isinstance(q, NVFP4Tensor)
    assert np.array_equal(q.packed_values.cpu().numpy(), golden_format["q_rand_packed"])
    assert np.array_equal(q.block_scales.cpu().numpy(), golden_format["q_rand_scales"])


def test_forward_drop_in_matches_capi_and_golden(golden_forward):
    import decoder_attention_cuda as dac

    g = golden_forward
    name = "fwd_decode_b2"
    b, t, h, hkv, d, p, c, _ = (int(v) for v in g[f"{name}_shape"])
    ws = {k: dev_weight(golden_storage(g, f"{name}_w{k}_")) for k in "qkvo"}
    kc, vc = dev_bf16(g[f"{name}_k_cache"]), dev_bf16(g[f"{name}_v_cache"])
    kptr = kc.data_ptr()
    out = dac.cuda_decoder_attention_forward_(
        dev_bf16(g[f"{name}_x"]), dev_bf16(g[f"{name}_g_in"]), ws["q"], ws["k"], ws["v"],
        dev_bf16(g[f"{name}_g_q"]), dev_bf16(g[f"{name}_g_k"]), ws["o"], kc, vc, p)
    assert out.shape == (b, t, h) and out.dtype == torch.bfloat16
    assert kc.data_ptr() == kptr
    assert_e2e_policy(host_bits(out), g[f"{name}_output"])
    assert_e2e_policy(host_bits(kc)[:, :, p:p + t], g[f"{name}_new_k"])
    assert_bitwise(host_bits(vc)[:, :, :p], g[f"{name}_v_cache"][:, :, :p])


def test_forward_rejects_bad_metadata_before_launch(golden_forward):
    import decoder_attention_cuda as dac

    g = golden_forward
    name = "fwd_decode_b2"
    ws = {k: dev_weight(golden_storage(g, f"{name}_w{k}_")) for k in "qkvo"}
    x, g_in = dev_bf16(g[f"{name}_x"]), dev_bf16(g[f"{name}_g_in"])
    g_q, g_k = dev_bf16(g[f"{name}_g_q"]), dev_bf16(g[f"{name}_g_k"])
    kc, vc = dev_bf16(g[f"{name}_k_cache"]), dev_bf16(g[f"{name}_v_cache"])
    before = host_bits(kc)
    with pytest.raises(ValueError, match="exceeds cache capacity"):
        dac.cuda_decoder_attention_forward_(x, g_in, ws["q"], ws["k"], ws["v"], g_q, g_k, ws["o"], kc, vc, 64)
    with pytest.raises(TypeError, match="q_weight must be an NVFP4Tensor"):
        dac.cuda_decoder_attention_forward_(x, g_in, object(), ws["k"], ws["v"], g_q, g_k, ws["o"], kc, vc, 1)
    with pytest.raises(ValueError, match="input_norm_weight must have shape"):
        dac.cuda_decoder_attention_forward_(x, g_in[:-2].contiguous(), ws["q"], ws["k"], ws["v"], g_q, g_k, ws["o"],
                                            kc, vc, 1)
    with pytest.raises(ValueError, match="q_weight.logical_shape"):
        dac.cuda_decoder_attention_forward_(x, g_in, ws["o"].__class__(ws["k"].packed_values, ws["k"].block_scales,
                                                                       ws["k"].global_decode_scale,
                                                                       tuple(ws["k"].logical_shape)),
                                            ws["k"], ws["v"], g_q, g_k, ws["o"], kc, vc, 1)
    assert_bitwise(host_bits(kc), before)
