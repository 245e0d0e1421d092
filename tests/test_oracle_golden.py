"""Pin the numpy oracle against vectors the reference itself produced.

CPU only.  Storage format, quantizer and cache append are bit-exact; FP32
stages rounded to BF16 are compared under the reference's own stage policy
(within one BF16 step or 2^-20), and the fraction of bit-identical elements is
required to be high so that a systematic difference cannot hide in the
tolerance.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

import oracle
from bf16_metrics import (assert_attention_policy, assert_bitwise, assert_e2e_policy,
                          assert_stage_policy, metrics)
from oracle.nvfp4 import NVFP4Storage


def storage(g: dict, prefix: str) -> NVFP4Storage:
    packed = g[prefix + "packed"]
    return NVFP4Storage(packed, g[prefix + "scales"], np.float32(g[prefix + "gamma"]),
                        (packed.shape[0], packed.shape[1] * 2))


# ------------------------------------------------------------------ format
def test_e2m1_decode_table_matches_reference(golden_format):
    dec = oracle.decode_e2m1(np.arange(16, dtype=np.uint8))
    assert np.array_equal(dec.view(np.uint32), golden_format["e2m1_decode"].view(np.uint32))
    assert np.array_equal(np.signbit(dec), golden_format["e2m1_decode_signbit"])
    assert np.signbit(dec[8]) and dec[8] == 0.0  # code 0x8 is -0.0


def test_every_canonical_ue4m3_byte_matches_reference(golden_format):
    dec = oracle.decode_ue4m3(np.arange(0x7F, dtype=np.uint8))
    assert np.array_equal(dec.view(np.uint32), golden_format["ue4m3_decode"].view(np.uint32))
    with pytest.raises(ValueError):
        oracle.decode_ue4m3(np.array([0x7F], dtype=np.uint8))
    with pytest.raises(ValueError):
        oracle.decode_ue4m3(np.array([0x80], dtype=np.uint8))


def test_e2m1_encoder_midpoints_and_saturation_match_reference(golden_format):
    codes = oracle.encode_e2m1(golden_format["e2m1_probe"])
    assert np.array_equal(codes, golden_format["e2m1_code"])


def test_ue4m3_encoder_midpoints_and_saturation_match_reference(golden_format):
    codes = oracle.encode_ue4m3(golden_format["ue4m3_probe"])
    assert np.array_equal(codes, golden_format["ue4m3_code"])


@pytest.mark.parametrize("case", ["q_rand", "q_zero", "q_zero_block", "q_local_underflow",
                                  "q_global_tiny", "q_bf16", "q_wide"])
def test_quantizer_is_byte_exact_with_reference(golden_format, case):
    g = golden_format
    if case + "_src_bf16" in g:
        src = oracle.bf16_to_f32(g[case + "_src_bf16"])
    else:
        src = g[case + "_src"]
    q = oracle.quantize(src)
    assert np.array_equal(q.packed_values, g[case + "_packed"])
    assert np.array_equal(q.block_scales, g[case + "_scales"])
    assert np.float32(q.global_decode_scale).view(np.uint32) == np.float32(g[case + "_gamma"]).view(np.uint32)


def test_pack_unpack_round_trip_and_nibble_order():
    codes = np.arange(32, dtype=np.uint8).reshape(2, 16) % 16
    packed = oracle.pack_e2m1(codes)
    assert packed[0, 0] == (0x0 | (0x1 << 4))  # even element low, odd high
    assert np.array_equal(oracle.unpack_e2m1(packed), codes)


# ------------------------------------------------------------------ stages
@pytest.mark.parametrize("i", range(4))
def test_w4a16_projection_matches_reference(golden_stages, i):
    g = golden_stages
    y = oracle.w4a16_linear(g[f"lin{i}_x"], storage(g, f"lin{i}_"))
    m = assert_stage_policy(y, g[f"lin{i}_y"])
    assert m.exact_fraction >= 0.98, str(m)


@pytest.mark.parametrize("i", range(5))
def test_rms_norm_matches_reference(golden_stages, i):
    g = golden_stages
    y = oracle.rms_norm(g[f"rms{i}_x"], g[f"rms{i}_w"], 1e-6)
    m = assert_stage_policy(y, g[f"rms{i}_y"])
    assert m.exact_fraction >= 0.99, str(m)


@pytest.mark.parametrize("i", range(6))
def test_rope_matches_reference(golden_stages, i):
    g = golden_stages
    y = oracle.apply_rope(g[f"rope{i}_x"], int(g[f"rope{i}_p"]), float(g[f"rope{i}_theta"]))
    m = assert_stage_policy(y, g[f"rope{i}_y"])
    assert m.exact_fraction >= 0.99, str(m)


@pytest.mark.parametrize("i", range(5))
def test_cached_gqa_matches_reference(golden_stages, i):
    g = golden_stages
    ctx = oracle.gqa_attention(g[f"att{i}_q"], g[f"att{i}_k"], g[f"att{i}_v"], int(g[f"att{i}_p"]))
    m = assert_attention_policy(ctx, g[f"att{i}_ctx"])
    assert m.exact_fraction >= 0.98, str(m)


# ------------------------------------------------------------------ forward
FORWARD = ["fwd_decode_b2", "fwd_multi_token", "fwd_p0_chunk", "fwd_gqa3"]


def run_oracle_forward(g: dict, name: str):
    b, t, h, hkv, d, p, c, _ = (int(v) for v in g[f"{name}_shape"])
    kc = g[f"{name}_k_cache"].copy()
    vc = g[f"{name}_v_cache"].copy()
    st = oracle.decoder_attention_nvfp4(
        g[f"{name}_x"], g[f"{name}_g_in"], storage(g, f"{name}_wq_"), storage(g, f"{name}_wk_"),
        storage(g, f"{name}_wv_"), g[f"{name}_g_q"], g[f"{name}_g_k"], storage(g, f"{name}_wo_"),
        kc, vc, p)
    return st, kc, vc, (b, t, h, hkv, d, p, c)


@pytest.mark.parametrize("name", FORWARD)
def test_forward_stages_match_reference(golden_forward, name):
    g = golden_forward
    st, kc, vc, (b, t, h, hkv, d, p, c) = run_oracle_forward(g, name)
    st.q_norm_w, st.k_norm_w = g[f"{name}_g_q"], g[f"{name}_g_k"]
    qw = {k: storage(g, f"{name}_w{k}_") for k in "qkvo"}
    check_stages_isolated(g, name, st, qw, p, h // d, hkv, d)
    # The cache write is pure storage movement of the stage tensors.
    assert_bitwise(kc[:, :, p:p + t], st.k_rope.transpose(0, 2, 1, 3))
    assert_bitwise(vc[:, :, p:p + t], st.v_projected.reshape(b, t, hkv, d).transpose(0, 2, 1, 3))
    # Prefix and suffix slots untouched.
    assert_bitwise(kc[:, :, :p], g[f"{name}_k_cache"][:, :, :p])
    assert_bitwise(kc[:, :, p + t:], g[f"{name}_k_cache"][:, :, p + t:])


def test_quantized_weight_hashes_pin_the_canonical_fixture(golden_forward):
    g = golden_forward
    for key in "qkvo":
        s = storage(g, f"fwd_decode_b2_w{key}_")
        h = hashlib.sha256()
        for a in (s.packed_values, s.block_scales, np.float32(s.global_decode_scale)):
            h.update(np.ascontiguousarray(a).tobytes())
        assert h.hexdigest() == str(g[f"fwd_decode_b2_w{key}_sha256"])


def test_metrics_helper_counts_adjacent_steps():
    a = np.array([0x3F80, 0x3F81, 0x8000, 0x0000], dtype=np.uint16)
    e = np.array([0x3F80, 0x3F80, 0x0000, 0x0000], dtype=np.uint16)
    m = metrics(a, e)
    assert m.max_adjacency == 1 and m.exact_fraction == 0.75


def quantize_case_weights(inputs) -> dict:
    return {k: oracle.quantize(v.numpy()) for k, v in inputs.weights_fp32.items()}


def torch_bits(t) -> np.ndarray:
    import torch

    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def check_stages_isolated(g: dict, name: str, st, qw: dict, p: int, hq: int, hkv: int, d: int):
    """Feed each oracle stage the reference's own upstream BF16 tensor, so a
    one-ulp flip upstream cannot mask or excuse a difference downstream."""
    assert_stage_policy(st.input_normalized, g[f"{name}_input_normalized"])
    xn = g[f"{name}_input_normalized"]
    for key, stage in (("q", "q_projected"), ("k", "k_projected"), ("v", "v_projected")):
        assert_stage_policy(oracle.w4a16_linear(xn, qw[key]), g[f"{name}_{stage}"])
    b, t = xn.shape[:2]
    qh = g[f"{name}_q_projected"].reshape(b, t, hq, d)
    kh = g[f"{name}_k_projected"].reshape(b, t, hkv, d)
    assert_stage_policy(oracle.rms_norm(qh, st.q_norm_w, 1e-6), g[f"{name}_q_normalized"])
    assert_stage_policy(oracle.rms_norm(kh, st.k_norm_w, 1e-6), g[f"{name}_k_normalized"])
    assert_stage_policy(oracle.apply_rope(g[f"{name}_q_normalized"], p, 1e4), g[f"{name}_q_rope"])
    assert_stage_policy(oracle.apply_rope(g[f"{name}_k_normalized"], p, 1e4), g[f"{name}_k_rope"])
    ctx = g[f"{name}_context"]
    assert_stage_policy(oracle.w4a16_linear(ctx.reshape(b, t, hq * d), qw["o"]), g[f"{name}_output"])
    # End to end (every stage computed by the oracle itself).
    assert_e2e_policy(st.context, g[f"{name}_context"])
    assert_e2e_policy(st.output, g[f"{name}_output"])


def test_canonical_config_matches_reference_outputs(golden_canonical):
    """configs[0] (B=1, T=1, H=3072, P=511, C=1024) regenerated from its seed."""
    import synthetic

    g = golden_canonical
    inp = synthetic.make_decode_inputs(synthetic.CANONICAL, seed=0)
    qw = quantize_case_weights(inp)
    for key, s in qw.items():
        h = hashlib.sha256()
        for a in (s.packed_values, s.block_scales, np.float32(s.global_decode_scale)):
            h.update(np.ascontiguousarray(a).tobytes())
        assert h.hexdigest() == str(g[f"c0_w{key}_sha256"]), key
    kc, vc = torch_bits(inp.k_cache), torch_bits(inp.v_cache)
    st = oracle.decoder_attention_nvfp4(
        torch_bits(inp.x), torch_bits(inp.input_norm_weight), qw["q"], qw["k"], qw["v"],
        torch_bits(inp.q_norm_weight), torch_bits(inp.k_norm_weight), qw["o"], kc, vc, 511)
    st.q_norm_w, st.k_norm_w = torch_bits(inp.q_norm_weight), torch_bits(inp.k_norm_weight)
    check_stages_isolated(g, "c0", st, qw, 511, 24, 6, 128)
    # The appended slot is pure storage movement of K after norm+RoPE and raw V.
    assert_bitwise(kc[:, :, 511:512], st.k_rope.transpose(0, 2, 1, 3))
    assert_bitwise(vc[:, :, 511:512], st.v_projected.reshape(1, 1, 6, 128).transpose(0, 2, 1, 3))
    assert_e2e_policy(kc[:, :, 511:512], g["c0_new_k"])
    assert_e2e_policy(vc[:, :, 511:512], g["c0_new_v"])
