"""GPU parity of the prefill forward (configs[4] in miniature).

With B*T >= 128 the forward takes the modular chain: input RMSNorm, Q/K/V on
the tcgen05 GEMM, per-head RMSNorm, RoPE, cache append, causal GQA, O on the
GEMM.  Each stage is checked against the oracle applied to the GPU's own
upstream tensor (bit-exact norm / RoPE / append, one BF16 step for the
projections, the attention policy for the context) and the output against the
oracle run end to end.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from bf16_metrics import assert_attention_policy, assert_bitwise, assert_e2e_policy, assert_stage_policy
from gpu_util import dev_weight, host_bits
from test_gpu_forward import check_isolated, run_forward, small_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,t,h,hkv,d,p,c", [
    (1, 256, 3072, 6, 128, 0, 512),     # prefill from an empty cache
    (2, 128, 3072, 6, 128, 100, 256),   # prefill after a prompt prefix
    (1, 512, 3072, 6, 128, 0, 1024),    # configs[4] head configuration, a quarter of its T
])
def test_prefill_forward_matches_oracle(b, t, h, hkv, d, p, c):
    inp, host_w = small_case(b, t, h, hkv, d, p, c, seed=t + p)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    kc_before = host_bits(inp.k_cache)
    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    out, st = run_forward(inp.x.cuda(), inp.input_norm_weight.cuda(), ws, inp.q_norm_weight.cuda(),
                          inp.k_norm_weight.cuda(), kc, vc, p)
    out_bits = host_bits(out)
    g_q, g_k = host_bits(inp.q_norm_weight), host_bits(inp.k_norm_weight)
    check_isolated(st, out_bits, kc_before, host_bits(kc), host_bits(vc), host_w, g_q, g_k, p, t)
    ref = oracle.decoder_attention_nvfp4(host_bits(inp.x), host_bits(inp.input_norm_weight), host_w["q"],
                                         host_w["k"], host_w["v"], g_q, g_k, host_w["o"], host_bits(inp.k_cache),
                                         host_bits(inp.v_cache), p)
    assert_e2e_policy(out_bits, ref.output)


def test_prefill_with_per_sequence_lengths():
    """Batched prefill continuing two sequences from different lengths."""
    pasts = (17, 90)
    b, t = 2, 64
    inp, host_w = small_case(b, t, 1024, 2, 128, pasts, 256, seed=9)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    kc_before = host_bits(inp.k_cache)
    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    pl = torch.tensor(pasts, dtype=torch.int64).cuda()
    out, st = run_forward(inp.x.cuda(), inp.input_norm_weight.cuda(), ws, inp.q_norm_weight.cuda(),
                          inp.k_norm_weight.cuda(), kc, vc, 0, past_lengths=pl, max_past=max(pasts))
    g_q, g_k = host_bits(inp.q_norm_weight), host_bits(inp.k_norm_weight)
    check_isolated(st, host_bits(out), kc_before, host_bits(kc), host_bits(vc), host_w, g_q, g_k,
                   np.array(pasts), t)


# Sampled (b, t) rows of the full configs[4] prefill: the first rows, tile and
# 64-token boundaries, the last row.
C4_ROWS = [(0, 0), (0, 1), (1, 63), (1, 64), (2, 777), (3, 1024), (0, 1500), (3, 2047)]


def test_prefill_config4_full_size_sampled_rows():
    """configs[4] at full size (B=4, T=2048, P=0, C=4096): every stage of the
    forward, stage-isolated, on sampled (sequence, token) rows -- the oracle
    applied to the GPU's own upstream rows (bit-exact norm, RoPE and append;
    one BF16 step for the projections; the attention policy for each sampled
    row's context over its 1 .. 2048 causal keys) -- and the cache slots past
    T untouched."""
    b, t, h, hkv, d, c = 4, 2048, 3072, 6, 128, 4096
    inp, host_w = small_case(b, t, h, hkv, d, 0, c, seed=404)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    kc_before, vc_before = host_bits(inp.k_cache), host_bits(inp.v_cache)
    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    out, st = run_forward(inp.x.cuda(), inp.input_norm_weight.cuda(), ws, inp.q_norm_weight.cuda(),
                          inp.k_norm_weight.cuda(), kc, vc, 0)
    out_bits, kc_after, vc_after = host_bits(out), host_bits(kc), host_bits(vc)
    x, g_in = host_bits(inp.x), host_bits(inp.input_norm_weight)
    g_q, g_k = host_bits(inp.q_norm_weight), host_bits(inp.k_norm_weight)
    hq = h // d
    np.testing.assert_array_equal(kc_after[:, :, t:], kc_before[:, :, t:])
    np.testing.assert_array_equal(vc_after[:, :, t:], vc_before[:, :, t:])
    for bi, ti in C4_ROWS:
        r = (slice(bi, bi + 1), slice(ti, ti + 1))
        xn = st["input_normalized"][r]
        assert_bitwise(xn, oracle.rms_norm(x[r], g_in, 1e-6))
        for key, stage in (("q", "q_projected"), ("k", "k_projected"), ("v", "v_projected")):
            assert_stage_policy(st[stage][r], oracle.w4a16_linear(xn, host_w[key]))
        qn = st["q_normalized"][r]
        kn = st["k_normalized"][r]
        assert_bitwise(qn, oracle.rms_norm(st["q_projected"][r].reshape(1, 1, hq, d), g_q, 1e-6))
        assert_bitwise(kn, oracle.rms_norm(st["k_projected"][r].reshape(1, 1, hkv, d), g_k, 1e-6))
        # token ti of a prefill from P = 0 sits at position ti
        q_rope = st["q_rope"][r]
        assert_bitwise(q_rope, oracle.apply_rope(qn, ti, 1e4))
        assert_bitwise(kc_after[bi, :, ti], oracle.apply_rope(kn, ti, 1e4)[0, 0])
        assert_bitwise(vc_after[bi, :, ti], st["v_projected"][r].reshape(hkv, d))
        ctx = oracle.gqa_attention(q_rope, kc_after[bi:bi + 1, :, :ti + 1], vc_after[bi:bi + 1, :, :ti + 1], ti)
        assert_attention_policy(st["context"][r], ctx)
        assert_stage_policy(out_bits[r], oracle.w4a16_linear(st["context"][r].reshape(1, 1, hq * d), host_w["o"]))
