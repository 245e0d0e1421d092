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
from bf16_metrics import assert_e2e_policy
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
