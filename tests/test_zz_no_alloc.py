"""The allocation-free forward entry point.

For callers that cannot allocate device memory (a fixed, pre-reserved HBM
budget or a host whose allocator owns all device memory), the library offers
nvfp4da_decoder_attention_forward_noalloc: the same forward, with its scratch
taken from an 8 MiB array built into the library instead of a caller workspace.
These tests call it through the C ABI and check it against the workspace entry
point on two calls in a row: the canonical decode step (the one-kernel step,
which keeps nothing in the scratch), and two steps that take the kernel chain
and so keep their q, context, split partials and combine counters in the
array -- a batch of 9 long sequences (the streaming attention kernel) and a
two-token step (global split partials of the short-cache kernel).  The
counters must start each call at zero although the array keeps the last
call's contents.  This file is named so pytest collects it last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from bf16_metrics import assert_bitwise
from gpu_util import dev_weight, host_bits

pytestmark = pytest.mark.gpu


def make_case(b, t, h, hkv, d, p, c, seed):
    import oracle
    import synthetic

    shape = synthetic.DecodeShape(batch=b, tokens=t, hidden=h, kv_heads=hkv, head_dim=d, capacity=c,
                                  past_lengths=(p,))
    inp = synthetic.make_decode_inputs(shape, seed)
    ws = {k: dev_weight(oracle.quantize(w.numpy())) for k, w in inp.weights_fp32.items()}
    return inp, ws


def forward_pair(inp, ws, p):
    """Two Forward objects on identical copies of the inputs and caches."""
    import nvfp4da_capi

    out = []
    for _ in range(2):
        x = inp.x.cuda()
        kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
        y = torch.empty_like(x)
        fw = nvfp4da_capi.Forward(x, inp.input_norm_weight.cuda(), ws["q"], ws["k"], ws["v"],
                                  inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda(), ws["o"], kc, vc, y,
                                  past_length=p)
        out.append((fw, y, kc, vc))
    return out


@pytest.mark.parametrize("b,t,h,hkv,d,p,c,step", [
    (1, 1, 3072, 6, 128, 511, 1024, True),    # configs[0]: the one-kernel step
    (9, 1, 768, 2, 128, 3000, 3072, False),   # B > 8: chain, streaming attention, counters in the array
    (1, 2, 3072, 6, 128, 1500, 2048, False),  # T = 2: chain, 47 splits combined through the array
])
def test_noalloc_forward_matches_workspace_forward_twice(b, t, h, hkv, d, p, c, step):
    inp, ws = make_case(b, t, h, hkv, d, p, c, seed=101)
    (ref_fw, ref_y, ref_kc, ref_vc), (na_fw, na_y, na_kc, na_vc) = forward_pair(inp, ws, p)
    assert na_fw.step_supported == step
    for call in range(2):  # the second call reuses the array left by the first
        ref_fw.run()
        na_fw.run_noalloc()
        torch.cuda.synchronize()
        assert_bitwise(host_bits(na_y), host_bits(ref_y))
        assert_bitwise(host_bits(na_kc), host_bits(ref_kc))
        assert_bitwise(host_bits(na_vc), host_bits(ref_vc))


def test_noalloc_forward_rejects_more_scratch_than_it_holds():
    import nvfp4da_capi

    lib = nvfp4da_capi.load()
    # T = 1024 tokens of H = 3072 need 2 x 6 MiB of q / context scratch > 8 MiB.
    inp, ws = make_case(1, 1024, 3072, 6, 128, 0, 1024, seed=5)
    fw = nvfp4da_capi.Forward(inp.x.cuda(), inp.input_norm_weight.cuda(), ws["q"], ws["k"], ws["v"],
                              inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda(), ws["o"], inp.k_cache.cuda(),
                              inp.v_cache.cuda(), torch.empty_like(inp.x, device="cuda"), past_length=0)
    status = lib.nvfp4da_decoder_attention_forward_noalloc(ctypes.byref(fw.args),
                                                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == nvfp4da_capi.ERR_WORKSPACE
    assert b"8388608" in lib.nvfp4da_last_error()
