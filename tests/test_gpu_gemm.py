"""GPU parity of the tcgen05 tensor-core W4A16 GEMM (prefill-sized M).

y = BF16(x @ W_hat.T) against the oracle (reference/w4a16.py:11-59), within
one BF16 step or 2^-20 (the reference's own W4A16 tolerance,
tests/test_cuda_w4a16.py:146-152).  Covers tile tails in M and N, several K,
and the automatic routing of nvfp4da_w4a16_linear for M >= 64.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from bf16_metrics import assert_stage_policy
from gpu_util import dev_weight, host_bits

pytestmark = pytest.mark.gpu


def make(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((m, k), generator=g).to(torch.bfloat16)
    w = (torch.randn((n, k), generator=g) * 0.02).numpy().astype(np.float32)
    return x, oracle.quantize(w)


@pytest.mark.parametrize("m,n,k", [
    (128, 128, 256),     # one tile, four K steps
    (300, 200, 512),     # tails in M and N
    (64, 768, 3072),     # the smallest routed M, K/V projection shape
    (1024, 3072, 3072),  # Q / O projection, 8 x 24 tiles
    (130, 4608, 3072),   # fused-QKV width, M tail of 2 rows
])
def test_tensor_core_gemm_matches_oracle(m, n, k):
    import nvfp4da_capi

    x, sw = make(m, n, k, seed=m + n + k)
    w = dev_weight(sw)
    y = nvfp4da_capi.w4a16_gemm(x.cuda(), w)
    torch.cuda.synchronize()
    assert_stage_policy(host_bits(y), oracle.w4a16_linear(host_bits(x), sw))


def test_linear_routes_prefill_sized_m_to_the_tensor_core_gemm():
    import nvfp4da_capi

    x, sw = make(256, 768, 3072, seed=3)
    w = dev_weight(sw)
    xd = x.cuda()
    auto = nvfp4da_capi.w4a16_linear(xd, w)
    forced = nvfp4da_capi.w4a16_gemm(xd, w)
    torch.cuda.synchronize()
    assert torch.equal(auto.view(torch.int16), forced.view(torch.int16))


def test_gemm_rejects_k_it_does_not_cover():
    import nvfp4da_capi

    x, sw = make(128, 128, 128, seed=4)  # K = 128: scale rows of 8 bytes are not a TMA row
    with pytest.raises(nvfp4da_capi.CapiError) as e:
        nvfp4da_capi.w4a16_gemm(x.cuda(), dev_weight(sw))
    assert e.value.status == nvfp4da_capi.ERR_UNSUPPORTED
