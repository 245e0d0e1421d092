"""GPU parity of the whole forward (fused three-kernel path and the modular
path for head dimensions that are not multiples of 32), through the C ABI.

Two kinds of checks per case:
* stage-isolated: each GPU stage against the oracle applied to the GPU's own
  upstream BF16 tensor (bit-exact for norm / RoPE / cache append, one BF16
  step for projections, attention policy for the context);
* end to end: output and context against the reference's golden vectors and
  against the oracle run on the same inputs (scale-relative tolerance, see
  ``bf16_metrics``).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from bf16_metrics import assert_attention_policy, assert_bitwise, assert_e2e_policy, assert_stage_policy
from gpu_util import dev_bf16, dev_weight, golden_storage, host_bits, host_storage, storage_sha

pytestmark = pytest.mark.gpu

STAGES = ("input_normalized", "q_projected", "k_projected", "v_projected", "q_normalized", "k_normalized",
          "q_rope", "context")


def run_forward(x, g_in, ws, g_q, g_k, kc, vc, past, *, past_lengths=None, max_past=None, stages=True):
    """Run the C-ABI forward on device tensors; returns (output, stage dict)."""
    import nvfp4da_capi

    b, t, h = x.shape
    hkv, d = kc.shape[1], kc.shape[3]
    hq = h // d
    out = torch.empty_like(x)
    st = None
    if stages:
        st = {
            "input_normalized": torch.empty((b, t, h), dtype=torch.bfloat16, device="cuda"),
            "q_projected": torch.empty((b, t, hq * d), dtype=torch.bfloat16, device="cuda"),
            "k_projected": torch.empty((b, t, hkv * d), dtype=torch.bfloat16, device="cuda"),
            "v_projected": torch.empty((b, t, hkv * d), dtype=torch.bfloat16, device="cuda"),
            "q_normalized": torch.empty((b, t, hq, d), dtype=torch.bfloat16, device="cuda"),
            "k_normalized": torch.empty((b, t, hkv, d), dtype=torch.bfloat16, device="cuda"),
            "q_rope": torch.empty((b, t, hq, d), dtype=torch.bfloat16, device="cuda"),
            "context": torch.empty((b, t, hq, d), dtype=torch.bfloat16, device="cuda"),
        }
    fw = nvfp4da_capi.Forward(x, g_in, ws["q"], ws["k"], ws["v"], g_q, g_k, ws["o"], kc, vc, out,
                              past_length=past, past_lengths=past_lengths, max_past_length=max_past, stages=st)
    fw.run()
    torch.cuda.synchronize()
    return out, ({k: host_bits(v) for k, v in st.items()} if st else None)


def check_isolated(st: dict, out_bits, kc_before, kc_after, vc_after, host_w: dict, g_q, g_k, pasts, t: int):
    """Each GPU stage vs the oracle applied to the GPU's own upstream stage."""
    b = st["input_normalized"].shape[0]
    hkv, d = kc_after.shape[1], kc_after.shape[3]
    hq = st["q_normalized"].shape[2]
    xn = st["input_normalized"]
    for key, stage in (("q", "q_projected"), ("k", "k_projected"), ("v", "v_projected")):
        assert_stage_policy(st[stage], oracle.w4a16_linear(xn, host_w[key]))
    assert_bitwise(st["q_normalized"], oracle.rms_norm(st["q_projected"].reshape(b, t, hq, d), g_q, 1e-6))
    assert_bitwise(st["k_normalized"], oracle.rms_norm(st["k_projected"].reshape(b, t, hkv, d), g_k, 1e-6))
    assert_bitwise(st["q_rope"], oracle.apply_rope(st["q_normalized"], pasts, 1e4))
    k_rope = oracle.apply_rope(st["k_normalized"], pasts, 1e4)
    pl = np.broadcast_to(np.asarray(pasts, dtype=np.int64), (b,))
    for i in range(b):
        p = int(pl[i])
        assert_bitwise(kc_after[i, :, p:p + t], k_rope[i].transpose(1, 0, 2))
        assert_bitwise(vc_after[i, :, p:p + t], st["v_projected"][i].reshape(t, hkv, d).transpose(1, 0, 2))
        assert_bitwise(kc_after[i, :, :p], kc_before[i, :, :p])
        assert_bitwise(kc_after[i, :, p + t:], kc_before[i, :, p + t:])
    ctx = oracle.gqa_attention(st["q_rope"], kc_after, vc_after, pasts)
    assert_attention_policy(st["context"], ctx)
    assert_stage_policy(out_bits, oracle.w4a16_linear(st["context"].reshape(b, t, hq * d), host_w["o"]))


FORWARD = ["fwd_decode_b2", "fwd_multi_token", "fwd_p0_chunk", "fwd_gqa3"]


@pytest.mark.parametrize("name", FORWARD)
def test_fused_forward_matches_reference_golden(golden_forward, name):
    g = golden_forward
    b, t, h, hkv, d, p, c, _ = (int(v) for v in g[f"{name}_shape"])
    host_w = {k: golden_storage(g, f"{name}_w{k}_") for k in "qkvo"}
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    kc, vc = dev_bf16(g[f"{name}_k_cache"]), dev_bf16(g[f"{name}_v_cache"])
    out, st = run_forward(dev_bf16(g[f"{name}_x"]), dev_bf16(g[f"{name}_g_in"]), ws, dev_bf16(g[f"{name}_g_q"]),
                          dev_bf16(g[f"{name}_g_k"]), kc, vc, p)
    out_bits = host_bits(out)
    check_isolated(st, out_bits, g[f"{name}_k_cache"], host_bits(kc), host_bits(vc), host_w, g[f"{name}_g_q"],
                   g[f"{name}_g_k"], p, t)
    assert_stage_policy(st["input_normalized"], g[f"{name}_input_normalized"])
    assert_e2e_policy(st["context"], g[f"{name}_context"])
    assert_e2e_policy(out_bits, g[f"{name}_output"])


def canonical_inputs(quantize_on_gpu=True):
    import nvfp4da_capi
    import synthetic
    from nvfp4_tensor import NVFP4Tensor

    inp = synthetic.make_decode_inputs(synthetic.CANONICAL, seed=0)
    ws = {}
    for k, w in inp.weights_fp32.items():
        packed, scales, gamma = nvfp4da_capi.quantize(w.cuda())
        ws[k] = NVFP4Tensor(packed, scales, gamma, tuple(w.shape))
    return inp, ws


def test_canonical_decode_step_matches_reference_and_oracle(golden_canonical):
    """B=1, T=1, H=3072, Hq=24, Hkv=6, D=128, P=511, C=1024."""
    g = golden_canonical
    inp, ws = canonical_inputs()
    host_w = {k: host_storage(w) for k, w in ws.items()}
    for k, s in host_w.items():
        assert storage_sha(s) == str(g[f"c0_w{k}_sha256"])
    kc_before = host_bits(inp.k_cache)
    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    out, st = run_forward(inp.x.cuda(), inp.input_norm_weight.cuda(), ws, inp.q_norm_weight.cuda(),
                          inp.k_norm_weight.cuda(), kc, vc, 511)
    out_bits = host_bits(out)
    g_q, g_k = host_bits(inp.q_norm_weight), host_bits(inp.k_norm_weight)
    check_isolated(st, out_bits, kc_before, host_bits(kc), host_bits(vc), host_w, g_q, g_k, 511, 1)
    assert_stage_policy(st["input_normalized"], g["c0_input_normalized"])
    assert_e2e_policy(st["context"], g["c0_context"])
    assert_e2e_policy(out_bits, g["c0_output"])
    # Against the oracle run end to end on the same inputs.
    kco, vco = host_bits(inp.k_cache), host_bits(inp.v_cache)
    ref = oracle.decoder_attention_nvfp4(host_bits(inp.x), host_bits(inp.input_norm_weight), host_w["q"],
                                         host_w["k"], host_w["v"], g_q, g_k, host_w["o"], kco, vco, 511)
    assert_e2e_policy(out_bits, ref.output)


def test_repeated_steps_are_deterministic():
    inp, ws = canonical_inputs()
    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    x = inp.x.cuda()
    args = (x, inp.input_norm_weight.cuda(), ws, inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda(), kc, vc, 511)
    first, _ = run_forward(*args, stages=False)
    for _ in range(3):
        again, _ = run_forward(*args, stages=False)
        assert torch.equal(again.view(torch.int16), first.view(torch.int16))


def small_case(b, t, h, hkv, d, p, c, seed):
    import synthetic

    shape = synthetic.DecodeShape(batch=b, tokens=t, hidden=h, kv_heads=hkv, head_dim=d, capacity=c,
                                  past_lengths=(p,) if np.isscalar(p) else tuple(p))
    inp = synthetic.make_decode_inputs(shape, seed)
    host_w = {k: oracle.quantize(w.numpy()) for k, w in inp.weights_fp32.items()}
    return inp, host_w


@pytest.mark.parametrize("b,t,h,hkv,d,p,c", [
    (1, 2, 32, 2, 8, 2, 11),     # reference test shapes (modular path)
    (2, 3, 32, 2, 8, 3, 19),
    (1, 4, 32, 1, 8, 0, 17),
    (1, 1, 96, 1, 48, 5, 9),      # D not a multiple of 32
    (3, 1, 256, 2, 64, 40, 64),   # fused path, D = 64
    (1, 2, 512, 1, 256, 9, 16),   # fused path, D = 256
    (12, 1, 3072, 6, 128, 100, 128),  # batched front half and O projection, 12 rows (two n-tiles)
    (2, 12, 1024, 2, 128, 7, 32),     # batched, T = 12: 24 rows at 12 positions per sequence
    (40, 1, 512, 1, 128, 33, 40),     # batched, 40 rows (eight n-tiles, the last partly empty)
])
def test_forward_general_shapes_match_oracle(b, t, h, hkv, d, p, c):
    inp, host_w = small_case(b, t, h, hkv, d, p, c, seed=b * 100 + t * 10 + d)
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


def test_batched_decode_with_per_sequence_lengths():
    """configs[2] in miniature: each sequence its own past length (device array)."""
    pasts = (1024, 3000, 8191, 1500)
    b = len(pasts)
    inp, host_w = small_case(b, 1, 3072, 6, 128, pasts, 8192, seed=7)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    kc_before = host_bits(inp.k_cache)
    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    pl = torch.tensor(pasts, dtype=torch.int64).cuda()
    out, st = run_forward(inp.x.cuda(), inp.input_norm_weight.cuda(), ws, inp.q_norm_weight.cuda(),
                          inp.k_norm_weight.cuda(), kc, vc, 0, past_lengths=pl, max_past=max(pasts))
    g_q, g_k = host_bits(inp.q_norm_weight), host_bits(inp.k_norm_weight)
    check_isolated(st, host_bits(out), kc_before, host_bits(kc), host_bits(vc), host_w, g_q, g_k,
                   np.array(pasts), 1)


def test_non_default_stream_orders_every_stage():
    inp, ws = canonical_inputs()
    import nvfp4da_capi

    side = torch.cuda.Stream()
    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    g_in, g_q, g_k = inp.input_norm_weight.cuda(), inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda()
    x_host = inp.x.pin_memory()
    expected, _ = run_forward(inp.x.cuda(), g_in, ws, g_q, g_k, kc.clone(), vc.clone(), 511, stages=False)
    with torch.cuda.stream(side):
        x = torch.empty_like(inp.x, device="cuda")
        torch.cuda._sleep(2_000_000)  # ~1 ms of device time before the input lands
        x.copy_(x_host, non_blocking=True)
        out = torch.empty_like(x)
        fw = nvfp4da_capi.Forward(x, g_in, ws["q"], ws["k"], ws["v"], g_q, g_k, ws["o"], kc, vc, out,
                                  past_length=511)
        fw.run(side)
        result = out.to("cpu", non_blocking=True)
    side.synchronize()
    assert torch.equal(result.view(torch.int16), expected.cpu().view(torch.int16))


def test_config2_batched_decode_full_size_sampled():
    """configs[2] at full size: B=64, T=1, P_b ~ U[1024, 8191] (seeded), C=8192,
    device-side per-sequence lengths.  Stage-isolated parity on sampled
    sequences (the oracle applied to the GPU's own upstream rows; the context
    over each sampled sequence's P_b + 1 keys), and every sequence's cache
    prefix and suffix bit for bit unchanged."""
    import synthetic

    shape = synthetic.batched_shape()
    b, h, hkv, d = shape.batch, shape.hidden, shape.kv_heads, shape.head_dim
    hq = h // d
    pasts = np.array(shape.past_lengths, dtype=np.int64)
    inp = synthetic.make_decode_inputs(shape, seed=2, cache_device="cuda")
    host_w = {k: oracle.quantize(w.numpy()) for k, w in inp.weights_fp32.items()}
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    kc, vc = inp.k_cache, inp.v_cache
    kc_before, vc_before = kc.clone(), vc.clone()
    pl = torch.from_numpy(pasts).cuda()
    out, st = run_forward(inp.x.cuda(), inp.input_norm_weight.cuda(), ws, inp.q_norm_weight.cuda(),
                          inp.k_norm_weight.cuda(), kc, vc, 0, past_lengths=pl, max_past=int(pasts.max()))
    for i in range(b):  # only slot P_b of each sequence changes
        p = int(pasts[i])
        assert torch.equal(kc[i, :, :p].view(torch.int16), kc_before[i, :, :p].view(torch.int16))
        assert torch.equal(kc[i, :, p + 1:].view(torch.int16), kc_before[i, :, p + 1:].view(torch.int16))
        assert torch.equal(vc[i, :, :p].view(torch.int16), vc_before[i, :, :p].view(torch.int16))
        assert torch.equal(vc[i, :, p + 1:].view(torch.int16), vc_before[i, :, p + 1:].view(torch.int16))
    out_bits = host_bits(out)
    x, g_in = host_bits(inp.x), host_bits(inp.input_norm_weight)
    g_q, g_k = host_bits(inp.q_norm_weight), host_bits(inp.k_norm_weight)
    for i in sorted({0, int(np.argmin(pasts)), int(np.argmax(pasts)), 17, 40, b - 1}):
        p = int(pasts[i])
        r = slice(i, i + 1)
        xn = st["input_normalized"][r]
        assert_bitwise(xn, oracle.rms_norm(x[r], g_in, 1e-6))
        for key, stage in (("q", "q_projected"), ("k", "k_projected"), ("v", "v_projected")):
            assert_stage_policy(st[stage][r], oracle.w4a16_linear(xn, host_w[key]))
        qn, kn = st["q_normalized"][r], st["k_normalized"][r]
        assert_bitwise(qn, oracle.rms_norm(st["q_projected"][r].reshape(1, 1, hq, d), g_q, 1e-6))
        assert_bitwise(kn, oracle.rms_norm(st["k_projected"][r].reshape(1, 1, hkv, d), g_k, 1e-6))
        assert_bitwise(st["q_rope"][r], oracle.apply_rope(qn, p, 1e4))
        k_seq, v_seq = host_bits(kc[r, :, :p + 1]), host_bits(vc[r, :, :p + 1])
        assert_bitwise(k_seq[0, :, p], oracle.apply_rope(kn, p, 1e4)[0, 0])
        assert_bitwise(v_seq[0, :, p], st["v_projected"][r].reshape(hkv, d))
        assert_attention_policy(st["context"][r], oracle.gqa_attention(st["q_rope"][r], k_seq, v_seq, p))
        assert_stage_policy(out_bits[r], oracle.w4a16_linear(st["context"][r].reshape(1, 1, hq * d), host_w["o"]))


def test_hostio_forward_matches_device_forward():
    """nvfp4da_decoder_attention_forward_hostio (host input in, forward, host
    output out in one call) gives the bits of the device-buffer forward."""
    import nvfp4da_capi

    inp, ws = canonical_inputs()
    g_in, g_q, g_k = inp.input_norm_weight.cuda(), inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda()
    expected, _ = run_forward(inp.x.cuda(), g_in, ws, g_q, g_k, inp.k_cache.cuda(), inp.v_cache.cuda(), 511,
                              stages=False)
    x = torch.zeros_like(inp.x, device="cuda")
    out = torch.empty_like(x)
    fw = nvfp4da_capi.Forward(x, g_in, ws["q"], ws["k"], ws["v"], g_q, g_k, ws["o"], inp.k_cache.cuda(),
                              inp.v_cache.cuda(), out, past_length=511)
    x_host = inp.x.pin_memory()
    out_host = torch.empty_like(inp.x).pin_memory()
    for _ in range(2):
        out_host.zero_()
        fw.run_hostio(x_host, out_host)
        torch.cuda.synchronize()
        assert torch.equal(out_host.view(torch.int16), expected.cpu().view(torch.int16))
