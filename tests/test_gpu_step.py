"""GPU parity of the one-kernel decode step (NVFP4DA_PATH_STEP) through the C ABI.

The step kernel computes the same forward as the three-kernel chain in one
cooperative launch.  Per case:
* the output against the oracle run end to end on the same inputs (scale-
  relative policy) and against the chain path on the same inputs;
* the cache: every slot but P_b unchanged bit for bit; the appended V row
  within one BF16 step of the oracle's V projection, the appended K row within
  the attention policy of the oracle's K after norm and RoPE;
* the appended K and V rows bit for bit equal to the chain's on the same
  inputs (the step recomputes the projections, the per-head norm and RoPE in
  its own code, so this pins them to the chain's bit-exact stages);
* no bounded wait gave up (the stream's sync status stays 0).
Plus repeated launches, graph replay, two streams at once, more streams than
the step has synchronisation slots, and the bounded-wait self-test.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from bf16_metrics import assert_attention_policy, assert_e2e_policy, assert_stage_policy
from gpu_util import dev_weight, host_bits

pytestmark = pytest.mark.gpu


def make_case(b, h, hkv, d, pasts, c, seed):
    import synthetic

    pasts = tuple(pasts) if not np.isscalar(pasts) else (pasts,)
    shape = synthetic.DecodeShape(batch=b, tokens=1, hidden=h, kv_heads=hkv, head_dim=d, capacity=c,
                                  past_lengths=pasts)
    inp = synthetic.make_decode_inputs(shape, seed)
    host_w = {k: oracle.quantize(w.numpy()) for k, w in inp.weights_fp32.items()}
    return inp, host_w


def forward(inp, ws, pasts, kc, vc, path):
    import nvfp4da_capi

    out = torch.empty_like(inp.x, device="cuda")
    pl = None
    past, maxp = int(np.max(pasts)), int(np.max(pasts))
    if not np.isscalar(pasts) and len(set(pasts)) > 1:
        pl = torch.tensor(pasts, dtype=torch.int64).cuda()
        past = 0
    fw = nvfp4da_capi.Forward(inp.x.cuda(), inp.input_norm_weight.cuda(), ws["q"], ws["k"], ws["v"],
                              inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda(), ws["o"], kc, vc, out,
                              past_length=past, past_lengths=pl, max_past_length=maxp)
    return fw, out


STEP_CASES = [
    # b, h, hkv, d, past(s), c
    (1, 3072, 6, 128, 511, 1024),          # configs[0]
    (1, 3072, 6, 128, 0, 1024),            # empty cache: one split, RoPE at position 0
    (1, 3072, 6, 128, 40, 64),             # one split, no partials
    (1, 3072, 6, 128, 4000, 4096),         # the longest tile that fits in shared memory
    (3, 256, 2, 64, 40, 64),               # D = 64, 2 query heads per KV head
    (1, 512, 1, 256, 9, 16),               # D = 256
    (8, 1024, 8, 128, 100, 128),           # 8 sequences, 1 query head per KV head
    (2, 2048, 2, 128, 700, 1024),          # 8 query heads per KV head
    (4, 3072, 6, 128, (5, 300, 511, 64), 512),  # per-sequence lengths (device array)
    (2, 3072, 6, 128, (1023, 17), 1024),
]


@pytest.mark.parametrize("b,h,hkv,d,pasts,c", STEP_CASES)
def test_step_matches_oracle_and_chain(b, h, hkv, d, pasts, c):
    import nvfp4da_capi

    inp, host_w = make_case(b, h, hkv, d, pasts, c, seed=b * 1000 + h + d)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    pl = np.broadcast_to(np.asarray(pasts, dtype=np.int64), (b,))
    kc_before = host_bits(inp.k_cache)
    vc_before = host_bits(inp.v_cache)

    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    fw, out = forward(inp, ws, pasts, kc, vc, nvfp4da_capi.PATH_STEP)
    assert fw.step_supported
    fw.run(path=nvfp4da_capi.PATH_STEP)
    assert nvfp4da_capi.sync_status() == 0
    import decoder_attention_cuda

    decoder_attention_cuda.check_wait_status()  # the drop-in module's check: no wait gave up
    out_bits, kc_bits, vc_bits = host_bits(out), host_bits(kc), host_bits(vc)

    kc2, vc2 = inp.k_cache.cuda(), inp.v_cache.cuda()
    fw2, out2 = forward(inp, ws, pasts, kc2, vc2, nvfp4da_capi.PATH_CHAIN)
    fw2.run(path=nvfp4da_capi.PATH_CHAIN)
    torch.cuda.synchronize()
    chain_bits = host_bits(out2)
    # The appended rows (and so the whole caches) equal the chain's bit for bit.
    np.testing.assert_array_equal(kc_bits, host_bits(kc2))
    np.testing.assert_array_equal(vc_bits, host_bits(vc2))

    g_q, g_k = host_bits(inp.q_norm_weight), host_bits(inp.k_norm_weight)
    ref = oracle.decoder_attention_nvfp4(host_bits(inp.x), host_bits(inp.input_norm_weight), host_w["q"],
                                         host_w["k"], host_w["v"], g_q, g_k, host_w["o"], kc_before.copy(),
                                         vc_before.copy(), pl if b > 1 else int(pl[0]))
    assert_e2e_policy(out_bits, ref.output)
    assert_e2e_policy(out_bits, chain_bits)

    # Cache: only slot P_b of each sequence changes.
    for i in range(b):
        p = int(pl[i])
        for after, before in ((kc_bits, kc_before), (vc_bits, vc_before)):
            np.testing.assert_array_equal(after[i, :, :p], before[i, :, :p])
            np.testing.assert_array_equal(after[i, :, p + 1:], before[i, :, p + 1:])
        v_new = ref.v_projected[i].reshape(1, hkv, d).transpose(1, 0, 2)
        assert_stage_policy(vc_bits[i, :, p:p + 1], v_new)
        assert_attention_policy(kc_bits[i, :, p:p + 1], ref.k_rope[i].transpose(1, 0, 2))


def test_step_is_deterministic_and_reusable_across_launches_and_graphs():
    """Many launches on one stream reuse one synchronisation slot; a graph
    replay reuses it too.  Every launch must give the same bits."""
    import nvfp4da_capi

    inp, host_w = make_case(1, 3072, 6, 128, 511, 1024, seed=3)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    fw, out = forward(inp, ws, 511, kc, vc, nvfp4da_capi.PATH_STEP)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        fw.run(s)
        first = out.clone()
        for _ in range(50):
            fw.run(s)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), first.view(torch.int16))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(4):
                fw.run(s)
        out.zero_()
        for _ in range(10):
            g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), first.view(torch.int16))
    assert nvfp4da_capi.sync_status(s) == 0


def test_step_on_two_streams_at_once():
    """Launches on different streams take different slots and may overlap."""
    import nvfp4da_capi

    inp, host_w = make_case(1, 3072, 6, 128, 511, 1024, seed=4)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    runs = []
    for _ in range(2):
        kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
        runs.append(forward(inp, ws, 511, kc, vc, nvfp4da_capi.PATH_STEP))
    ref_fw, ref_out = runs[0]
    ref_fw.run()
    torch.cuda.synchronize()
    expected = ref_out.clone()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for _ in range(20):
        for (fw, _), st in zip(runs, streams):
            fw.run(st)
    torch.cuda.synchronize()
    for (_, out), st in zip(runs, streams):
        assert torch.equal(out.view(torch.int16), expected.view(torch.int16))
        assert nvfp4da_capi.sync_status(st) == 0


def test_more_streams_than_synchronisation_slots():
    """The step keeps per-stream hand-off slots (64 per device, never
    released).  Past them, AUTO takes the chain instead of failing: 70 fresh
    streams all give the step's or the chain's bits.  Runs in a child process:
    the slots it uses up stay used for the life of the process."""
    import subprocess
    import sys
    from pathlib import Path

    here = Path(__file__).resolve().parent
    code = (f"import sys; sys.path[:0] = [{str(here)!r}, {str(here.parent)!r}, "
            f"{str(here.parent / 'cuda-nvfp4-decoder-attention_b200')!r}]\n"
            "import test_gpu_step as t; t._many_streams_child()\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "many-streams ok" in r.stdout


def _many_streams_child():
    import nvfp4da_capi

    inp, host_w = make_case(1, 3072, 6, 128, 511, 1024, seed=8)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    expect = {}
    for path in (nvfp4da_capi.PATH_STEP, nvfp4da_capi.PATH_CHAIN):
        fw, out = forward(inp, ws, 511, inp.k_cache.cuda(), inp.v_cache.cuda(), path)
        fw.run(path=path)
        torch.cuda.synchronize()
        expect[path] = out.view(torch.int16).clone()
    fw, out = forward(inp, ws, 511, inp.k_cache.cuda(), inp.v_cache.cuda(), nvfp4da_capi.PATH_AUTO)
    # Fresh CUDA streams (torch.cuda.Stream() cycles through a fixed pool).
    from cuda.bindings import runtime as cudart

    streams = []
    for _ in range(70):
        err, handle = cudart.cudaStreamCreate()
        assert int(err) == 0
        streams.append(torch.cuda.ExternalStream(int(handle)))
    took = {nvfp4da_capi.PATH_STEP: 0, nvfp4da_capi.PATH_CHAIN: 0}
    for st in streams:
        out.zero_()
        torch.cuda.synchronize()
        fw.run(st)
        st.synchronize()
        got = out.view(torch.int16)
        match = [p for p, e in expect.items() if torch.equal(got, e)]
        assert match, "output of neither path"
        took[match[0]] += 1
    if not torch.equal(expect[nvfp4da_capi.PATH_STEP], expect[nvfp4da_capi.PATH_CHAIN]):
        assert took[nvfp4da_capi.PATH_CHAIN] >= 70 - 64
    with pytest.raises(nvfp4da_capi.CapiError) as e:  # an explicit step request still reports the limit
        fw.run(streams[-1], path=nvfp4da_capi.PATH_STEP)
    assert e.value.status == nvfp4da_capi.ERR_UNSUPPORTED
    torch.cuda.synchronize()
    for st in streams:
        cudart.cudaStreamDestroy(st.cuda_stream)
    print("many-streams ok", flush=True)


def test_auto_path_matches_one_of_the_explicit_paths():
    """AUTO must be one of the two explicit paths bit for bit (it only picks)."""
    import nvfp4da_capi

    inp, host_w = make_case(1, 3072, 6, 128, 511, 1024, seed=5)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    outs = {}
    for path in (nvfp4da_capi.PATH_AUTO, nvfp4da_capi.PATH_CHAIN, nvfp4da_capi.PATH_STEP):
        fw, out = forward(inp, ws, 511, inp.k_cache.cuda(), inp.v_cache.cuda(), path)
        fw.run(path=path)
        torch.cuda.synchronize()
        outs[path] = out.view(torch.int16).clone()
    assert torch.equal(outs[nvfp4da_capi.PATH_AUTO], outs[nvfp4da_capi.PATH_CHAIN]) or \
        torch.equal(outs[nvfp4da_capi.PATH_AUTO], outs[nvfp4da_capi.PATH_STEP])


@pytest.mark.parametrize("b,h,hkv,d,pasts,c", [
    (1, 96, 1, 48, 5, 9),                          # D = 48
    (4, 3072, 6, 128, (5, 300, 1023, 64), 1024),   # K/V tiles too large for shared memory
])
def test_step_path_rejects_what_it_does_not_cover(b, h, hkv, d, pasts, c):
    """Configurations the one-kernel step does not cover: PATH_STEP refuses
    them, PATH_AUTO falls back to the chain."""
    import nvfp4da_capi

    inp, host_w = make_case(b, h, hkv, d, pasts, c, seed=6)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    fw, out = forward(inp, ws, pasts, inp.k_cache.cuda(), inp.v_cache.cuda(), nvfp4da_capi.PATH_STEP)
    assert not fw.step_supported
    with pytest.raises(nvfp4da_capi.CapiError) as e:
        fw.run(path=nvfp4da_capi.PATH_STEP)
    assert e.value.status == nvfp4da_capi.ERR_UNSUPPORTED
    fw.run()
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()


def test_bounded_wait_gives_up_and_reports():
    """The wait primitive of the step kernel, on a counter nothing sets: it
    must return after its time limit with the timeout flag set, and the
    context must stay usable."""
    import nvfp4da_capi

    assert nvfp4da_capi.wait_timeout_probe(2_000_000) == 1  # 2 ms limit
    x = torch.ones(4, device="cuda")
    assert float((x + 1).sum()) == 8.0


@pytest.mark.parametrize("b,h,x_kind,out_kind", [
    (1, 3072, "pinned", "pinned"),      # rows in the parameter block
    (1, 3072, "pageable", "pinned"),    # parameter block: any host memory
    (2, 3072, "pinned", "pinned"),      # 12 KB: read by the kernel from mapped memory
    (2, 3072, "pageable", "pageable"),  # copied in, copied out
    (1, 1024, "pinned", "pageable"),    # parameter block in, output copied out
])
def test_hostio_input_routes_match_the_device_forward(b, h, x_kind, out_kind):
    """nvfp4da_decoder_attention_forward_hostio on the one-kernel step: the
    activation rows reach the kernel through its parameter block, through
    mapped page-locked memory, or by a copy, and the output is written to
    mapped memory or copied; every route gives the device forward's bits."""
    import nvfp4da_capi

    pasts = tuple(range(300, 300 + b))
    inp, host_w = make_case(b, h, max(1, h // 512), 128, pasts if b > 1 else pasts[0], 512, seed=77 + b + h)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    fw, out = forward(inp, ws, pasts if b > 1 else pasts[0], inp.k_cache.cuda(), inp.v_cache.cuda(),
                      nvfp4da_capi.PATH_AUTO)
    assert fw.step_supported
    fw.run()
    expected = host_bits(out)
    x_host = inp.x.clone()
    out_host = torch.empty_like(inp.x)
    if x_kind == "pinned":
        x_host = x_host.pin_memory()
    if out_kind == "pinned":
        out_host = out_host.pin_memory()
    fw._keep[0].zero_()  # the device rows: only the copy route writes them again
    for _ in range(2):
        out_host.zero_()
        fw.run_hostio(x_host, out_host)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host_bits(out_host), expected)
    assert nvfp4da_capi.sync_status() == 0
