"""GPU parity of KV-length-sharded decode (configs[3] in miniature).

Single-process emulation: G cache shards on one GPU run the sharded stages
(front half with the owner-only append, per-shard log-sum-exp partials) and
the combine exactly as the ranks would, with the all-gather replaced by a
stack in rank order.  The output must match the unsharded chain forward and
the oracle (end-to-end policy); the concatenated cache shards must equal the
unsharded forward's cache bit for bit.  A real two-process NCCL run follows
when the box has two GPUs.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

import oracle
from bf16_metrics import assert_attention_policy, assert_e2e_policy
from gpu_util import dev_weight, host_bits

pytestmark = pytest.mark.gpu


def make_case(b, h, hkv, d, past, cap, seed):
    import synthetic

    shape = synthetic.DecodeShape(batch=b, tokens=1, hidden=h, kv_heads=hkv, head_dim=d, capacity=cap,
                                  past_lengths=(past,))
    inp = synthetic.make_decode_inputs(shape, seed)
    host_w = {k: oracle.quantize(w.numpy()) for k, w in inp.weights_fp32.items()}
    return inp, host_w


def unsharded(inp, ws, past):
    import nvfp4da_capi

    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    out = torch.empty_like(inp.x, device="cuda")
    fw = nvfp4da_capi.Forward(inp.x.cuda(), inp.input_norm_weight.cuda(), ws["q"], ws["k"], ws["v"],
                              inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda(), ws["o"], kc, vc, out,
                              past_length=past)
    fw.run(path=nvfp4da_capi.PATH_CHAIN)
    torch.cuda.synchronize()
    return out, kc, vc


@pytest.mark.parametrize("b,h,hkv,d,past,cap,shards", [
    (1, 3072, 6, 128, 511, 1024, 2),   # configs[0] split over two GPUs
    (1, 3072, 6, 128, 511, 1024, 4),
    (1, 3072, 6, 128, 100, 1024, 4),   # the last shards see no key at all
    (2, 1024, 2, 128, 4000, 4096, 3),  # long context, uneven shards, many splits per shard
    (8, 3072, 6, 128, 2047, 2048, 8),  # configs[3] shape (B=8, full cache) at 1/16 of the length
])
def test_sharded_stages_match_unsharded_forward(b, h, hkv, d, past, cap, shards):
    import kv_sharding

    inp, host_w = make_case(b, h, hkv, d, past, cap, seed=past + shards)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    ref_out, ref_kc, ref_vc = unsharded(inp, ws, past)

    st = kv_sharding.CudaStages()
    ranges = kv_sharding.shard_ranges(cap, shards)
    x, g_in = inp.x.cuda(), inp.input_norm_weight.cuda()
    g_q, g_k = inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda()
    kcs = [inp.k_cache[:, :, s.start:s.stop].contiguous().cuda() for s in ranges]
    vcs = [inp.v_cache[:, :, s.start:s.stop].contiguous().cuda() for s in ranges]
    qs, parts = [], []
    for s, kc, vc in zip(ranges, kcs, vcs):
        q = st.front(x, g_in, ws["q"], ws["k"], ws["v"], g_q, g_k, kc, vc, s, cap, past, 1e-6, 1e4)
        qs.append(q)
        parts.append(st.partials(q, kc, vc, s, past))
    ctx = st.combine(torch.stack(parts), qs[0].shape)
    out = st.o_proj(ctx, ws["o"])
    torch.cuda.synchronize()

    for q in qs[1:]:  # every rank computes the same q
        assert torch.equal(q.view(torch.int16), qs[0].view(torch.int16))
    np.testing.assert_array_equal(host_bits(torch.cat(kcs, dim=2)), host_bits(ref_kc))
    np.testing.assert_array_equal(host_bits(torch.cat(vcs, dim=2)), host_bits(ref_vc))
    # Context against the oracle's attention on the same q and caches.
    ctx_ref = oracle.gqa_attention(host_bits(qs[0]), host_bits(ref_kc), host_bits(ref_vc), past)
    assert_attention_policy(host_bits(ctx), ctx_ref)
    assert_e2e_policy(host_bits(out), host_bits(ref_out))
    g_qb, g_kb = host_bits(inp.q_norm_weight), host_bits(inp.k_norm_weight)
    ref = oracle.decoder_attention_nvfp4(host_bits(inp.x), host_bits(inp.input_norm_weight), host_w["q"],
                                         host_w["k"], host_w["v"], g_qb, g_kb, host_w["o"],
                                         host_bits(inp.k_cache).copy(), host_bits(inp.v_cache).copy(), past)
    assert_e2e_policy(host_bits(out), ref.output)


def test_shard_front_rejects_a_shard_outside_the_cache():
    import kv_sharding
    import nvfp4da_capi

    inp, host_w = make_case(1, 3072, 6, 128, 511, 1024, seed=1)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    st = kv_sharding.CudaStages()
    kc = inp.k_cache[:, :, :512].contiguous().cuda()
    vc = inp.v_cache[:, :, :512].contiguous().cuda()
    with pytest.raises(nvfp4da_capi.CapiError):
        st.front(inp.x.cuda(), inp.input_norm_weight.cuda(), ws["q"], ws["k"], ws["v"], inp.q_norm_weight.cuda(),
                 inp.k_norm_weight.cuda(), kc, vc, kv_sharding.KVShard(600, 512), 1024, 511, 1e-6, 1e4)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank: int, world: int, port: int, queue) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import kv_sharding

        inp, host_w = make_case(1, 3072, 6, 128, 511, 1024, seed=21)
        ws = {k: dev_weight(s) for k, s in host_w.items()}
        sh = kv_sharding.ShardedDecoderAttention(1024)
        kc = inp.k_cache[:, :, sh.shard.start:sh.shard.stop].contiguous().cuda()
        vc = inp.v_cache[:, :, sh.shard.start:sh.shard.stop].contiguous().cuda()
        out = sh.forward_(inp.x.cuda(), inp.input_norm_weight.cuda(), ws["q"], ws["k"], ws["v"],
                          inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda(), ws["o"], kc, vc, 511)
        torch.cuda.synchronize()
        queue.put((rank, host_bits(out)))
    except Exception as e:
        queue.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_match_unsharded_forward():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(isinstance(v, np.ndarray) for v in results.values()), results
    inp, host_w = make_case(1, 3072, 6, 128, 511, 1024, seed=21)
    ws = {k: dev_weight(s) for k, s in host_w.items()}
    ref_out, _, _ = unsharded(inp, ws, 511)
    np.testing.assert_array_equal(results[0], results[1])
    assert_e2e_policy(results[0], host_bits(ref_out))
