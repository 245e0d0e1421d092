"""Host logic of KV-length-sharded decode on CPU ranks (gloo, world size 2).

The CUDA stages are replaced by oracle-based stages on CPU tensors; the
partitioning, the owner-only append, the all-gather of the log-sum-exp
partials and the combine order are the product code of ``kv_sharding``.  The
sharded output must match the unsharded oracle forward (end-to-end policy)
and every rank's cache shard must equal its slice of the oracle's updated
cache bit for bit.
"""

from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from bf16_metrics import assert_e2e_policy

SHAPE = dict(b=2, h=256, hkv=2, d=64, past=40, cap=64)


def test_shard_ranges_cover_the_cache_contiguously():
    import kv_sharding

    for cap, world in ((64, 2), (65, 2), (32768, 8), (10, 3), (7, 7)):
        shards = kv_sharding.shard_ranges(cap, world)
        assert len(shards) == world
        assert shards[0].start == 0 and shards[-1].stop == cap
        for a, b in zip(shards, shards[1:]):
            assert a.stop == b.start
        assert max(s.capacity for s in shards) - min(s.capacity for s in shards) <= 1
        for pos in (0, cap // 2, cap - 1):
            r = kv_sharding.owner_of(pos, shards)
            assert shards[r].start <= pos < shards[r].stop
    with pytest.raises(ValueError):
        kv_sharding.shard_ranges(3, 4)
    with pytest.raises(ValueError):
        kv_sharding.owner_of(64, kv_sharding.shard_ranges(64, 2))


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16).copy()).view(torch.bfloat16)


class OracleStages:
    """The four stages on CPU tensors, computed with the oracle (test only)."""

    def __init__(self, host_w):
        self.w = host_w

    def front(self, x, g_in, wq, wk, wv, g_q, g_k, k_shard, v_shard, shard, global_capacity, past_length,
              rms_eps, rope_theta):
        b, t, h = x.shape
        hkv, d = k_shard.shape[1], k_shard.shape[3]
        xn = oracle.rms_norm(_bits(x), _bits(g_in), rms_eps)
        qp = oracle.w4a16_linear(xn, self.w["q"]).reshape(b, t, h // d, d)
        kp = oracle.w4a16_linear(xn, self.w["k"]).reshape(b, t, hkv, d)
        vp = oracle.w4a16_linear(xn, self.w["v"]).reshape(b, t, hkv, d)
        qr = oracle.apply_rope(oracle.rms_norm(qp, _bits(g_q), rms_eps), past_length, rope_theta)
        kr = oracle.apply_rope(oracle.rms_norm(kp, _bits(g_k), rms_eps), past_length, rope_theta)
        kc, vc = _bits(k_shard), _bits(v_shard)
        for i in range(t):
            slot = past_length + i - shard.start
            if 0 <= slot < shard.capacity:
                kc[:, :, slot] = kr[:, i]
                vc[:, :, slot] = vp[:, i]
        k_shard.copy_(_bf16(kc))
        v_shard.copy_(_bf16(vc))
        return _bf16(qr)

    def partials(self, q, k_shard, v_shard, shard, past_length):
        b, t, hq, d = q.shape
        hkv = k_shard.shape[1]
        group = hq // hkv
        qf = oracle.bf16_to_f32(_bits(q)).astype(np.float64)
        kf = oracle.bf16_to_f32(_bits(k_shard)).astype(np.float64)
        vf = oracle.bf16_to_f32(_bits(v_shard)).astype(np.float64)
        scale = np.float32(1.0 / math.sqrt(d))
        out = np.zeros((b * t * hq, d + 2), dtype=np.float32)
        for bi in range(b):
            for ti in range(t):
                n = min(past_length + ti + 1 - shard.start, shard.capacity)
                for h in range(hq):
                    row = (bi * t + ti) * hq + h
                    if n <= 0:
                        out[row, d] = -np.inf
                        continue
                    s = ((kf[bi, h // group, :n] @ qf[bi, ti, h]).astype(np.float32) * scale).astype(np.float32)
                    m = s.max()
                    e = np.exp((s - m).astype(np.float64)).astype(np.float32)
                    out[row, :d] = (e.astype(np.float64) @ vf[bi, h // group, :n]).astype(np.float32)
                    out[row, d], out[row, d + 1] = m, np.float32(e.astype(np.float64).sum())
        return torch.from_numpy(out)

    def combine(self, gathered, out_shape):
        g = gathered.numpy().astype(np.float64)
        d = g.shape[2] - 2
        m = g[:, :, d]
        mx = m.max(axis=0)
        f = np.where(np.isneginf(m), 0.0, np.exp(m - mx))
        l = (g[:, :, d + 1] * f).sum(axis=0)
        o = (g[:, :, :d] * f[:, :, None]).sum(axis=0) / l[:, None]
        return _bf16(oracle.f32_to_bf16(o.astype(np.float32)).reshape(out_shape))

    def o_proj(self, ctx, wo):
        b, t, hq, d = ctx.shape
        return _bf16(oracle.w4a16_linear(_bits(ctx).reshape(b, t, hq * d), self.w["o"]))


def _case():
    import synthetic

    shape = synthetic.DecodeShape(batch=SHAPE["b"], tokens=1, hidden=SHAPE["h"], kv_heads=SHAPE["hkv"],
                                  head_dim=SHAPE["d"], capacity=SHAPE["cap"], past_lengths=(SHAPE["past"],))
    inp = synthetic.make_decode_inputs(shape, 11)
    host_w = {k: oracle.quantize(w.numpy()) for k, w in inp.weights_fp32.items()}
    return inp, host_w


def _rank_main(rank: int, world: int, port: int, queue) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import kv_sharding

        inp, host_w = _case()
        sh = kv_sharding.ShardedDecoderAttention(SHAPE["cap"], stages=OracleStages(host_w))
        kc = inp.k_cache[:, :, sh.shard.start:sh.shard.stop].clone()
        vc = inp.v_cache[:, :, sh.shard.start:sh.shard.stop].clone()
        out = sh.forward_(inp.x, inp.input_norm_weight, None, None, None, inp.q_norm_weight, inp.k_norm_weight,
                          None, kc, vc, SHAPE["past"])
        queue.put((rank, _bits(out).copy(), _bits(kc).copy(), _bits(vc).copy(), sh.shard.start, sh.shard.stop))
    except Exception as e:  # report instead of leaving the parent waiting
        queue.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_match_the_unsharded_oracle():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=240) for _ in range(world)]
    errors = [r for r in results if len(r) == 2]
    assert not errors, errors
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    inp, host_w = _case()
    kc, vc = _bits(inp.k_cache).copy(), _bits(inp.v_cache).copy()
    ref = oracle.decoder_attention_nvfp4(_bits(inp.x), _bits(inp.input_norm_weight), host_w["q"], host_w["k"],
                                         host_w["v"], _bits(inp.q_norm_weight), _bits(inp.k_norm_weight),
                                         host_w["o"], kc, vc, SHAPE["past"])
    outs = {}
    for rank, out, kcs, vcs, start, stop in results:
        outs[rank] = out
        np.testing.assert_array_equal(kcs, kc[:, :, start:stop])
        np.testing.assert_array_equal(vcs, vc[:, :, start:stop])
        assert_e2e_policy(out, ref.output)
    np.testing.assert_array_equal(outs[0], outs[1])  # every rank combines in the same order

