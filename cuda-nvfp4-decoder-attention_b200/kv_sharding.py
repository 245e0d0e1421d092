"""KV-length-sharded decode step across the GPUs of one node.

One process per GPU.  Every rank holds a contiguous slice of positions of
every sequence's cache, ``[B, Hkv, shard.capacity, D]`` for global positions
``[shard.start, shard.start + shard.capacity)``.  A step:

1. every rank runs the fused front half (input RMSNorm, Q/K/V projection,
   per-head RMSNorm, RoPE at the global position); only the rank whose shard
   holds slot ``P_b + t`` appends the new K/V row;
2. every rank computes the log-sum-exp partials ``(o, m, l)`` of attention
   over its own slice (``[B*T*Hq, D + 2]`` float32);
3. an all-gather of the partials over the process group (NCCL over NVLink on
   a B200 node), then the combine (same order on every rank, so every rank
   gets the same context bits);
4. the O projection.

The reference has one GPU and one cache; the math is its cached GQA
(reference decoder_attention.py:273-381) with the softmax split over shards
and recombined, as a flash-decoding split is.  The stage implementation is
injectable so the host logic (partitioning, owner append, gather, combine
order) can be exercised on CPU ranks with the ``gloo`` backend.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class KVShard:
    start: int     # first global position held
    capacity: int  # positions held

    @property
    def stop(self) -> int:
        return self.start + self.capacity


def shard_ranges(global_capacity: int, world: int) -> list[KVShard]:
    """Contiguous, near-equal slices of ``[0, global_capacity)``; the first
    ``global_capacity % world`` ranks hold one position more."""
    if world <= 0 or global_capacity < world:
        raise ValueError(f"cannot split a capacity of {global_capacity} over {world} ranks")
    base, extra = divmod(global_capacity, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append(KVShard(start, n))
        start += n
    return out


def owner_of(position: int, shards: list[KVShard]) -> int:
    """Rank whose shard holds global cache position ``position``."""
    for r, s in enumerate(shards):
        if s.start <= position < s.stop:
            return r
    raise ValueError(f"position {position} is outside the cache")


class CudaStages:
    """The stages on this rank's GPU through the C ABI (libnvfp4da.so).

    A decode loop calls the stages with the same tensors every step, so the
    C argument structs and the intermediate buffers (q, workspace, partials,
    context) are built once per set of tensors and reused: a step costs one
    library call per stage and no allocation but its output."""

    def __init__(self):
        import nvfp4da_capi

        self.capi = nvfp4da_capi
        self.lib = nvfp4da_capi.load()
        self._front = {}
        self._part = {}
        self._ctx = {}
        self._wo = {}

    @staticmethod
    def _key(*tensors):
        return tuple((t.data_ptr(), tuple(t.shape)) for t in tensors)

    @staticmethod
    def _bounded(cache: dict) -> dict:
        """Entries keep their tensors alive: forget them all past 16 sets."""
        if len(cache) >= 16:
            cache.clear()
        return cache

    def front(self, x, g_in, wq, wk, wv, g_q, g_k, k_shard, v_shard, shard: KVShard, global_capacity: int,
              past_length: int, rms_eps: float, rope_theta: float) -> torch.Tensor:
        capi = self.capi
        key = self._key(x, g_in, g_q, g_k, k_shard, v_shard, wq.packed_values, wk.packed_values, wv.packed_values)
        hit = self._front.get(key)
        if hit is None:
            b, t, h = x.shape
            hkv, d = k_shard.shape[1], k_shard.shape[3]
            a = capi.ForwardArgs()
            a.x, a.input_norm_weight = x.data_ptr(), g_in.data_ptr()
            a.q_weight, a.k_weight, a.v_weight = capi.weight(wq), capi.weight(wk), capi.weight(wv)
            a.out_weight = capi.weight(wq)  # not used by the front half; any valid [H, H] weight
            a.q_norm_weight, a.k_norm_weight = g_q.data_ptr(), g_k.data_ptr()
            a.k_cache, a.v_cache = k_shard.data_ptr(), v_shard.data_ptr()
            q = torch.empty((b, t, h // d, d), dtype=torch.bfloat16, device=x.device)
            a.output = q.data_ptr()
            a.batch, a.tokens, a.hidden, a.kv_heads, a.head_dim, a.capacity = b, t, h, hkv, d, shard.capacity
            a.past_lengths = None
            # scratch of the batched front half (normalised rows, RoPE table), if the shape takes it
            wsb = self.lib.nvfp4da_qkv_rope_append_shard_workspace_size(C.byref(a))
            ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=x.device)
            # keep everything the struct points into alive with it
            hit = self._bounded(self._front)[key] = (a, q, (ws, wsb), (x, g_in, g_q, g_k, k_shard, v_shard, wq, wk, wv))
        a, q, (ws, wsb), _ = hit
        a.past_length, a.max_past_length = past_length, past_length
        a.rms_eps, a.rope_theta = rms_eps, rope_theta
        st = self.lib.nvfp4da_qkv_rope_append_shard(C.byref(a), shard.start, global_capacity, q.data_ptr(),
                                                    ws.data_ptr() if wsb else None, wsb,
                                                    torch.cuda.current_stream().cuda_stream)
        self.capi._check(st)
        return q

    def partials(self, q, k_shard, v_shard, shard: KVShard, past_length: int) -> torch.Tensor:
        b, t, hq, d = q.shape
        hkv = k_shard.shape[1]
        lib = self.lib
        key = self._key(q, k_shard, v_shard) + ((shard.start, shard.capacity, past_length),)
        hit = self._part.get(key)
        if hit is None:
            wsb = lib.nvfp4da_gqa_attention_partials_workspace_size(b, t, hq, hkv, d, shard.start, shard.capacity,
                                                                    past_length)
            ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=q.device)
            part = torch.empty((b * t * hq, d + 2), dtype=torch.float32, device=q.device)
            hit = self._bounded(self._part)[key] = (ws, part, (q, k_shard, v_shard))
        ws, part, _ = hit
        st = lib.nvfp4da_gqa_attention_partials(q.data_ptr(), k_shard.data_ptr(), v_shard.data_ptr(),
                                                part.data_ptr(), b, t, hq, hkv, shard.capacity, d, shard.start,
                                                past_length, None, past_length, ws.data_ptr(), ws.numel(),
                                                torch.cuda.current_stream().cuda_stream)
        self.capi._check(st)
        return part

    def combine(self, gathered: torch.Tensor, out_shape) -> torch.Tensor:
        shards, rows, d2 = gathered.shape
        key = self._key(gathered) + (tuple(out_shape),)
        ctx = self._ctx.get(key)
        if ctx is None:
            ctx = self._bounded(self._ctx)[key] = torch.empty(out_shape, dtype=torch.bfloat16, device=gathered.device)
        st = self.lib.nvfp4da_attention_combine(gathered.data_ptr(), shards, rows, d2 - 2, ctx.data_ptr(),
                                                torch.cuda.current_stream().cuda_stream)
        self.capi._check(st)
        return ctx

    def o_proj(self, ctx: torch.Tensor, wo) -> torch.Tensor:
        b, t, hq, d = ctx.shape
        key = (wo.packed_values.data_ptr(), wo.block_scales.data_ptr(), wo.global_decode_scale.data_ptr())
        wt = self._wo.get(key)
        if wt is None:
            wt = self._bounded(self._wo)[key] = (self.capi.weight(wo), wo)
        y = torch.empty((b, t, hq * d), dtype=torch.bfloat16, device=ctx.device)
        st = self.lib.nvfp4da_w4a16_linear(ctx.data_ptr(), b * t, C.byref(wt[0]), y.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
        self.capi._check(st)
        return y


class ShardedDecoderAttention:
    """Decoder-attention forward over a KV cache split by position across the
    ranks of ``group`` (all ranks call ``forward_`` with the same x, weights
    and past_length; each passes its own cache shard)."""

    def __init__(self, global_capacity: int, group=None, stages=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.global_capacity = int(global_capacity)
        self.shards = shard_ranges(self.global_capacity, self.world)
        self.shard = self.shards[self.rank]
        self.stages = stages if stages is not None else CudaStages()
        self._gather = None  # all-gather buffer, reused while the partials' shape stays

    def forward_(self, x, input_norm_weight, q_weight, k_weight, v_weight, q_norm_weight, k_norm_weight,
                 out_weight, k_shard, v_shard, past_length: int, *, rms_eps: float = 1e-6,
                 rope_theta: float = 10_000.0) -> torch.Tensor:
        b, t, h = x.shape
        if k_shard.shape[2] != self.shard.capacity or v_shard.shape != k_shard.shape:
            raise ValueError(f"rank {self.rank} must hold a cache shard of {self.shard.capacity} positions, "
                             f"got {tuple(k_shard.shape)}")
        if past_length < 0 or past_length + t > self.global_capacity:
            raise ValueError(f"past_length + current token count exceeds cache capacity "
                             f"({past_length + t} > {self.global_capacity})")
        st = self.stages
        q = st.front(x, input_norm_weight, q_weight, k_weight, v_weight, q_norm_weight, k_norm_weight, k_shard,
                     v_shard, self.shard, self.global_capacity, past_length, rms_eps, rope_theta)
        part = st.partials(q, k_shard, v_shard, self.shard, past_length)
        if self.world > 1:
            shape = (self.world * part.shape[0], part.shape[1])
            flat = self._gather
            if flat is None or tuple(flat.shape) != shape or flat.device != part.device:
                flat = self._gather = torch.empty(shape, dtype=part.dtype, device=part.device)
            dist.all_gather_into_tensor(flat, part.contiguous(), group=self.group)
            gathered = flat.view(self.world, *part.shape)
        else:
            gathered = part.unsqueeze(0)
        ctx = st.combine(gathered, q.shape)
        return st.o_proj(ctx, out_weight)
