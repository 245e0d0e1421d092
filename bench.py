"""Benchmark: canonical NVFP4-W4A16 decoder-attention decode step on B200.

Metric: decode tokens/s and us/step at B=1 (configs[0]:
T=1, H=3072, Hq=24, Hkv=6, D=128, P=511, C=1024), HBM GB/s as % of peak.

A "step" is one forward of one decode token through the library's default
path: the one-kernel cooperative decode step (norms, W4A16 Q/K/V, RoPE,
append, split-KV attention and O projection in one launch); the three-kernel
PDL chain is timed beside it (paths_us_per_step).  Inputs are resident in HBM; steps
rotate over R replicas of weights + caches + activations whose total exceeds
2x the 126 MB L2, so every step streams its 14.9 MB from HBM.  The timed loop
replays a CUDA graph of R steps.

Multi-GPU (torchrun, one process per GPU): every rank decodes its own
independent sequence (weak scaling, no collective on the data path); value is
the tokens of all ranks over the max-over-ranks device time.

The line also carries `workloads`, the other configs measured in the same run
at the same N: configs[2] batch-sharded (B=64 split into 64/N sequences per
rank, device-side past lengths, no collective), configs[3] KV-length-sharded
(32768/N cache positions per rank, NCCL all-gather of the log-sum-exp
partials) and configs[4] prefill (replicated per rank), each with per-GPU HBM
GB/s or TFLOP/s against the measured peaks.

--impl reference times the reference's CPU path (the numpy restatement of
reference/decoder_attention_nvfp4.py in oracle/; the Python reference itself
cannot travel to the GPU box) on the host cores, on the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "cuda-nvfp4-decoder-attention_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "decode tokens/s (B=1 canonical decode step)"
UNIT = "tokens/s"
WORKLOAD = ("configs[0] canonical decode: B=1 T=1 H=3072 Hq=24 Hkv=6 D=128 P=511 C=1024, "
            "NVFP4 W4A16 Q/K/V/O, BF16 caches")
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


# ---------------------------------------------------------------- algorithmic bytes
def step_bytes(shape) -> dict:
    """Algorithmic (each byte once) HBM traffic of one decode step."""
    h, d, hkv, hq = shape.hidden, shape.head_dim, shape.kv_heads, shape.q_heads
    m = shape.batch * shape.tokens
    kvw = hkv * d
    w = lambda n, k: n * (k // 2 + k // 16) + 4  # noqa: E731
    w_qkv = w(h, h) + 2 * w(kvw, h)
    w_o = w(h, h)
    s = shape.past(0) + shape.tokens
    kv_read = shape.batch * s * 2 * kvw * 2
    append = m * 2 * kvw * 2
    act = m * h * 2
    norms = h * 2 + 2 * d * 2
    qkv = w_qkv + act + norms + m * hq * d * 2 + append  # x, gains, q out, K/V append
    attn = kv_read + 2 * m * hq * d * 2  # caches, q in, context out
    o = w_o + 2 * act  # weights, context in, output out
    total = w_qkv + w_o + kv_read + append + 2 * act + norms
    return {"qkv": qkv, "attention": attn, "o_proj": o, "step": total}


KERNEL_HEADERS = {"decode_step": "decode_step.cuh", "qkv_fused": "qkv_fused.cuh", "attn_stream": "attention_stream.cuh",
                  "qkv_batched": "gemv_batched.cuh", "o_batched": "gemv_batched.cuh"}


def kernel_source_digest(header: str) -> str:
    """First 16 hex digits of the SHA-256 over a kernel's header and every
    header it includes from csrc/ (transitively, in name order): a profile
    captured from other sources no longer describes the kernel that runs."""
    import hashlib
    import re

    csrc = PKG / "csrc"
    seen, todo = set(), [header]
    while todo:
        f = todo.pop()
        if f in seen or not (csrc / f).is_file():
            continue
        seen.add(f)
        todo += re.findall(r'#include "([^"/]+)"', (csrc / f).read_text())
    h = hashlib.sha256()
    for f in sorted(seen):
        h.update(f.encode())
        h.update((csrc / f).read_bytes())
    return h.hexdigest()[:16]


def ncu_traffic(kernel: str, summary: str | None = None) -> float | None:
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu
    summary (profiles/<kernel>_canonical.md, or profiles/<summary>, line
    `dram_bytes_per_launch: N`), or None when the summary's
    `kernel_sources: <digest>` line does not match kernel_source_digest of the
    kernel's header in this tree (the capture predates a kernel change)."""
    import re

    p = ROOT / "profiles" / (summary or f"{kernel}_canonical.md")
    try:
        text = p.read_text()
    except OSError:
        return None
    # The capture that describes this tree: the `dram_bytes_per_launch` line
    # last seen before a `kernel_sources` line whose digest matches.
    want = kernel_source_digest(KERNEL_HEADERS[kernel])
    last = None
    for line in text.splitlines():
        m = re.match(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", line)
        if m:
            last = float(m.group(1))
        m = re.match(r"kernel_sources:\s*([0-9a-f]+)", line)
        if m and m.group(1) == want:
            return last
    return None


def measured_peak_gbs() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        # NCCL's version banner goes to stdout, where rank 0's JSON line is.
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- GPU arm
class Replica:
    def __init__(self, inp, ws, capi):
        dev = "cuda"
        self.x = inp.x.to(dev)
        self.g_in = inp.input_norm_weight.to(dev)
        self.g_q = inp.q_norm_weight.to(dev)
        self.g_k = inp.k_norm_weight.to(dev)
        self.kc = inp.k_cache.to(dev)
        self.vc = inp.v_cache.to(dev)
        self.ws = {k: w.to(dev) for k, w in ws.items()}
        self.out = torch.empty_like(self.x)
        self.q_rope = torch.empty((1, 1, 24, 128), dtype=torch.bfloat16, device=dev)
        self.ctx = torch.empty_like(self.q_rope)
        self.fw = capi.Forward(self.x, self.g_in, self.ws["q"], self.ws["k"], self.ws["v"], self.g_q, self.g_k,
                               self.ws["o"], self.kc, self.vc, self.out, past_length=511)
        lib = capi.load()
        self.attn_ws_bytes = lib.nvfp4da_gqa_attention_workspace_size(1, 1, 24, 6, 128, 511)
        self.attn_ws = torch.empty(max(1, self.attn_ws_bytes), dtype=torch.uint8, device=dev)


def timed_graph(fn_list, reps: int, stream) -> float:
    """Capture fn_list (one call each) into a graph, replay `reps` times; ms total."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for fn in fn_list:
            fn()
    g.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(reps):
            g.replay()
        end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def run_gpu(args) -> None:
    world, rank, local = dist_setup()
    import cuda_primitives  # noqa: F401  (loads the operator library; fails loudly if unbuilt)
    import decoder_attention_cuda
    import nvfp4da_capi as capi
    import synthetic
    from nvfp4_tensor import NVFP4Tensor

    capi.load()
    shape = synthetic.CANONICAL
    inp = synthetic.make_decode_inputs(shape, seed=0)
    ws = {}
    for k, w in inp.weights_fp32.items():
        packed, scales, gamma = capi.quantize(w.cuda())
        ws[k] = NVFP4Tensor(packed, scales, gamma, tuple(w.shape))
    nbytes = step_bytes(shape)
    replica_bytes = nbytes["step"] + 2 * inp.k_cache.numel() * 2
    n_rep = max(2, math.ceil(2 * L2_BYTES / replica_bytes))
    reps = [Replica(inp, ws, capi) for _ in range(n_rep)]
    stream = torch.cuda.Stream()

    # warm-up (untimed)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            reps[i % n_rep].fw.run(stream)
    torch.cuda.synchronize()

    # ---- timed region: exactly K steps, graph replays of n_rep steps (+ a tail graph)
    k = args.steps
    full, tail = divmod(k, n_rep)
    step_fns = [(lambda r=r: r.fw.run(stream)) for r in reps]
    g_full = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_full, stream=stream):
        for fn in step_fns:
            fn()
    g_tail = None
    if tail:
        g_tail = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_tail, stream=stream):
            for fn in step_fns[:tail]:
                fn()
    g_full.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)  # let the sampler start before the timed region
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(full):
            g_full.replay()
        if g_tail is not None:
            g_tail.replay()
        end.record(stream)
    end.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms = max_over_ranks(start.elapsed_time(end), world)
    tokens = world * shape.batch * shape.tokens * k
    value = tokens / (ms / 1e3)
    ms_per_step = ms / k

    # ---- per-kernel device time in isolation (same rotation, graphs of n_rep launches)
    lib = capi.load()

    def attn_call(r):
        st = lib.nvfp4da_gqa_attention_cached(r.q_rope.data_ptr(), r.kc.data_ptr(), r.vc.data_ptr(),
                                              r.ctx.data_ptr(), 1, 1, 24, 6, 1024, 128, 511, None, 511,
                                              r.attn_ws.data_ptr(), r.attn_ws_bytes,
                                              torch.cuda.current_stream().cuda_stream)
        assert st == 0, lib.nvfp4da_last_error()

    reps_k = max(20, min(2000, k // n_rep))
    kern_ms = {
        "qkv": timed_graph([(lambda r=r: r.fw.run_qkv(r.q_rope, stream)) for r in reps], reps_k, stream),
        "attention": timed_graph([(lambda r=r: attn_call(r)) for r in reps], reps_k, stream),
        "o_proj": timed_graph([(lambda r=r: capi.w4a16_linear(r.ctx.view(1, 3072), r.ws["o"],
                                                              r.out.view(1, 3072), stream)) for r in reps],
                              reps_k, stream),
    }
    # both forward paths, whole steps (the same graph form as the timed region)
    path_ms = {name: timed_graph([(lambda r=r, pth=pth: r.fw.run(stream, pth)) for r in reps], reps_k, stream)
               for name, pth in (("chain", capi.PATH_CHAIN), ("step", capi.PATH_STEP))
               if pth != capi.PATH_STEP or reps[0].fw.step_supported}
    per_launch_us = {n: v * 1e3 / (reps_k * n_rep) for n, v in kern_ms.items()}
    peak, peak_src = measured_peak_gbs()
    kernels = {n: {"us": round(per_launch_us[n], 3), "bytes": nbytes[n],
                   "gbs": round(nbytes[n] / (per_launch_us[n] * 1e-6) / 1e9, 1)} for n in kern_ms}
    qkv_gbs = nbytes["qkv"] / (per_launch_us["qkv"] * 1e-6) / 1e9
    step_gbs = nbytes["step"] / (ms_per_step * 1e-3) / 1e9

    # Dominant kernel: the one-kernel step (the default path, one launch per
    # step) when it covers the shape, else the chain's fused QKV kernel.
    if "step" in path_ms:
        step_us = path_ms["step"] * 1e3 / (reps_k * n_rep)
        gbs = nbytes["step"] / (step_us * 1e-6) / 1e9
        roofline = {"bound": "hbm", "kernel": "decode_step_kernel (the whole step, one cooperative launch)",
                    "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                    "peak_source": peak_src, "traffic": ncu_traffic("decode_step"),
                    "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch "
                                      "(profiles/decode_step_canonical.md)",
                    "bytes_per_launch": nbytes["step"]}
    else:
        roofline = {"bound": "hbm", "kernel": "qkv_fused (input norm + W4A16 QKV + head norm + RoPE + append)",
                    "achieved": round(qkv_gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(qkv_gbs / peak, 4),
                    "peak_source": peak_src, "traffic": ncu_traffic("qkv_fused"),
                    "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch "
                                      "(profiles/qkv_fused_canonical.md)",
                    "bytes_per_launch": nbytes["qkv"]}
    roofline.update({"step_achieved": round(step_gbs, 1), "step_frac": round(step_gbs / peak, 4),
                     "step_bytes": nbytes["step"]})

    # ---- end to end through the drop-in Python API with host buffers
    step_supported = reps[0].fw.step_supported
    e2e = run_e2e_hostio(args, reps, stream, world)
    e2e["torch_op"] = run_e2e(args, reps, decoder_attention_cuda, stream, world)

    # ---- the other configs: batch-sharded configs[2], KV-sharded configs[3], prefill configs[4]
    workloads = {}
    if not args.skip_workloads:
        del reps
        torch.cuda.empty_cache()
        for name, fn in (("c2_batch_sharded", lambda: run_c2_batch_sharded(capi, world, rank, stream, peak)),
                         ("c3_kv_sharded", lambda: run_c3_kv_sharded(capi, world, rank, stream, peak)),
                         ("c4_prefill", lambda: run_c4_prefill(capi, world, rank, stream))):
            workloads[name] = fn()
            torch.cuda.empty_cache()

    if rank != 0:
        _finish(world)
        return
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": k,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "us_per_step": round(ms_per_step * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; configs[0] distributions, random-init NVFP4 weights)",
        "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": 512,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": f"inputs larger than L2: {n_rep} rotating weight+cache replicas "
                         f"({n_rep * replica_bytes / 2**20:.0f} MiB > 2 x 126 MB L2)",
                   "timing": f"CUDA graph of {n_rep} steps replayed, CUDA events"},
        "roofline": roofline,
        "kernels": kernels,
        "paths_us_per_step": {n: round(v * 1e3 / (reps_k * n_rep), 3) for n, v in path_ms.items()},
        "e2e": e2e,
        "workloads": workloads,
        "gpu_launches": (1 if step_supported else 3) * k,
        "clocks": clk,
    }
    if world == 1 and not args.skip_cpu:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    print(json.dumps(line), flush=True)
    _finish(world)


# ---------------------------------------------------------------- sharded workloads (sub-objects of the line)
def _quantized_weights(inp, capi):
    from nvfp4_tensor import NVFP4Tensor

    ws = {}
    for k, w in inp.weights_fp32.items():
        packed, scales, gamma = capi.quantize(w.cuda())
        ws[k] = NVFP4Tensor(packed, scales, gamma, tuple(w.shape))
    return ws


def _weight_bytes(h: int, kvw: int) -> int:
    w = lambda n, k: n * (k // 2 + k // 16) + 4  # noqa: E731
    return 2 * w(h, h) + 2 * w(kvw, h)


def _time_steps(fn, steps: int, warmup: int, stream, world: int, graph_ok: bool = True):
    """Device ms of `steps` calls of fn (replays of a CUDA graph of one call
    when graph_ok and it captures, else eager), max over ranks; and whether a
    graph was used."""
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            fn()
    torch.cuda.synchronize()
    graph = None
    if graph_ok:
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                fn()
            graph = g
        except Exception:
            torch.cuda.synchronize()
            graph = None
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            if graph is not None:
                graph.replay()
            else:
                fn()
        end.record(stream)
    end.synchronize()
    barrier(world)
    return max_over_ranks(start.elapsed_time(end), world), graph is not None


def run_c2_batch_sharded(capi, world, rank, stream, peak, steps=50) -> dict:
    """B=64, P_b ~ U[1024, 8191] (seeded), C=8192; the 64
    sequences split into contiguous groups of 64/N, one per rank, each rank
    running the forward on its own group with device-side past lengths (no
    collective on the data path)."""
    import synthetic

    full = synthetic.batched_shape()
    if full.batch % world:
        return {"skipped": f"B=64 does not split over {world} ranks"}
    per = full.batch // world
    pasts = full.past_lengths[rank * per:(rank + 1) * per]
    shape = synthetic.DecodeShape(batch=per, capacity=full.capacity, past_lengths=tuple(pasts))
    inp = synthetic.make_decode_inputs(shape, seed=2 + rank, cache_device="cuda")
    ws = _quantized_weights(inp, capi)
    h, kvw = shape.hidden, shape.kv_width
    kv_read = sum((p + 1) * 2 * kvw * 2 for p in pasts)
    bytes_rank = _weight_bytes(h, kvw) + kv_read + per * 2 * kvw * 2 + 2 * per * h * 2
    # Rotate cache replicas so that one step's traffic stays above 2 x L2.
    n_rep = max(1, math.ceil(2 * L2_BYTES / bytes_rank))
    x, g_in = inp.x.cuda(), inp.input_norm_weight.cuda()
    g_q, g_k = inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda()
    pl = torch.tensor(pasts, dtype=torch.int64, device="cuda")
    fws = []
    for r in range(n_rep):
        kc = inp.k_cache if r == 0 else inp.k_cache.clone()
        vc = inp.v_cache if r == 0 else inp.v_cache.clone()
        out = torch.empty_like(x)
        fws.append(capi.Forward(x, g_in, ws["q"], ws["k"], ws["v"], g_q, g_k, ws["o"], kc, vc, out, past_length=0,
                                past_lengths=pl, max_past_length=max(pasts)))

    def step_all():
        for fw in fws:
            fw.run(stream)

    reps = max(1, steps // n_rep)
    ms, graphed = _time_steps(step_all, reps, 3, stream, world)
    ms_step = ms / (reps * n_rep)
    # bytes of the slowest rank bound the step; report this rank's and the job's
    gbs = bytes_rank / (ms_step * 1e-3) / 1e9
    tot = torch.tensor([float(bytes_rank)], dtype=torch.float64, device="cuda")
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(tot)
    return {"config": "configs[2]: B=64 T=1 P_b~U[1024,8191] seed 2024 C=8192, batch-sharded "
                      f"{per} sequences per rank", "ranks": world,
            "tokens_per_s": round(full.batch / (ms_step * 1e-3), 1), "ms_per_step": round(ms_step, 5),
            "hbm_gbs_per_gpu": round(gbs, 1), "frac_per_gpu": round(gbs / peak, 4),
            "bytes_per_step_job": int(tot.item()), "bytes_per_step_rank0": bytes_rank,
            "path": ("input RMSNorm + batched QKV/head epilogue (4-CTA clusters, split K) + streaming split-KV "
                     "attention + batched O projection (4 PDL-chained launches per rank)"),
            "replicas": n_rep, "graph": graphed, "steps": reps * n_rep}


def run_c3_kv_sharded(capi, world, rank, stream, peak, steps=30) -> dict:
    """B=8, P=32767, C=32768; the KV length split into N
    contiguous shards, one per rank: replicated projections, per-shard
    log-sum-exp partials, NCCL all-gather of the partials, combine, O."""
    import synthetic
    from kv_sharding import ShardedDecoderAttention

    full = synthetic.LONG_CONTEXT
    sda = ShardedDecoderAttention(full.capacity, group=None)
    shard = sda.shard
    shape = synthetic.DecodeShape(batch=full.batch, capacity=shard.capacity, past_lengths=full.past_lengths)
    inp = synthetic.make_decode_inputs(shape, seed=3 + rank, cache_device="cuda")
    ws = _quantized_weights(inp, capi)
    x, g_in = inp.x.cuda(), inp.input_norm_weight.cuda()
    g_q, g_k = inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda()
    past = full.past_lengths[0]
    h, kvw, b = shape.hidden, shape.kv_width, shape.batch
    visible = max(0, min(shard.capacity, past + 1 - shard.start))
    gather = world * b * shape.q_heads * (shape.head_dim + 2) * 4
    bytes_rank = _weight_bytes(h, kvw) + b * visible * 2 * kvw * 2 + 2 * b * h * 2 + gather

    def step():
        sda.forward_(x, g_in, ws["q"], ws["k"], ws["v"], g_q, g_k, ws["o"], inp.k_cache, inp.v_cache, past)

    # Eager at N > 1 (the step holds an NCCL collective); a graph of 4 steps at N = 1.
    ms, graphed = _time_steps(lambda: [step() for _ in range(4)], max(1, steps // 4), 3, stream, world,
                              graph_ok=world == 1)
    ms_step = ms / (4 * max(1, steps // 4))
    # the all-gather alone (same partial size), for its share of the step
    ag_share = None
    if world > 1:
        import torch.distributed as dist

        part = torch.zeros((b * shape.q_heads, shape.head_dim + 2), dtype=torch.float32, device="cuda")
        flat = torch.empty((world * part.shape[0], part.shape[1]), dtype=torch.float32, device="cuda")
        ag_ms, _ = _time_steps(lambda: dist.all_gather_into_tensor(flat, part), 50, 3, stream, world,
                               graph_ok=False)
        ag_share = round((ag_ms / 50) / ms_step, 4)
    gbs = bytes_rank / (ms_step * 1e-3) / 1e9
    return {"config": f"configs[3]: B=8 T=1 P=32767 C=32768, KV length sharded {shard.capacity} positions per rank",
            "ranks": world, "tokens_per_s": round(b / (ms_step * 1e-3), 1), "ms_per_step": round(ms_step, 5),
            "hbm_gbs_per_gpu": round(gbs, 1), "frac_per_gpu": round(gbs / peak, 4),
            "bytes_per_step_rank0": bytes_rank, "allgather_share_of_step": ag_share,
            "path": "fused front half (shard append) + streaming attention partials + NCCL all-gather "
                    "+ combine + O GEMV", "graph": graphed, "steps": 4 * max(1, steps // 4)}


def run_c4_prefill(capi, world, rank, stream, steps=10) -> dict:
    """B=4, T=2048, P=0, C=4096 on every rank (replicas: the
    prefill batch does not shard in this design).  Tensor roofline on the
    GEMM and the causal attention."""
    import synthetic

    shape = synthetic.PREFILL
    inp = synthetic.make_decode_inputs(shape, seed=4, cache_device="cuda")
    ws = _quantized_weights(inp, capi)
    x = inp.x.cuda()
    out = torch.empty_like(x)
    fw = capi.Forward(x, inp.input_norm_weight.cuda(), ws["q"], ws["k"], ws["v"], inp.q_norm_weight.cuda(),
                      inp.k_norm_weight.cuda(), ws["o"], inp.k_cache, inp.v_cache, out, past_length=0)
    m, h, kvw = shape.batch * shape.tokens, shape.hidden, shape.kv_width
    ms, _ = _time_steps(lambda: fw.run(stream), steps, 3, stream, world)
    ms_step = ms / steps
    xin = torch.randn((m, h), device="cuda").to(torch.bfloat16)
    y = torch.empty((m, h), dtype=torch.bfloat16, device="cuda")
    g_ms, _ = _time_steps(lambda: capi.w4a16_gemm(xin, ws["q"], y, stream), steps, 3, stream, world)
    lib = capi.load()
    q = torch.randn((shape.batch, shape.tokens, shape.q_heads, shape.head_dim), device="cuda").to(torch.bfloat16)
    ctx = torch.empty_like(q)
    wsb = lib.nvfp4da_gqa_attention_workspace_size(shape.batch, shape.tokens, shape.q_heads, shape.kv_heads,
                                                   shape.head_dim, 0)
    aws = torch.empty(max(wsb, 256), dtype=torch.uint8, device="cuda")

    def attn():
        st = lib.nvfp4da_gqa_attention_cached(q.data_ptr(), inp.k_cache.data_ptr(), inp.v_cache.data_ptr(),
                                              ctx.data_ptr(), shape.batch, shape.tokens, shape.q_heads,
                                              shape.kv_heads, shape.capacity, shape.head_dim, 0, None, 0,
                                              aws.data_ptr(), wsb, stream.cuda_stream)
        assert st == 0, lib.nvfp4da_last_error()

    a_ms, _ = _time_steps(attn, steps, 3, stream, world)
    try:
        peak = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
        src = "measured (MEASURED_PEAKS.json bf16_tflops)"
    except Exception:
        peak, src = 1590.0, "fallback 1.59 PFLOP/s"
    gemm_fl = 2.0 * m * h * h
    attn_fl = 2.0 * 2.0 * shape.batch * shape.q_heads * (shape.tokens * (shape.tokens + 1) / 2) * shape.head_dim
    step_fl = 2.0 * m * h * (2 * h + 2 * kvw) + attn_fl
    g_tf = gemm_fl / (g_ms / steps * 1e-3) / 1e12
    a_tf = attn_fl / (a_ms / steps * 1e-3) / 1e12
    return {"config": "configs[4]: B=4 T=2048 P=0 C=4096 (replicated per rank)", "ranks": world,
            "tokens_per_s": round(world * m / (ms_step * 1e-3), 1), "ms_per_step": round(ms_step, 4),
            "step_tflops": round(step_fl / (ms_step * 1e-3) / 1e12, 1),
            "gemm_q_tflops": round(g_tf, 1), "gemm_frac": round(g_tf / peak, 4),
            "attention_tflops": round(a_tf, 1), "attention_frac": round(a_tf / peak, 4),
            "attention_ms": round(a_ms / steps, 4), "peak_tflops": peak, "peak_source": src,
            "flops_note": "attention counts the causal half: 4*B*Hq*D*T(T+1)/2"}


def run_prefill(args) -> None:
    """configs[4] (B=4, T=2048, P=0, C=4096): the prefill forward (modular chain
    with tcgen05 GEMM projections); not the default workload.  Roofline on the
    tensor-core GEMM (BF16 dense, measured cuBLAS peak)."""
    world, rank, local = dist_setup()
    import nvfp4da_capi as capi
    import synthetic
    from nvfp4_tensor import NVFP4Tensor

    capi.load()
    shape = synthetic.DecodeShape(batch=4, tokens=2048, hidden=3072, kv_heads=6, head_dim=128, capacity=4096,
                                  past_lengths=(0,))
    inp = synthetic.make_decode_inputs(shape, seed=0)
    ws = {}
    for k, w in inp.weights_fp32.items():
        packed, scales, gamma = capi.quantize(w.cuda())
        ws[k] = NVFP4Tensor(packed, scales, gamma, tuple(w.shape))
    x = inp.x.cuda()
    kc, vc = inp.k_cache.cuda(), inp.v_cache.cuda()
    out = torch.empty_like(x)
    fw = capi.Forward(x, inp.input_norm_weight.cuda(), ws["q"], ws["k"], ws["v"], inp.q_norm_weight.cuda(),
                      inp.k_norm_weight.cuda(), ws["o"], kc, vc, out, past_length=0)
    stream = torch.cuda.Stream()
    m, h, kvw = 4 * 2048, 3072, 6 * 128
    xin = torch.randn((m, h), device="cuda").to(torch.bfloat16)
    y = torch.empty((m, h), dtype=torch.bfloat16, device="cuda")
    yk = torch.empty((m, kvw), dtype=torch.bfloat16, device="cuda")
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            fw.run(stream)
            capi.w4a16_gemm(xin, ws["q"], y, stream)
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 20))
    ms = timed_graph([lambda: fw.run(stream)], steps, stream) / steps
    gemm_ms = {
        "q_or_o": timed_graph([lambda: capi.w4a16_gemm(xin, ws["q"], y, stream)], steps, stream) / steps,
        "k_or_v": timed_graph([lambda: capi.w4a16_gemm(xin, ws["k"], yk, stream)], steps, stream) / steps,
    }
    fl = {"q_or_o": 2.0 * m * h * h, "k_or_v": 2.0 * m * kvw * h}
    tflops = {n: fl[n] / (gemm_ms[n] * 1e-3) / 1e12 for n in fl}
    try:
        peak = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
        src = "measured (MEASURED_PEAKS.json bf16_tflops)"
    except Exception:
        peak, src = 1590.0, "fallback 1.59 PFLOP/s"
    step_flops = 2.0 * m * h * (h + 2 * kvw + h) + 4 * 24 * 2 * 2048 * 2048 * 128  # projections + causal attention
    if rank == 0:
        print(json.dumps({
            "metric": "prefill tokens/s (configs[4])", "value": round(m / (ms * 1e-3), 1), "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; configs[4] distributions, random-init NVFP4 weights)",
            "config": {"workload": "configs[4] prefill: B=4 T=2048 H=3072 Hq=24 Hkv=6 D=128 P=0 C=4096",
                       "global_batch": 4, "seq_len": 2048, "parallelism": "single"},
            "roofline": {"bound": "tensor", "kernel": "w4a16_gemm_tc_kernel (Q/O projection, M=8192 N=3072 K=3072)",
                         "achieved": round(tflops["q_or_o"], 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tflops["q_or_o"] / peak, 4), "peak_source": src, "traffic": None},
            "gemm_ms": {n: round(v, 4) for n, v in gemm_ms.items()},
            "gemm_tflops": {n: round(v, 1) for n, v in tflops.items()},
            "step_tflops": round(step_flops / (ms * 1e-3) / 1e12, 1),
            "gpu_launches": 11 * steps,  # norm, 3 GEMMs, 2 head norms, 2 RoPE, append, attention, O GEMM
        }), flush=True)
    _finish(world)


def run_attention_workload(args) -> None:
    """One attention kernel on its config, timed alone (a separate line, not
    the default workload): attention-c3 = configs[3] decode attention (B=8,
    P=32767, C=32768; the streaming kernel, HBM roofline), attention-c4 =
    configs[4] causal prefill attention (B=4, T=2048; tcgen05, tensor
    roofline)."""
    world, rank, local = dist_setup()
    import nvfp4da_capi as capi

    lib = capi.load()
    c3 = args.workload == "attention-c3"
    b, t, hq, hkv, d = (8, 1, 24, 6, 128) if c3 else (4, 2048, 24, 6, 128)
    cap, past = (32768, 32767) if c3 else (4096, 0)
    if c3 and args.positions:  # a shorter cache of the same shape (profiling captures)
        cap, past = args.positions, args.positions - 1
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn((b, t, hq, d), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((b, hkv, cap, d), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((b, hkv, cap, d), generator=g, device="cuda").to(torch.bfloat16)
    ctx = torch.empty_like(q)
    wsb = lib.nvfp4da_gqa_attention_workspace_size(b, t, hq, hkv, d, past)
    ws = torch.zeros(max(wsb, 256), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()

    def call():
        st = lib.nvfp4da_gqa_attention_cached(q.data_ptr(), k.data_ptr(), v.data_ptr(), ctx.data_ptr(), b, t, hq,
                                              hkv, cap, d, past, None, past, ws.data_ptr(), wsb, stream.cuda_stream)
        assert st == 0, lib.nvfp4da_last_error()

    steps = max(3, min(args.steps, 50))
    ms, _ = _time_steps(call, steps, max(args.warmup, 3), stream, world)
    ms /= steps
    if c3:
        byts = b * (past + 1) * 2 * hkv * d * 2 + 2 * b * hq * d * 2
        peak, src = measured_peak_gbs()
        ach = byts / (ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "peak_source": src, "bytes_per_launch": byts,
                "traffic": None if args.positions else ncu_traffic("attn_stream", "attn_stream_configs3.md"),
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch "
                                  "(profiles/attn_stream_configs3.md)"}
        metric, value, unit = "configs[3] decode attention HBM GB/s", round(ach, 1), "GB/s"
    else:
        fl = 4.0 * b * hq * d * t * (t + 1) / 2
        try:
            peak = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
            src = "measured (MEASURED_PEAKS.json bf16_tflops)"
        except Exception:
            peak, src = 1590.0, "fallback 1.59 PFLOP/s"
        ach = fl / (ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(ach / peak, 4), "peak_source": src, "flops_per_launch": fl,
                "flops_note": "the causal half: 4*B*Hq*D*T(T+1)/2"}
        metric, value, unit = "configs[4] causal prefill attention TFLOP/s", round(ach, 1), "TFLOP/s"
    if rank == 0:
        print(json.dumps({"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": steps,
                          "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
                          "dtype": "bf16", "data": "synthetic (seeded N(0,1) q/k/v)",
                          "config": {"workload": args.workload, "capacity": cap, "past_length": past},
                          "roofline": roof}), flush=True)
    _finish(world)


def run_projections_workload(args) -> None:
    """configs[2]'s projections alone (a separate line, not the default
    workload): the batched front half (input RMSNorm + RoPE table, then Q/K/V
    with per-head norm, RoPE and cache append in 4-CTA clusters) and the
    batched O projection at M = 64 rows, each timed over 12 rotating weight
    replicas (160 MB > L2).  Roofline: HBM bytes of weights and rows, and the
    tensor FLOPs beside them."""
    world, rank, local = dist_setup()
    import nvfp4da_capi as capi
    import synthetic

    lib = capi.load()
    b, h, hkv, d, cap = 64, 3072, 6, 128, 16
    shape = synthetic.DecodeShape(batch=b, capacity=cap, past_lengths=tuple(i % cap for i in range(b)))
    inp = synthetic.make_decode_inputs(shape, seed=5, cache_device="cuda")
    x, g_in = inp.x.cuda(), inp.input_norm_weight.cuda()
    g_q, g_k = inp.q_norm_weight.cuda(), inp.k_norm_weight.cuda()
    ctx = torch.randn((b, h), generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).cuda()
    y = torch.empty_like(ctx)
    pl = torch.tensor(shape.past_lengths, dtype=torch.int64, device="cuda")
    reps = []
    for _ in range(12):
        ws = _quantized_weights(inp, capi)
        q = torch.empty((b, 1, h // d, d), dtype=torch.bfloat16, device="cuda")
        fw = capi.Forward(x, g_in, ws["q"], ws["k"], ws["v"], g_q, g_k, ws["o"], inp.k_cache, inp.v_cache, y,
                          past_length=0, past_lengths=pl, max_past_length=cap - 1)
        wsb = lib.nvfp4da_qkv_rope_append_shard_workspace_size(C_byref(fw.args))
        assert wsb > 0, "the batched front half does not cover configs[2]"
        buf = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        reps.append((fw, ws, q, buf, wsb))
    stream = torch.cuda.Stream()

    def front():
        for fw, _, q, buf, wsb in reps:
            st = lib.nvfp4da_qkv_rope_append_shard(C_byref(fw.args), 0, cap, q.data_ptr(), buf.data_ptr(), wsb,
                                                   stream.cuda_stream)
            assert st == 0, lib.nvfp4da_last_error()

    def oproj():
        for _, ws, _, _, _ in reps:
            capi.w4a16_linear(ctx, ws["o"], y, stream)

    steps = max(3, min(args.steps, 200))
    res = {}
    for name, fn, n_out, k_rows in (("front", front, h + 2 * hkv * d, h), ("o_proj", oproj, h, h)):
        ms, _ = _time_steps(fn, steps, max(args.warmup, 3), stream, world)
        us = ms / (steps * len(reps)) * 1e3
        byts = n_out * (k_rows // 2 + k_rows // 16) + 2 * b * k_rows * 2 + (b * 2 * hkv * d * 2 if name == "front" else 0)
        fl = 2.0 * b * n_out * k_rows
        res[name] = {"us": round(us, 3), "hbm_bytes": byts, "hbm_gbs": round(byts / (us * 1e-6) / 1e9, 1),
                     "tflops": round(fl / (us * 1e-6) / 1e12, 1)}
    peak, src = measured_peak_gbs()
    tot_us = res["front"]["us"] + res["o_proj"]["us"]
    tot_b = res["front"]["hbm_bytes"] + res["o_proj"]["hbm_bytes"]
    ach = tot_b / (tot_us * 1e-6) / 1e9
    if rank == 0:
        print(json.dumps({"metric": "configs[2] batched projections us per step (M=64)", "value": round(tot_us, 3),
                          "unit": "us", "n_gpus": world, "steps": steps, "warmup": args.warmup,
                          "higher_is_better": False, "dtype": "bf16 MMA on exact W4A16 products, fp32 accumulate",
                          "data": "synthetic (seeded), 12 rotating weight replicas (160 MB > L2)",
                          "config": {"workload": args.workload, "rows": b, "hidden": h},
                          "kernels": res,
                          "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                                       "frac": round(ach / peak, 4), "peak_source": src, "traffic": None}}),
              flush=True)
    _finish(world)


def C_byref(obj):
    import ctypes

    return ctypes.byref(obj)


def run_e2e_hostio(args, reps, stream, world) -> dict:
    """Same metric through the C ABI with host buffers: one library call per
    step copies a pinned host input in, runs the forward and copies the output
    back (nvfp4da_decoder_attention_forward_hostio), all inside the timing."""
    n = max(10, min(args.steps, args.e2e_steps))
    x_host = [r.x.cpu().pin_memory() for r in reps]
    out_host = torch.empty((1, 1, 3072), dtype=torch.bfloat16).pin_memory()
    with torch.cuda.stream(stream):
        for i in range(10):
            reps[i % len(reps)].fw.run_hostio(x_host[i % len(reps)], out_host, stream)
        torch.cuda.synchronize()
        barrier(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(n):
            reps[i % len(reps)].fw.run_hostio(x_host[i % len(reps)], out_host, stream)
        end.record(stream)
    end.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world)
    return {"value": round(world * n / (ms / 1e3), 1), "unit": UNIT, "steps": n,
            "h2d_bytes_per_step": 3072 * 2, "d2h_bytes_per_step": 3072 * 2,
            "path": "C ABI nvfp4da_decoder_attention_forward_hostio (ctypes): pinned host x in, forward, "
                    "output out, one call per step"}


def run_e2e(args, reps, dac, stream, world) -> dict:
    """Same metric through cuda_decoder_attention_forward_ with pinned host
    input copied in and the output copied out every step (inside the timing)."""
    n = max(10, min(args.steps, args.e2e_steps))
    x_host = [r.x.cpu().pin_memory() for r in reps]
    out_host = torch.empty((1, 1, 3072), dtype=torch.bfloat16).pin_memory()

    def step(i):
        r = reps[i % len(reps)]
        r.x.copy_(x_host[i % len(reps)], non_blocking=True)
        y = dac.cuda_decoder_attention_forward_(r.x, r.g_in, r.ws["q"], r.ws["k"], r.ws["v"], r.g_q, r.g_k,
                                                r.ws["o"], r.kc, r.vc, 511)
        out_host.copy_(y, non_blocking=True)

    with torch.cuda.stream(stream):
        for i in range(10):
            step(i)
        torch.cuda.synchronize()
        barrier(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(n):
            step(i)
        end.record(stream)
    end.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world)
    return {"value": round(world * n / (ms / 1e3), 1), "unit": UNIT, "steps": n,
            "h2d_bytes_per_step": 3072 * 2, "d2h_bytes_per_step": 3072 * 2,
            "path": "decoder_attention_cuda.cuda_decoder_attention_forward_ (drop-in Python op), "
                    "pinned host x in, output out, per step"}


def _finish(world):
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# ---------------------------------------------------------------- CPU path (reference arm / cpu_baseline)
def _oracle_inputs():
    sys.path.insert(0, str(ROOT))
    import oracle
    import synthetic

    inp = synthetic.make_decode_inputs(synthetic.CANONICAL, seed=0)

    def bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()

    qw = {k: oracle.quantize(v.numpy()) for k, v in inp.weights_fp32.items()}
    return oracle, (bits(inp.x), bits(inp.input_norm_weight), qw, bits(inp.q_norm_weight),
                    bits(inp.k_norm_weight), bits(inp.k_cache), bits(inp.v_cache))


def cpu_rate(seconds: float, max_steps: int | None = None) -> dict:
    """Decode steps of the CPU restatement, one independent sequence per host
    thread (numpy releases the GIL in its kernels), for about `seconds`."""
    from concurrent.futures import ThreadPoolExecutor

    oracle, (x, g_in, qw, g_q, g_k, kc, vc) = _oracle_inputs()
    threads = os.cpu_count() or 1
    deadline = time.perf_counter() + seconds
    counts = [0] * threads

    def worker(i):
        kci, vci = kc.copy(), vc.copy()
        while time.perf_counter() < deadline and (max_steps is None or counts[i] < max_steps):
            oracle.decoder_attention_nvfp4(x, g_in, qw["q"], qw["k"], qw["v"], g_q, g_k, qw["o"], kci, vci, 511)
            counts[i] += 1

    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(worker, range(threads)))
    wall = time.perf_counter() - t0
    steps = sum(counts)
    return {"value": round(steps / wall, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{steps} canonical decode steps of oracle/ (numpy restatement of "
                      f"reference/decoder_attention_nvfp4.py), {threads} threads x independent sequences, "
                      f"{wall:.1f} s wall"}


def cpu_baseline(seconds: float) -> dict:
    return cpu_rate(seconds)


def run_reference(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # warm-up: one untimed step per thread, then a bounded timed sample.
    cpu_rate(1.0, max_steps=1)
    res = cpu_rate(args.cpu_seconds)
    line = {
        "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 / res["value"], 3) if res["value"] else None,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded; configs[0] distributions)", "impl": "reference",
        "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": 512, "parallelism": "host threads"},
        "cpu_baseline": res,
        "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "each step is a bounded sample: the timed run lasts about --cpu-seconds regardless of --steps",
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=160000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--e2e-steps", type=int, default=2000)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-workloads", action="store_true",
                    help="only the configs[0] line (no configs[2]/[3]/[4] sub-objects)")
    ap.add_argument("--workload", choices=("decode", "prefill", "attention-c3", "attention-c4", "projections-c2"),
                    default="decode",
                    help="decode = configs[0] (the metric's workload); prefill = configs[4], reported separately; "
                         "attention-c3 / attention-c4 = one attention kernel on configs[3] / configs[4]; "
                         "projections-c2 = the batched projections of configs[2] (M = 64)")
    ap.add_argument("--positions", type=int, default=0,
                    help="attention-c3 only: cache positions per sequence (default 32768, the config's)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload.startswith("attention-"):
        run_attention_workload(args)
    elif args.workload == "projections-c2":
        run_projections_workload(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
