"""Decoder-attention forward on B200 (drop-in for the reference's
``decoder_attention_cuda.py``, reference decoder_attention_cuda.py:149-417).

``cuda_decoder_attention_forward_`` keeps the reference signature and its
host-side validation (same exception types and messages, all raised before any
launch), then runs one registered operator.  For a T = 1 decode step that it
covers, the operator launches the one-kernel cooperative decode step (input
RMSNorm, Q/K/V projection, per-head norm, RoPE, cache append, split-KV
attention and O projection in one launch); otherwise three kernels chained by
programmatic dependent launch (fused front half; split-KV attention -- the
persistent streaming kernel for caches of 2,048 positions and more; O
projection), or for prefill-sized inputs the modular chain on the tensor-core
GEMM.  The trailing underscore means the physical ``[B, Hkv, C, D]`` caches are
mutated in place at slots ``past_length .. past_length + T - 1``.
"""

from __future__ import annotations

import math
import os

import torch

import cuda_primitives
from nvfp4_tensor import NVFP4Tensor, is_nvfp4_tensor

_ops = torch.ops.cuda_nvfp4_decoder_attention
_INT64_MAX = 2**63 - 1
# Debug switch: NVFP4DA_CHECK_WAITS=1 makes every forward synchronise its
# stream and raise if a bounded wait of the one-kernel step gave up.
_CHECK_WAITS = os.environ.get("NVFP4DA_CHECK_WAITS", "") not in ("", "0")


def check_wait_status(stream: torch.cuda.Stream | None = None) -> None:
    """Raise ``RuntimeError`` if a bounded wait of a one-kernel decode step on
    ``stream`` (default: the current stream) gave up since the last check.

    The step kernel orders its phases by polling words in device memory, each
    wait bounded in time; a wait that runs out records a flag and the kernel
    finishes with garbage output instead of hanging.  The forward itself never
    reads that flag back (it would cost a device-to-host synchronisation per
    call); this function does, synchronises the stream and clears the flag.
    """
    import nvfp4da_capi

    s = stream if stream is not None else torch.cuda.current_stream()
    try:
        flags = nvfp4da_capi.sync_status(s, clear=True)
    except nvfp4da_capi.CapiError as e:
        if e.status == nvfp4da_capi.ERR_UNSUPPORTED:  # no step slot: no one-kernel step ran on this stream
            s.synchronize()
            return
        raise
    if flags:
        raise RuntimeError(f"a bounded wait of the one-kernel decode step timed out (flags 0x{flags:x}); "
                           "the outputs of the forwards since the last check are not valid")


def _tensor(name: str, value: object, rank: int) -> torch.Tensor:
    if not isinstance(value, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if value.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if value.dtype != torch.bfloat16:
        raise TypeError(f"{name} must have dtype torch.bfloat16, got {value.dtype}")
    if value.ndim != rank:
        raise ValueError(f"{name} must have rank {rank}, got rank {value.ndim}")
    if not value.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if any(s <= 0 for s in value.shape):
        raise ValueError(f"{name} dimensions must all be positive")
    return value


def _real(name: str, value: object) -> float:
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError(f"{name} must be a real number")
    v = float(value)
    if not math.isfinite(v) or v <= 0.0:
        raise ValueError(f"{name} must be finite and positive, got {value}")
    return v


def _shape(name: str, t: torch.Tensor, expected: tuple) -> None:
    if tuple(t.shape) != expected:
        raise ValueError(f"{name} must have shape {expected}, got {tuple(t.shape)}")


def _weight(name: str, w: object, shape: tuple[int, int], device: torch.device):
    if not is_nvfp4_tensor(w):
        raise TypeError(f"{name} must be an NVFP4Tensor")
    if tuple(w.logical_shape) != shape:
        raise ValueError(f"{name}.logical_shape must be {shape}, got {tuple(w.logical_shape)}")
    rows, cols = shape
    for field, t, dtype, want in (("packed_values", w.packed_values, torch.uint8, (rows, cols // 2)),
                                  ("block_scales", w.block_scales, torch.uint8, (rows, cols // 16)),
                                  ("global_decode_scale", w.global_decode_scale, torch.float32, ())):
        q = f"{name}.{field}"
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{q} must be a torch.Tensor")
        if t.device.type != "cuda":
            raise ValueError(f"{q} must be a CUDA tensor")
        if t.device != device:
            raise ValueError(f"{q} must be on device {device}, got {t.device}")
        if t.dtype != dtype:
            raise TypeError(f"{q} must have dtype {dtype}, got {t.dtype}")
        if t.ndim != len(want):
            raise ValueError(f"{q} must have rank {len(want)}, got rank {t.ndim}")
        if not t.is_contiguous():
            raise ValueError(f"{q} must be contiguous")
        _shape(q, t, want)
    return w


def _validate(x, input_norm_weight, q_weight, k_weight, v_weight, q_norm_weight, k_norm_weight, out_weight,
              k_cache, v_cache, max_past: int, rms_eps, rope_theta):
    x = _tensor("x", x, 3)
    g_in = _tensor("input_norm_weight", input_norm_weight, 1)
    g_q = _tensor("q_norm_weight", q_norm_weight, 1)
    g_k = _tensor("k_norm_weight", k_norm_weight, 1)
    kc = _tensor("k_cache", k_cache, 4)
    vc = _tensor("v_cache", v_cache, 4)
    eps = _real("rms_eps", rms_eps)
    theta = _real("rope_theta", rope_theta)
    b, t, h = x.shape
    cb, hkv, cap, d = kc.shape
    if tuple(vc.shape) != tuple(kc.shape):
        raise ValueError(f"v_cache must have the same shape as k_cache, got {tuple(vc.shape)} and {tuple(kc.shape)}")
    if cb != b:
        raise ValueError(f"x and cache batch sizes must match ({b} != {cb})")
    if h % d:
        raise ValueError(f"hidden size must be divisible by cache head dimension ({h} % {d} != 0)")
    hq = h // d
    if hq % hkv:
        raise ValueError(f"number of query heads must be divisible by number of KV heads ({hq} % {hkv} != 0)")
    if d < 2 or d % 2:
        raise ValueError(f"cache head dimension must be even and at least 2, got {d}")
    if max_past > _INT64_MAX - t:
        raise OverflowError("past_length + current token count overflows int64")
    if max_past + t > cap:
        raise ValueError(f"past_length + current token count exceeds cache capacity ({max_past + t} > {cap})")
    dev = x.device
    for name, tensor in (("input_norm_weight", g_in), ("q_norm_weight", g_q), ("k_norm_weight", g_k),
                         ("k_cache", kc), ("v_cache", vc)):
        if tensor.device != dev:
            raise ValueError(f"{name} must be on device {dev}, got {tensor.device}")
    _shape("input_norm_weight", g_in, (h,))
    _shape("q_norm_weight", g_q, (d,))
    _shape("k_norm_weight", g_k, (d,))
    kvw = hkv * d
    ws = (_weight("q_weight", q_weight, (h, h), dev), _weight("k_weight", k_weight, (kvw, h), dev),
          _weight("v_weight", v_weight, (kvw, h), dev), _weight("out_weight", out_weight, (h, h), dev))
    return x, g_in, g_q, g_k, kc, vc, ws, eps, theta


def _flat(ws):
    q, k, v, o = ws
    return ((q.packed_values, q.block_scales, q.global_decode_scale),
            (k.packed_values, k.block_scales, k.global_decode_scale),
            (v.packed_values, v.block_scales, v.global_decode_scale),
            (o.packed_values, o.block_scales, o.global_decode_scale))


def cuda_decoder_attention_forward_(x, input_norm_weight, q_weight, k_weight, v_weight, q_norm_weight,
                                    k_norm_weight, out_weight, k_cache, v_cache, past_length, *,
                                    rms_eps: float = 1.0e-6, rope_theta: float = 10_000.0) -> torch.Tensor:
    """One decoder-attention forward over capacity-backed caches; appends K/V in place.

    Same contract as reference decoder_attention_cuda.py:149-164: x ``[B, T, H]``
    BF16, NVFP4 weights, BF16 caches ``[B, Hkv, C, D]``, ``past_length`` a
    Python int with ``past_length + T <= C``.  Returns ``[B, T, H]`` BF16.
    """
    if isinstance(past_length, bool) or not isinstance(past_length, int):
        raise TypeError("past_length must be an integer")
    if past_length < 0:
        raise ValueError(f"past_length must be nonnegative, got {past_length}")
    # Fast path: the operator itself checks every tensor property the Python
    # validation below checks (dtype, rank, contiguity, device, shapes,
    # capacity, eps/theta) before any launch.  NVFP4Tensor weights were
    # validated when constructed.  Only when the operator rejects the call is
    # the Python validation run, to raise the reference's exception type and
    # message.
    ws4 = (q_weight, k_weight, v_weight, out_weight)
    if all(type(w) is NVFP4Tensor for w in ws4) and type(rms_eps) is float and type(rope_theta) in (float, int):
        (qp, qs, qg), (kp, ks, kg), (vp, vs, vg), (op, os_, og) = _flat(ws4)
        try:
            y = _ops.cuda_decoder_attention_forward_(x, input_norm_weight, qp, qs, qg, kp, ks, kg, vp, vs, vg,
                                                     q_norm_weight, k_norm_weight, op, os_, og, k_cache, v_cache,
                                                     past_length, rms_eps, float(rope_theta))
            if _CHECK_WAITS:
                check_wait_status()
            return y
        except Exception:
            _validate(x, input_norm_weight, q_weight, k_weight, v_weight, q_norm_weight, k_norm_weight, out_weight,
                      k_cache, v_cache, past_length, rms_eps, rope_theta)
            raise
    x, g_in, g_q, g_k, kc, vc, ws, eps, theta = _validate(
        x, input_norm_weight, q_weight, k_weight, v_weight, q_norm_weight, k_norm_weight, out_weight, k_cache,
        v_cache, past_length, rms_eps, rope_theta)
    (qp, qs, qg), (kp, ks, kg), (vp, vs, vg), (op, os_, og) = _flat(ws)
    y = _ops.cuda_decoder_attention_forward_(x, g_in, qp, qs, qg, kp, ks, kg, vp, vs, vg, g_q, g_k, op, os_, og,
                                             kc, vc, past_length, eps, theta)
    if _CHECK_WAITS:
        check_wait_status()
    return y


def cuda_decoder_attention_forward_varlen_(x, input_norm_weight, q_weight, k_weight, v_weight, q_norm_weight,
                                           k_norm_weight, out_weight, k_cache, v_cache, past_lengths: torch.Tensor,
                                           max_past_length: int, *, rms_eps: float = 1.0e-6,
                                           rope_theta: float = 10_000.0) -> torch.Tensor:
    """Batched decode with one past length per sequence (extension, no reference counterpart).

    ``past_lengths`` is a CUDA int64 ``[B]`` tensor read only on the device;
    ``max_past_length`` is a host-side bound ``>= max(past_lengths)`` used to
    plan the split-KV grid (no device-to-host read).  Sequence ``b`` sees keys
    ``0 .. past_lengths[b] + t`` and appends at ``past_lengths[b] + t``.
    """
    if isinstance(max_past_length, bool) or not isinstance(max_past_length, int):
        raise TypeError("max_past_length must be an integer")
    if max_past_length < 0:
        raise ValueError(f"max_past_length must be nonnegative, got {max_past_length}")
    if not isinstance(past_lengths, torch.Tensor) or past_lengths.dtype != torch.int64:
        raise TypeError("past_lengths must be an int64 torch.Tensor")
    x, g_in, g_q, g_k, kc, vc, ws, eps, theta = _validate(
        x, input_norm_weight, q_weight, k_weight, v_weight, q_norm_weight, k_norm_weight, out_weight, k_cache,
        v_cache, max_past_length, rms_eps, rope_theta)
    (qp, qs, qg), (kp, ks, kg), (vp, vs, vg), (op, os_, og) = _flat(ws)
    y = _ops.cuda_decoder_attention_forward_varlen_(x, g_in, qp, qs, qg, kp, ks, kg, vp, vs, vg, g_q, g_k, op,
                                                    os_, og, kc, vc, past_lengths, max_past_length, eps, theta)
    if _CHECK_WAITS:
        check_wait_status()
    return y


__all__ = ["cuda_decoder_attention_forward_", "cuda_decoder_attention_forward_varlen_", "check_wait_status"]
