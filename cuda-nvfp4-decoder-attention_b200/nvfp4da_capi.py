"""ctypes binding of the C ABI (``include/nvfp4_decoder_attention.h``).

This is the binding a non-PyTorch host would write; the parity tests and the benchmark call the kernels through it.  Tensors passed in
must already live on the current CUDA device; the helpers only take their data
pointers and sizes.  ``CapiError`` carries the library's status and message.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("NVFP4DA_LIBRARY",
                               Path(__file__).resolve().parent / "lib" / "libnvfp4da.so"))

OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA = 0, 1, 2, 3, 4

# Every symbol the header declares (checked by the CPU test suite).
EXPORTED = (
    "nvfp4da_last_error", "nvfp4da_abi_version", "nvfp4da_unpack_e2m1_codes", "nvfp4da_dequantize_nvfp4",
    "nvfp4da_quantize_workspace_size", "nvfp4da_quantize_nvfp4", "nvfp4da_rms_norm", "nvfp4da_apply_rope",
    "nvfp4da_w4a16_linear", "nvfp4da_kv_cache_append", "nvfp4da_gqa_attention_workspace_size",
    "nvfp4da_gqa_attention_cached", "nvfp4da_forward_workspace_size", "nvfp4da_decoder_attention_forward",
    "nvfp4da_qkv_rope_append", "nvfp4da_decoder_attention_forward_noalloc",
    "nvfp4da_decoder_attention_forward_path", "nvfp4da_forward_step_supported", "nvfp4da_forward_sync_status",
    "nvfp4da_debug_wait_timeout", "nvfp4da_qkv_rope_append_shard", "nvfp4da_qkv_rope_append_shard_workspace_size",
    "nvfp4da_gqa_attention_partials_workspace_size", "nvfp4da_gqa_attention_partials",
    "nvfp4da_attention_combine", "nvfp4da_w4a16_gemm", "nvfp4da_decoder_attention_forward_hostio",
)

PATH_AUTO, PATH_CHAIN, PATH_STEP = 0, 1, 2


class CapiError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"nvfp4da status {status}: {message}")
        self.status = status


class Weight(C.Structure):
    _fields_ = [("packed_values", C.c_void_p), ("block_scales", C.c_void_p),
                ("global_decode_scale", C.c_void_p), ("rows", C.c_int64), ("cols", C.c_int64)]


class Stages(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("input_normalized", "q_projected", "k_projected", "v_projected",
                                          "q_normalized", "k_normalized", "q_rope", "context")]


class ForwardArgs(C.Structure):
    _fields_ = [("x", C.c_void_p), ("input_norm_weight", C.c_void_p), ("q_weight", Weight),
                ("k_weight", Weight), ("v_weight", Weight), ("out_weight", Weight),
                ("q_norm_weight", C.c_void_p), ("k_norm_weight", C.c_void_p), ("k_cache", C.c_void_p),
                ("v_cache", C.c_void_p), ("output", C.c_void_p), ("batch", C.c_int64), ("tokens", C.c_int64),
                ("hidden", C.c_int64), ("kv_heads", C.c_int64), ("head_dim", C.c_int64),
                ("capacity", C.c_int64), ("past_length", C.c_int64), ("past_lengths", C.c_void_p),
                ("max_past_length", C.c_int64), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("stages", C.POINTER(Stages))]


_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Load ``libnvfp4da.so`` (raises ``OSError`` if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.is_file():
        raise OSError(f"{LIB_PATH} not found; run `python cuda-nvfp4-decoder-attention_b200/build.py`")
    lib = C.CDLL(str(LIB_PATH))
    i64, vp, sz = C.c_int64, C.c_void_p, C.c_size_t
    sig = {
        "nvfp4da_last_error": (C.c_char_p, []),
        "nvfp4da_abi_version": (C.c_int, []),
        "nvfp4da_unpack_e2m1_codes": (C.c_int, [vp, vp, i64, i64, vp]),
        "nvfp4da_dequantize_nvfp4": (C.c_int, [C.POINTER(Weight), vp, vp]),
        "nvfp4da_quantize_workspace_size": (sz, [i64, i64]),
        "nvfp4da_quantize_nvfp4": (C.c_int, [vp, C.c_int, i64, i64, vp, vp, vp, vp, sz, vp]),
        "nvfp4da_rms_norm": (C.c_int, [vp, vp, vp, i64, i64, C.c_float, vp]),
        "nvfp4da_apply_rope": (C.c_int, [vp, vp, i64, i64, i64, i64, i64, C.c_float, vp]),
        "nvfp4da_w4a16_linear": (C.c_int, [vp, i64, C.POINTER(Weight), vp, vp]),
        "nvfp4da_kv_cache_append": (C.c_int, [vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, vp, vp]),
        "nvfp4da_gqa_attention_workspace_size": (sz, [i64, i64, i64, i64, i64, i64]),
        "nvfp4da_gqa_attention_cached": (C.c_int, [vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, vp, i64,
                                                   vp, sz, vp]),
        "nvfp4da_forward_workspace_size": (sz, [C.POINTER(ForwardArgs)]),
        "nvfp4da_decoder_attention_forward": (C.c_int, [C.POINTER(ForwardArgs), vp, sz, vp]),
        "nvfp4da_qkv_rope_append": (C.c_int, [C.POINTER(ForwardArgs), vp, vp]),
        "nvfp4da_decoder_attention_forward_noalloc": (C.c_int, [C.POINTER(ForwardArgs), vp]),
        "nvfp4da_decoder_attention_forward_path": (C.c_int, [C.POINTER(ForwardArgs), vp, sz, vp, C.c_int]),
        "nvfp4da_forward_step_supported": (C.c_int, [C.POINTER(ForwardArgs)]),
        "nvfp4da_forward_sync_status": (C.c_int, [vp, C.POINTER(C.c_uint), C.c_int]),
        "nvfp4da_debug_wait_timeout": (C.c_int, [vp, C.c_ulonglong, C.POINTER(C.c_uint)]),
        "nvfp4da_qkv_rope_append_shard": (C.c_int, [C.POINTER(ForwardArgs), i64, i64, vp, vp, sz, vp]),
        "nvfp4da_qkv_rope_append_shard_workspace_size": (sz, [C.POINTER(ForwardArgs)]),
        "nvfp4da_gqa_attention_partials_workspace_size": (sz, [i64, i64, i64, i64, i64, i64, i64, i64]),
        "nvfp4da_gqa_attention_partials": (C.c_int, [vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, i64, vp,
                                                     i64, vp, sz, vp]),
        "nvfp4da_attention_combine": (C.c_int, [vp, C.c_int, i64, i64, vp, vp]),
        "nvfp4da_w4a16_gemm": (C.c_int, [vp, i64, C.POINTER(Weight), vp, vp]),
        "nvfp4da_decoder_attention_forward_hostio": (C.c_int, [C.POINTER(ForwardArgs), vp, vp, vp, sz, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _check(status: int) -> None:
    if status != OK:
        raise CapiError(status, load().nvfp4da_last_error().decode())


def _p(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream: torch.cuda.Stream | None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def weight(w) -> Weight:
    """C view of an NVFP4Tensor-like object (device tensors)."""
    rows, cols = (int(v) for v in w.logical_shape)
    return Weight(w.packed_values.data_ptr(), w.block_scales.data_ptr(), w.global_decode_scale.data_ptr(),
                  rows, cols)


# ---------------------------------------------------------------- wrappers
def w4a16_linear(x: torch.Tensor, w, y: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    rows, cols = (int(v) for v in w.logical_shape)
    m = x.numel() // cols
    if y is None:
        y = torch.empty((*x.shape[:-1], rows), dtype=torch.bfloat16, device=x.device)
    wt = weight(w)
    _check(load().nvfp4da_w4a16_linear(_p(x), m, C.byref(wt), _p(y), _stream(stream)))
    return y


def w4a16_gemm(x: torch.Tensor, w, y: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """The projection forced onto the tcgen05 tensor-core GEMM."""
    rows, cols = (int(v) for v in w.logical_shape)
    m = x.numel() // cols
    if y is None:
        y = torch.empty((*x.shape[:-1], rows), dtype=torch.bfloat16, device=x.device)
    wt = weight(w)
    _check(load().nvfp4da_w4a16_gemm(_p(x), m, C.byref(wt), _p(y), _stream(stream)))
    return y


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, stream=None) -> torch.Tensor:
    out = torch.empty_like(x)
    _check(load().nvfp4da_rms_norm(_p(x), _p(w), _p(out), x.numel() // x.shape[-1], x.shape[-1], eps,
                                   _stream(stream)))
    return out


def apply_rope(x: torch.Tensor, past_length: int, theta: float, stream=None) -> torch.Tensor:
    out = torch.empty_like(x)
    b, t, h, d = x.shape
    _check(load().nvfp4da_apply_rope(_p(x), _p(out), b, t, h, d, past_length, theta, _stream(stream)))
    return out


def kv_cache_append(k_cache, v_cache, new_k, new_v, past_length: int, past_lengths=None, stream=None) -> None:
    b, hkv, c, d = k_cache.shape
    _check(load().nvfp4da_kv_cache_append(_p(k_cache), _p(v_cache), _p(new_k), _p(new_v), b, hkv, c, d,
                                          new_k.shape[1], past_length, _p(past_lengths), _stream(stream)))


def gqa_attention_cached(q, k_cache, v_cache, past_length: int, past_lengths=None, max_past_length=None,
                         stream=None) -> torch.Tensor:
    b, t, hq, d = q.shape
    hkv, c = k_cache.shape[1], k_cache.shape[2]
    maxp = past_length if max_past_length is None else max_past_length
    lib = load()
    wsb = lib.nvfp4da_gqa_attention_workspace_size(b, t, hq, hkv, d, maxp)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=q.device)
    ctx = torch.empty_like(q)
    _check(lib.nvfp4da_gqa_attention_cached(_p(q), _p(k_cache), _p(v_cache), _p(ctx), b, t, hq, hkv, c, d,
                                            past_length, _p(past_lengths), maxp, _p(ws), wsb, _stream(stream)))
    return ctx


def dequantize(w, stream=None) -> torch.Tensor:
    rows, cols = (int(v) for v in w.logical_shape)
    out = torch.empty((rows, cols), dtype=torch.float32, device=w.packed_values.device)
    wt = weight(w)
    _check(load().nvfp4da_dequantize_nvfp4(C.byref(wt), _p(out), _stream(stream)))
    return out


def unpack(packed: torch.Tensor, stream=None) -> torch.Tensor:
    out = torch.empty((packed.shape[0], packed.shape[1] * 2), dtype=torch.uint8, device=packed.device)
    _check(load().nvfp4da_unpack_e2m1_codes(_p(packed), _p(out), packed.shape[0], packed.shape[1],
                                            _stream(stream)))
    return out


def quantize(source: torch.Tensor, stream=None):
    """Returns (packed_values, block_scales, global_decode_scale) device tensors."""
    n, k = source.shape
    lib = load()
    packed = torch.empty((n, k // 2), dtype=torch.uint8, device=source.device)
    scales = torch.empty((n, k // 16), dtype=torch.uint8, device=source.device)
    gamma = torch.empty((), dtype=torch.float32, device=source.device)
    wsb = lib.nvfp4da_quantize_workspace_size(n, k)
    ws = torch.empty(wsb, dtype=torch.uint8, device=source.device)
    _check(lib.nvfp4da_quantize_nvfp4(_p(source), 1 if source.dtype == torch.bfloat16 else 0, n, k, _p(packed),
                                      _p(scales), _p(gamma), _p(ws), wsb, _stream(stream)))
    return packed, scales, gamma


def sync_status(stream=None, clear: bool = True) -> int:
    """Error flags of one-kernel steps on ``stream`` (bit 0: a bounded wait
    timed out); synchronises the stream."""
    flags = C.c_uint(0)
    _check(load().nvfp4da_forward_sync_status(_stream(stream), C.byref(flags), 1 if clear else 0))
    return flags.value


def wait_timeout_probe(timeout_ns: int, stream=None) -> int:
    """Run the bounded-wait self-test; returns its error flags."""
    flags = C.c_uint(0)
    _check(load().nvfp4da_debug_wait_timeout(_stream(stream), timeout_ns, C.byref(flags)))
    return flags.value


class Forward:
    """A prepared forward call: arguments and workspace bound once, then
    ``run()`` re-launches the kernels (the form a serving loop or a CUDA graph
    capture uses)."""

    def __init__(self, x, input_norm_weight, q_w, k_w, v_w, q_norm_weight, k_norm_weight, o_w, k_cache, v_cache,
                 output, past_length: int = 0, past_lengths: torch.Tensor | None = None,
                 max_past_length: int | None = None, rms_eps: float = 1e-6, rope_theta: float = 1e4,
                 stages: dict[str, torch.Tensor] | None = None):
        b, t, h = x.shape
        _, hkv, c, d = k_cache.shape
        # The C arguments hold raw pointers: keep every tensor they point into
        # (weights included) alive as long as this object.
        self._keep = [x, input_norm_weight, q_norm_weight, k_norm_weight, k_cache, v_cache, output, past_lengths,
                      q_w, k_w, v_w, o_w]
        self.args = ForwardArgs()
        a = self.args
        a.x, a.input_norm_weight = x.data_ptr(), input_norm_weight.data_ptr()
        a.q_weight, a.k_weight, a.v_weight, a.out_weight = weight(q_w), weight(k_w), weight(v_w), weight(o_w)
        a.q_norm_weight, a.k_norm_weight = q_norm_weight.data_ptr(), k_norm_weight.data_ptr()
        a.k_cache, a.v_cache, a.output = k_cache.data_ptr(), v_cache.data_ptr(), output.data_ptr()
        a.batch, a.tokens, a.hidden, a.kv_heads, a.head_dim, a.capacity = b, t, h, hkv, d, c
        a.past_length = past_length
        a.past_lengths = None if past_lengths is None else past_lengths.data_ptr()
        a.max_past_length = past_length if max_past_length is None else max_past_length
        a.rms_eps, a.rope_theta = rms_eps, rope_theta
        self._stages = None
        if stages:
            st = Stages()
            for k, v in stages.items():
                setattr(st, k, v.data_ptr())
            self._stages = st
            self._keep.extend(stages.values())
            a.stages = C.pointer(st)
        lib = load()
        self.workspace_bytes = lib.nvfp4da_forward_workspace_size(C.byref(a))
        if self.workspace_bytes == 0:
            raise CapiError(ERR_INVALID_ARGUMENT, lib.nvfp4da_last_error().decode())
        self.workspace = torch.empty(self.workspace_bytes, dtype=torch.uint8, device=x.device)

    def run(self, stream=None, path: int = PATH_AUTO) -> None:
        """One forward; ``path`` picks the kernels (PATH_AUTO: the one-kernel
        decode step where it applies, else the three-kernel chain)."""
        _check(load().nvfp4da_decoder_attention_forward_path(C.byref(self.args), _p(self.workspace),
                                                              self.workspace_bytes, _stream(stream), path))

    @property
    def step_supported(self) -> bool:
        return bool(load().nvfp4da_forward_step_supported(C.byref(self.args)))

    def run_qkv(self, q_rope_out: torch.Tensor, stream=None) -> None:
        """Only the fused front half (norm, QKV, per-head norm, RoPE, append)."""
        _check(load().nvfp4da_qkv_rope_append(C.byref(self.args), _p(q_rope_out), _stream(stream)))

    def run_hostio(self, x_host: torch.Tensor, out_host: torch.Tensor, stream=None) -> None:
        """One forward with host buffers: x_host -> x, forward, output ->
        out_host, enqueued on the stream in one library call (pinned host
        tensors keep the copies asynchronous)."""
        _check(load().nvfp4da_decoder_attention_forward_hostio(C.byref(self.args), _p(x_host), _p(out_host),
                                                                _p(self.workspace), self.workspace_bytes,
                                                                _stream(stream)))

    def run_noalloc(self, stream=None) -> None:
        """The same forward through the allocation-free entry point (scratch
        from the library's built-in device array instead of self.workspace)."""
        _check(load().nvfp4da_decoder_attention_forward_noalloc(C.byref(self.args), _stream(stream)))
