"""CPU checks of the drop-in boundary: the C-ABI library loads and exports
every function ``include/nvfp4_decoder_attention.h`` declares, and the
operator library registers the reference's nine schemas unchanged
(reference src/bindings.cpp:888-916).  No kernel is launched."""

from __future__ import annotations

import ctypes
import re

import pytest
import torch

from conftest import PACKAGE_DIR, REPO

HEADER = REPO / "include" / "nvfp4_decoder_attention.h"

REFERENCE_SCHEMAS = {
    "cuda_unpack_e2m1_codes": "cuda_unpack_e2m1_codes(Tensor packed_values) -> Tensor",
    "cuda_dequantize_nvfp4": "cuda_dequantize_nvfp4(Tensor packed_values, Tensor block_scales, "
                             "Tensor global_decode_scale) -> Tensor",
    "cuda_rms_norm": "cuda_rms_norm(Tensor x, Tensor weight, float eps) -> Tensor",
    "cuda_apply_rope": "cuda_apply_rope(Tensor x, int past_length, float rope_theta=10000.) -> Tensor",
    "cuda_w4a16_linear": "cuda_w4a16_linear(Tensor x, Tensor packed_values, Tensor block_scales, "
                         "Tensor global_decode_scale) -> Tensor",
    "cuda_w4a16_linear_grouped_decode": "cuda_w4a16_linear_grouped_decode(Tensor x, Tensor packed_values, "
                                        "Tensor block_scales, Tensor global_decode_scale) -> Tensor",
    "cuda_gqa_attention": "cuda_gqa_attention(Tensor q, Tensor present_k, Tensor present_v, int past_length) "
                          "-> Tensor",
    "cuda_gqa_attention_cached": "cuda_gqa_attention_cached(Tensor q, Tensor k_cache, Tensor v_cache, "
                                 "int past_length) -> Tensor",
    "cuda_kv_cache_append_": "cuda_kv_cache_append_(Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor new_k, "
                             "Tensor new_v, int past_length) -> ()",
}


def header_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"\b(nvfp4da_\w+)\s*\(", text))


def test_header_declares_the_exported_list():
    import nvfp4da_capi

    assert header_functions() == set(nvfp4da_capi.EXPORTED)


def test_capi_library_loads_and_exports_every_declared_symbol():
    import nvfp4da_capi

    lib = ctypes.CDLL(str(nvfp4da_capi.LIB_PATH))
    for name in header_functions():
        assert hasattr(lib, name), name
    bound = nvfp4da_capi.load()
    assert bound.nvfp4da_abi_version() == 1
    assert bound.nvfp4da_last_error() == b""


def test_capi_rejects_invalid_arguments_without_a_gpu():
    import nvfp4da_capi

    lib = nvfp4da_capi.load()
    st = lib.nvfp4da_rms_norm(None, None, None, 1, 8, 1e-6, None)
    assert st == nvfp4da_capi.ERR_INVALID_ARGUMENT
    assert b"invalid" in lib.nvfp4da_last_error()
    w = nvfp4da_capi.Weight(1, 1, 1, 4, 24)  # K not a multiple of 16
    assert lib.nvfp4da_dequantize_nvfp4(ctypes.byref(w), ctypes.c_void_p(16), None) == \
        nvfp4da_capi.ERR_INVALID_ARGUMENT
    assert b"multiple of 16" in lib.nvfp4da_last_error()
    # workspace sizing is pure host arithmetic
    assert lib.nvfp4da_quantize_workspace_size(8, 32) >= 4


def test_operator_library_registers_reference_schemas():
    import cuda_primitives  # noqa: F401

    ns = torch.ops.cuda_nvfp4_decoder_attention
    for name, schema in REFERENCE_SCHEMAS.items():
        op = getattr(ns, name)
        got = str(op.default._schema).replace("cuda_nvfp4_decoder_attention::", "")
        assert got == schema, (got, schema)
    for extra in ("cuda_decoder_attention_forward_", "cuda_decoder_attention_forward_varlen_",
                  "cuda_quantize_nvfp4"):
        assert hasattr(ns, extra)


def test_operators_reject_cpu_tensors_with_reference_messages():
    import cuda_primitives

    x = torch.ones((1, 1, 8), dtype=torch.bfloat16)
    w = torch.ones(8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="x must be a CUDA tensor"):
        cuda_primitives.cuda_rms_norm(x, w, 1e-6)
    with pytest.raises(RuntimeError, match="x must be a CUDA tensor"):
        cuda_primitives.cuda_apply_rope(x.reshape(1, 1, 1, 8), 0)
    with pytest.raises(TypeError, match="past_length must be an integer"):
        cuda_primitives.cuda_gqa_attention_cached(x, x, x, 1.0)
    with pytest.raises(TypeError, match="weight must be an NVFP4Tensor"):
        cuda_primitives.cuda_w4a16_linear(x, object())


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    import importlib
    import sys

    monkeypatch.setenv("CUDA_PRIMITIVES_LIBRARY", str(tmp_path / "absent.so"))
    saved = sys.modules.pop("cuda_primitives", None)
    try:
        with pytest.raises(ImportError, match="not found"):
            importlib.import_module("cuda_primitives")
    finally:
        sys.modules.pop("cuda_primitives", None)
        if saved is not None:
            sys.modules["cuda_primitives"] = saved


def test_forward_validation_runs_before_any_launch():
    import decoder_attention_cuda as dac

    x = torch.ones((1, 1, 8), dtype=torch.bfloat16)
    with pytest.raises(TypeError, match="past_length must be an integer"):
        dac.cuda_decoder_attention_forward_(x, x, None, None, None, x, x, None, x, x, 1.5)
    with pytest.raises(ValueError, match="past_length must be nonnegative"):
        dac.cuda_decoder_attention_forward_(x, x, None, None, None, x, x, None, x, x, -1)
    with pytest.raises(ValueError, match="x must be a CUDA tensor"):
        dac.cuda_decoder_attention_forward_(x, x, None, None, None, x, x, None, x, x, 0)


def test_package_has_no_oracle_imports():
    """The shipped package never imports the test oracle."""
    for f in PACKAGE_DIR.glob("*.py"):
        text = f.read_text()
        assert "import oracle" not in text and "from oracle" not in text, f
