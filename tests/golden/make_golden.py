"""Generate the golden vectors in ``tests/golden/*.npz`` from the reference itself.

Runs in the build container only: it imports the reference's own PyTorch
correctness path (``reference/`` of PatrickZChen/cuda-nvfp4-decoder-attention)
from ``$NVFP4_REFERENCE_ROOT`` (default: the read-only mount next to this
repository).  The GPU box never runs it; tests read the committed ``.npz``.

Usage:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REF_ROOT = Path(os.environ.get("NVFP4_REFERENCE_ROOT", "/root/reference"))
sys.path.insert(0, str(REF_ROOT))
sys.path.insert(0, str(REPO / "cuda-nvfp4-decoder-attention_b200"))

from reference import (  # noqa: E402
    apply_rope_reference,
    decode_e2m1,
    decode_ue4m3,
    decoder_attention_nvfp4_reference,
    encode_e2m1,
    encode_ue4m3,
    gqa_attention_reference,
    quantize_nvfp4_reference,
    rms_norm_reference,
    w4a16_linear_reference,
)
import synthetic  # noqa: E402

torch.set_num_threads(max(1, os.cpu_count() or 1))


def bits(t: torch.Tensor) -> np.ndarray:
    assert t.dtype == torch.bfloat16
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).contiguous().numpy().copy()


def q_fields(prefix: str, q, out: dict) -> None:
    out[prefix + "packed"] = q.packed_values.numpy().copy()
    out[prefix + "scales"] = q.block_scales.numpy().copy()
    out[prefix + "gamma"] = np.float32(q.global_decode_scale.item())


def sha(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def gen(seed: int) -> torch.Generator:
    return torch.Generator(device="cpu").manual_seed(seed)


# ---------------------------------------------------------------- format
def make_format() -> dict:
    out: dict = {}
    out["e2m1_decode"] = f32(decode_e2m1(torch.arange(16, dtype=torch.uint8)))
    out["e2m1_decode_signbit"] = np.signbit(out["e2m1_decode"])
    out["ue4m3_decode"] = f32(decode_ue4m3(torch.arange(0x7F, dtype=torch.uint8)))
    levels = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    probes = [0.0, -0.0, 0.1, 0.25, 0.2500001, 0.75, 0.7499999, 1.25, 1.2500001, 1.75,
              1.7499999, 2.5, 2.5000002, 3.5, 3.4999998, 5.0, 5.0000005, 6.0, 6.5, 100.0,
              1e30, -1e30, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0]
    probes += [(a + b) / 2 for a, b in zip(levels, levels[1:])]
    probes += list(torch.randn(2000, generator=gen(11)).mul(3).tolist())
    p = torch.tensor(probes, dtype=torch.float32)
    out["e2m1_probe"] = f32(p)
    out["e2m1_code"] = encode_e2m1(p).numpy().copy()
    ue = out["ue4m3_decode"].astype(np.float64)
    mids = (ue[1:] + ue[:-1]) / 2
    cands = np.concatenate([ue, mids, [0.0, 1e-9, 448.0, 449.0, 464.0, 1e10, 3.4e38],
                            np.abs(torch.randn(2000, generator=gen(12)).numpy()) * 50]).astype(np.float32)
    out["ue4m3_probe"] = cands
    out["ue4m3_code"] = encode_ue4m3(torch.from_numpy(cands)).numpy().copy()

    def quant_case(name: str, src: torch.Tensor) -> None:
        q = quantize_nvfp4_reference(src)
        if src.dtype == torch.bfloat16:
            out[name + "_src_bf16"] = bits(src)
        else:
            out[name + "_src"] = f32(src)
        q_fields(name + "_", q, out)

    quant_case("q_rand", torch.randn((64, 512), generator=gen(21)) * 0.02)
    quant_case("q_zero", torch.zeros((4, 32)))
    zb = torch.randn((8, 64), generator=gen(22))
    zb[3, 16:32] = 0.0
    quant_case("q_zero_block", zb)
    uf = torch.randn((8, 64), generator=gen(23))
    uf[5, 32:48] = uf[5, 32:48] * 1e-6  # local block-scale underflow
    uf[0, 0] = 3000.0
    quant_case("q_local_underflow", uf)
    quant_case("q_global_tiny", torch.randn((4, 32), generator=gen(24)) * 1e-40)
    quant_case("q_bf16", (torch.randn((16, 64), generator=gen(25)) * 3).to(torch.bfloat16))
    wide = torch.randn((32, 128), generator=gen(26)) * torch.logspace(-8, 8, 128)[None, :]
    quant_case("q_wide", wide)
    return out


# ---------------------------------------------------------------- stages
def make_stages() -> dict:
    out: dict = {}
    # W4A16 projections at several (M, N, K).
    for i, (m, n, k) in enumerate([(1, 96, 3072), (4, 64, 128), (16, 32, 256), (3, 40, 1024)]):
        x = torch.randn((m, k), generator=gen(100 + i)).to(torch.bfloat16)
        q = quantize_nvfp4_reference(torch.randn((n, k), generator=gen(200 + i)) * 0.02)
        y = w4a16_linear_reference(x, q)
        out[f"lin{i}_x"] = bits(x)
        q_fields(f"lin{i}_", q, out)
        out[f"lin{i}_y"] = bits(y)
    # RMSNorm over the reference's test shape matrix.
    for i, shape in enumerate([(1, 1, 4), (2, 3, 64), (1, 1, 3072), (2, 1, 24, 128), (1, 1, 6, 128)]):
        x = (torch.randn(shape, generator=gen(300 + i)) * 0.75).to(torch.bfloat16)
        w = (1 + 0.05 * torch.randn((shape[-1],), generator=gen(400 + i))).to(torch.bfloat16)
        out[f"rms{i}_x"] = bits(x)
        out[f"rms{i}_w"] = bits(w)
        out[f"rms{i}_y"] = bits(rms_norm_reference(x, w, 1e-6))
    # RoPE.
    for i, (shape, p, th) in enumerate([((1, 1, 3, 2), 1, 1e4), ((2, 3, 3, 8), 11, 1e4),
                                        ((1, 4, 24, 128), 2048, 1e4), ((2, 1, 6, 128), 511, 1e4),
                                        ((1, 2, 4, 64), 17, 1e3), ((1, 1, 6, 128), 32767, 1e4)]):
        x = (torch.randn(shape, generator=gen(500 + i)) * 0.75).to(torch.bfloat16)
        out[f"rope{i}_x"] = bits(x)
        out[f"rope{i}_p"] = np.int64(p)
        out[f"rope{i}_theta"] = np.float64(th)
        out[f"rope{i}_y"] = bits(apply_rope_reference(x, p, th))
    # Cached GQA: q [B,T,Hq,D], present = first P+T slots of a [B,Hkv,C,D] cache.
    for i, (b, t, hq, hkv, d, p, c) in enumerate([(1, 1, 4, 1, 8, 5, 8), (1, 1, 24, 6, 128, 511, 512),
                                                  (1, 3, 6, 2, 64, 0, 4), (2, 4, 8, 2, 128, 37, 64),
                                                  (1, 1, 3, 3, 16, 700, 704)]):
        g = gen(600 + i)
        q = torch.randn((b, t, hq, d), generator=g).to(torch.bfloat16)
        kc = torch.randn((b, hkv, c, d), generator=g).to(torch.bfloat16)
        vc = torch.randn((b, hkv, c, d), generator=g).to(torch.bfloat16)
        _, _, ctx = gqa_attention_reference(q, kc[:, :, :p + t].contiguous(),
                                            vc[:, :, :p + t].contiguous(), p, return_attention=False)
        out[f"att{i}_q"] = bits(q)
        out[f"att{i}_k"] = bits(kc)
        out[f"att{i}_v"] = bits(vc)
        out[f"att{i}_p"] = np.int64(p)
        out[f"att{i}_ctx"] = bits(ctx)
    return out


# ---------------------------------------------------------------- forward
FORWARD_CASES = {
    # name: (B, T, H, Hkv, D, P, C, seed)
    "fwd_decode_b2": (2, 1, 512, 2, 128, 37, 64, 31),
    "fwd_multi_token": (1, 5, 256, 1, 128, 7, 16, 32),
    "fwd_p0_chunk": (1, 3, 512, 1, 128, 0, 8, 33),
    "fwd_gqa3": (1, 1, 384, 1, 128, 20, 40, 34),
}


def run_forward(shape: synthetic.DecodeShape, seed: int):
    inp = synthetic.make_decode_inputs(shape, seed)
    qw = {k: quantize_nvfp4_reference(v) for k, v in inp.weights_fp32.items()}
    p = shape.past_lengths[0]
    res = decoder_attention_nvfp4_reference(
        inp.x, inp.input_norm_weight, qw["q"], qw["k"], qw["v"], inp.q_norm_weight,
        inp.k_norm_weight, qw["o"], inp.k_cache[:, :, :p].contiguous(),
        inp.v_cache[:, :, :p].contiguous(), rms_eps=1e-6, rope_theta=1e4, return_debug=True)
    return inp, qw, res


def store_forward(name: str, inp, qw, res, out: dict, with_inputs: bool) -> None:
    dbg = res.debug
    for stage in ("input_normalized", "q_projected", "k_projected", "v_projected",
                  "q_normalized", "k_normalized", "q_rope", "k_rope", "context"):
        out[f"{name}_{stage}"] = bits(getattr(dbg, stage))
    out[f"{name}_output"] = bits(res.output)
    p = inp.shape.past_lengths[0]
    out[f"{name}_new_k"] = bits(res.present_k[:, :, p:].contiguous())
    out[f"{name}_new_v"] = bits(res.present_v[:, :, p:].contiguous())
    for key, q in qw.items():
        if with_inputs:
            q_fields(f"{name}_w{key}_", q, out)
        out[f"{name}_w{key}_sha256"] = sha(q.packed_values.numpy(), q.block_scales.numpy(),
                                           np.float32(q.global_decode_scale.item()))
    if with_inputs:
        out[f"{name}_x"] = bits(inp.x)
        out[f"{name}_g_in"] = bits(inp.input_norm_weight)
        out[f"{name}_g_q"] = bits(inp.q_norm_weight)
        out[f"{name}_g_k"] = bits(inp.k_norm_weight)
        out[f"{name}_k_cache"] = bits(inp.k_cache)
        out[f"{name}_v_cache"] = bits(inp.v_cache)


def make_forward() -> dict:
    out: dict = {}
    for name, (b, t, h, hkv, d, p, c, seed) in FORWARD_CASES.items():
        shape = synthetic.DecodeShape(batch=b, tokens=t, hidden=h, kv_heads=hkv, head_dim=d,
                                      capacity=c, past_lengths=(p,))
        inp, qw, res = run_forward(shape, seed)
        store_forward(name, inp, qw, res, out, with_inputs=True)
        out[f"{name}_shape"] = np.array([b, t, h, hkv, d, p, c, seed], dtype=np.int64)
    return out


def make_canonical() -> dict:
    """configs[0] regenerated from its seed; inputs are not stored (13 MB), only
    the SHA-256 of the reference's quantised weights and the reference outputs."""
    out: dict = {}
    shape = synthetic.CANONICAL
    inp, qw, res = run_forward(shape, seed=0)
    store_forward("c0", inp, qw, res, out, with_inputs=False)
    out["c0_shape"] = np.array([1, 1, 3072, 6, 128, 511, 1024, 0], dtype=np.int64)
    return out


def main() -> None:
    np.savez_compressed(HERE / "format.npz", **make_format())
    np.savez_compressed(HERE / "stages.npz", **make_stages())
    np.savez_compressed(HERE / "forward.npz", **make_forward())
    np.savez_compressed(HERE / "canonical.npz", **make_canonical())
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
