"""CPU oracle for the NVFP4-W4A16 decoder-attention forward.

TEST INFRASTRUCTURE ONLY.  This package is a numpy restatement of the
reference's PyTorch correctness path (``reference/*.py`` of
PatrickZChen/cuda-nvfp4-decoder-attention).  It exists to check the CUDA
kernels: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py`` may import it.  The shipped package never calls it and has no
CPU fallback.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference itself (in
the build container, where its sources are present) and stores its outputs as
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this oracle
against those vectors (bit-exact for the storage format, the quantizer and the
cache append; within one BF16 step for floating-point stages, where torch's
CPU reduction order and SLEEF transcendentals differ from the correctly
rounded sums and trig used here).
"""

from .nvfp4 import (  # noqa: F401
    E2M1_TABLE,
    UE4M3_TABLE,
    NVFP4Storage,
    decode_e2m1,
    decode_ue4m3,
    dequantize,
    encode_e2m1,
    encode_ue4m3,
    global_scales,
    pack_e2m1,
    quantize,
    unpack_e2m1,
)
from .decoder_attention import (  # noqa: F401
    apply_rope,
    bf16_to_f32,
    decoder_attention_nvfp4,
    f32_to_bf16,
    gqa_attention,
    rms_norm,
    rope_cos_sin,
    w4a16_linear,
)
