"""Build the in-tree shared libraries for sm_100a.

* ``lib/libnvfp4da.so``    — the CUDA kernels behind the C ABI
  (``include/nvfp4_decoder_attention.h``), nvcc, static CUDA runtime.
* ``lib/cuda_primitives.so`` — the PyTorch operator library (namespace
  ``cuda_nvfp4_decoder_attention``) linked against ``libnvfp4da.so``.

Run ``python cuda-nvfp4-decoder-attention_b200/build.py`` (add ``--force`` to
rebuild).  nvcc cross-compiles without a GPU.  The built files stay in the
tree so that they travel with it; nothing is installed into site-packages.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
INCLUDE = PKG.parent / "include"
CAPI_SO = LIB / "libnvfp4da.so"
OPS_SO = LIB / "cuda_primitives.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    exe = Path(cuda) / "bin" / "nvcc"
    return str(exe) if exe.exists() else (shutil.which("nvcc") or "nvcc")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_capi(force: bool = False, verbose_ptxas: bool = False) -> Path:
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "nvfp4_decoder_attention.h"]
    if not force and not _stale(CAPI_SO, sources):
        return CAPI_SO
    LIB.mkdir(exist_ok=True)
    cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-cudart", "static", "-o", str(CAPI_SO), str(CSRC / "capi.cu"), str(CSRC / "noalloc.cu")]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd)
    return CAPI_SO


def build_torch_ops(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    sources = [CSRC / "torch_ops.cpp", INCLUDE / "nvfp4_decoder_attention.h", CAPI_SO]
    if not force and not _stale(OPS_SO, sources):
        return OPS_SO
    LIB.mkdir(exist_ok=True)
    includes = cpp_extension.include_paths(device_type="cuda") if "device_type" in \
        cpp_extension.include_paths.__code__.co_varnames else cpp_extension.include_paths(cuda=True)
    cuda_inc = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in includes], f"-I{cuda_inc}", f"-I{sysconfig.get_paths()['include']}",
           str(CSRC / "torch_ops.cpp"), "-o", str(OPS_SO),
           f"-L{LIB}", "-lnvfp4da", f"-L{torch_lib}", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10",
           "-lc10_cuda", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    _run(cmd)
    return OPS_SO


def build_all(force: bool = False) -> tuple[Path, Path]:
    return build_capi(force), build_torch_ops(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
