"""Build the sm_100a attention library ``libffa_sm100.so`` in-tree with nvcc.

The library is one translation unit (``csrc/ffa_capi.cu`` includes every kernel
header) compiled for ``sm_100a`` only.  ``python -m fastflashattention_b200.build``
rebuilds it when a source is newer than the shared object.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_NAME = "libffa_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME
# torch operators (C++ host path and autograd node) over the C ABI, linked to LIB_NAME
TORCH_LIB_PATH = PKG_DIR / "libffa_torch.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the sm_100a library cannot be built")
    return cand


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources)


def needs_build() -> bool:
    return _stale(LIB_PATH, _sources()) or _stale(TORCH_LIB_PATH, [CSRC / "ffa_torch.cpp", LIB_PATH,
                                                                   *INCLUDE.glob("*.h")])


def build_torch_ops(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``libffa_torch.so`` (g++, against torch's headers and libraries) if stale."""
    if not force and not _stale(TORCH_LIB_PATH, [CSRC / "ffa_torch.cpp", LIB_PATH, *INCLUDE.glob("*.h")]):
        return TORCH_LIB_PATH
    import torch
    from torch.utils import cpp_extension as ce
    cuda_home = Path(ce.CUDA_HOME or "/usr/local/cuda")
    inc = [*ce.include_paths(), str(cuda_home / "include")]
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_LIB_PATH.with_suffix(".so.tmp")
    cmd = [shutil.which("g++") or "g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", *(f"-I{p}" for p in inc), str(CSRC / "ffa_torch.cpp"),
           f"-L{torch_lib}", f"-L{PKG_DIR}", "-lffa_sm100", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10",
           "-lc10_cuda", f"-Wl,-rpath,$ORIGIN:{torch_lib}", "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed ({res.returncode}):\n{res.stderr[-4000:]}")
    os.replace(tmp, TORCH_LIB_PATH)
    return TORCH_LIB_PATH


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``libffa_sm100.so`` (sm_100a) and the torch operators over it
    (``libffa_torch.so``) if missing or stale; return the kernel library's path."""
    if not force and not _stale(LIB_PATH, _sources()):
        build_torch_ops(force, verbose)
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, str(CSRC / "ffa_capi.cu"), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-4000:]}")
    if verbose:
        print(res.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    build_torch_ops(True, verbose)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
