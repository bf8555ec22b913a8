"""CPU: the C-ABI library loads and exports every symbol include/ffa.h declares, and its
argument validation answers before touching the GPU."""
import ctypes
import re
from pathlib import Path

import pytest

from fastflashattention_b200 import _lib
from fastflashattention_b200.build import LIB_PATH

HEADER = Path(__file__).resolve().parents[1] / "include" / "ffa.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ffa_[a-z0-9_]+)\s*\(", text)))


def test_library_built_in_tree():
    assert LIB_PATH.exists(), "run python -m fastflashattention_b200.build"
    assert LIB_PATH.parent.name == "fastflashattention_b200"


def test_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(LIB_PATH))
    syms = declared_symbols()
    assert len(syms) >= 7
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signatures out of sync with include/ffa.h"


def test_version():
    assert _lib.load().ffa_version().decode().endswith("sm100a")


@pytest.mark.parametrize("D", [32, 96, 256])
def test_unsupported_head_dim_rejected_before_launch(D):
    lib = _lib.load()
    rc = lib.ffa_fwd(16, 16, 16, 16, None, 1, 128, D, 128 * D, D, 0.1, 1, None)
    assert rc == _lib.FFA_ERR_UNSUPPORTED
    assert "head_dim" in _lib.last_error()


def test_invalid_arguments_rejected_before_launch():
    lib = _lib.load()
    assert lib.ffa_fwd(16, 16, 16, 16, None, -1, 128, 64, 8192, 64, 0.1, 1, None) == _lib.FFA_ERR_INVALID
    assert lib.ffa_fwd(16, 16, 16, 16, None, 2, 128, 64, 100, 64, 0.1, 1, None) == _lib.FFA_ERR_INVALID
    assert lib.ffa_fwd(None, 16, 16, 16, None, 1, 128, 64, 8192, 64, 0.1, 1, None) == _lib.FFA_ERR_INVALID
    assert lib.ffa_fwd(18, 16, 16, 16, None, 1, 128, 64, 8192, 64, 0.1, 1, None) == _lib.FFA_ERR_INVALID
    assert lib.ffa_bwd(16, 16, 16, 16, 16, 16, 16, 16, 16, 16, 1, 64, 48, 64 * 48, 48, 0.1, 0, None) \
        == _lib.FFA_ERR_UNSUPPORTED
    assert lib.ffa_lse_merge(16, 16, 16, 16, 4, 130, 0, None) == _lib.FFA_ERR_INVALID
    # one CTA per 128-row block of every slice in a 1-D grid: at most 2^31-1 CTAs
    assert lib.ffa_fwd(16, 16, 16, 16, None, 1 << 30, 1024, 64, 1024 * 64, 64, 0.1, 1, None) \
        == _lib.FFA_ERR_UNSUPPORTED
    assert "grid" in _lib.last_error()


def test_empty_problems_are_noops():
    lib = _lib.load()
    assert lib.ffa_fwd(16, 16, 16, 16, None, 0, 128, 64, 8192, 64, 0.1, 1, None) == _lib.FFA_OK
    assert lib.ffa_fwd(16, 16, 16, 16, None, 4, 0, 128, 0, 128, 0.1, 0, None) == _lib.FFA_OK
    assert lib.ffa_lse_merge(16, 16, 16, 16, 0, 128, 1, None) == _lib.FFA_OK


def test_torch_operators_load_and_register():
    """The C++ host path (libffa_torch.so) loads on a machine without a GPU and registers
    every operator the Python layer calls."""
    from fastflashattention_b200.build import TORCH_LIB_PATH
    assert TORCH_LIB_PATH.exists() and TORCH_LIB_PATH.parent.name == "fastflashattention_b200"
    ops = _lib.ops()
    for name in ("forward", "forward_lse", "backward", "attention"):
        assert hasattr(ops, name), name
