"""ctypes binding of the C ABI in ``include/ffa.h`` (``libffa_sm100.so``).

The shared object is built in-tree for sm_100a by ``fastflashattention_b200.build``.
There is no fallback: if the library is missing or cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .build import LIB_PATH, TORCH_LIB_PATH

FFA_OK = 0
FFA_ERR_INVALID = 1
FFA_ERR_UNSUPPORTED = 2
FFA_ERR_LAUNCH = 3
FFA_ERR_DEVICE = 4

# Every symbol ``include/ffa.h`` declares, with (restype, argtypes).
_VP = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_D = ctypes.c_double
_FP = ctypes.POINTER(ctypes.c_float)
SIGNATURES = {
    "ffa_fwd": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _LL, _LL, _D, _I, _VP]),
    "ffa_fwd_merge": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _LL, _LL, _D, _I, _I, _VP]),
    "ffa_bwd_preprocess": (_I, [_VP, _VP, _VP, _I, _I, _I, _LL, _LL, _VP]),
    "ffa_bwd": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _LL, _LL, _D, _I, _VP]),
    "ffa_bwd_noalloc": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _LL, _LL, _D, _I, _VP]),
    "ffa_bwd_dkdv": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _LL, _LL, _D, _I, _VP]),
    "ffa_bwd_dq": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _LL, _LL, _D, _I, _VP]),
    "ffa_bwd_dkdv_acc": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _LL, _LL, _D, _I, _VP]),
    "ffa_bwd_dq_acc": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _LL, _LL, _D, _I, _VP]),
    "ffa_lse_merge": (_I, [_VP, _VP, _VP, _VP, _LL, _I, _I, _VP]),
    "ffa_last_error": (_I, [ctypes.c_char_p, _I]),
    "ffa_device_status": (_I, [ctypes.POINTER(ctypes.c_uint)]),
    "ffa_version": (ctypes.c_char_p, []),
}

_lock = threading.Lock()
_lib = None


class FFAError(RuntimeError):
    """A C-ABI call returned a nonzero status."""

    def __init__(self, code: int, fn: str, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library; raises if it does not exist."""
    global _lib
    if path is None and _lib is not None:  # loaded: no lock needed
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise ImportError(
                f"{p.name} is not built; run `python -m fastflashattention_b200.build` "
                "(nvcc, sm_100a) — there is no CPU or eager fallback")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


_ops_loaded = False
_ops_lock = threading.Lock()


def ops():
    """The torch operators of ``libffa_torch.so`` (``torch.ops.ffa_b200``), loaded once.

    They are the C++ host path (tensor preparation, launch on the current stream and the
    autograd node) over the same C ABI; raises if the library is not built."""
    global _ops_loaded
    import torch
    if not _ops_loaded:
        load()  # the kernel library first (outside _ops_lock), so both bindings share one copy
        with _ops_lock:
            if not _ops_loaded:
                if not TORCH_LIB_PATH.exists():
                    raise ImportError(f"{TORCH_LIB_PATH.name} is not built; run `python -m fastflashattention_b200.build`")
                torch.ops.load_library(str(TORCH_LIB_PATH))
                _ops_loaded = True
    return torch.ops.ffa_b200


def last_error() -> str:
    buf = ctypes.create_string_buffer(256)
    load().ffa_last_error(buf, 256)
    return buf.value.decode(errors="replace")


def check(rc: int, fn: str) -> None:
    if rc != FFA_OK:
        raise FFAError(rc, fn, last_error())


def device_status() -> tuple[int, int, int, int]:
    """Read and clear the device-side timeout record (synchronises the device)."""
    out = (ctypes.c_uint * 4)()
    rc = load().ffa_device_status(out)
    vals = tuple(int(x) for x in out)
    if rc not in (FFA_OK, FFA_ERR_DEVICE):
        check(rc, "ffa_device_status")
    return vals
