"""ctypes binding of the C ABI in ``include/lthc_b200.h``.

This is the same stub a Python user of the reference would add to call the
library.  Loading fails loudly: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("liblthc_b200.so")

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

STATUS_NAMES = {
    0: "LTHC_OK",
    1: "LTHC_ERR_NULL_POINTER",
    2: "LTHC_ERR_SHAPE",
    3: "LTHC_ERR_DTYPE",
    4: "LTHC_ERR_ALIGNMENT",
    5: "LTHC_ERR_WORKSPACE",
    6: "LTHC_ERR_LAUNCH",
    7: "LTHC_ERR_DEVICE",
    8: "LTHC_ERR_TIMEOUT",
}

_P = c_void_p
_PP = POINTER(c_void_p)
_I = c_int
_L = c_int64

# name -> (restype, argtypes); must match include/lthc_b200.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "lthc_version": (_I, []),
    "lthc_status_string": (c_char_p, [_I]),
    "lthc_last_error_message": (c_char_p, []),
    "lthc_device_status": (_I, [POINTER(c_int), _P]),
    "lthc_selftest_wait_timeout": (_I, [_I, _P, _P]),
    "lthc_write_fwd": (_I, [_P, _P, _I, _P, _L, _L, _L, _I, _P]),
    "lthc_write_add_fwd": (_I, [_P, _P, _P, _I, _P, _L, _L, _L, _I, _P]),
    "lthc_materialise_fwd": (_I, [_P, _PP, _PP, _I, _I, _P, _L, _L, _L, _I, _P]),
    "lthc_materialise12_fwd": (_I, [_P, _PP, _PP, _I, _P, _L, _L, _L, _I, _P]),
    "lthc_materialise_bwd_workspace_bytes": (c_size_t, [_L, _L, _L, _I]),
    "lthc_materialise_bwd": (_I, [_P, _PP, _PP, _I, _I, _PP, _P, _P, c_size_t, _L, _L, _L, _I, _P]),
    "lthc_materialise_bwd_uses_tensor_cores": (_I, [_L, _L, _L, _I, _I]),
    "lthc_write_bwd_workspace_bytes": (c_size_t, [_L, _L, _L]),
    "lthc_write_bwd": (_I, [_P, _P, _P, _I, _P, _P, _P, c_size_t, _L, _L, _L, _I, _P]),
    "lthc_read_fwd": (_I, [_P, _P, _I, _P, _L, _L, _L, _I, _P]),
    "lthc_weight_grad_workspace_bytes": (c_size_t, [_L, _L, _L, _I]),
    "lthc_weight_grad": (_I, [_P, _PP, _I, _P, _P, c_size_t, _L, _L, _L, _I, _P]),
    "lthc_weight_grad_noalloc": (_I, [_P, _PP, _I, _P, _L, _L, _L, _I, _P]),
    "lthc_read_bwd_workspace_bytes": (c_size_t, [_L, _L, _L]),
    "lthc_read_bwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, c_size_t, _L, _L, _L, _I, _P]),
    "lthc_lazy_update_fwd": (_I, [_P, _P, _P, _I, _P, _I, _P, _L, _L, _I, _P]),
    "lthc_lazy_update_bwd_workspace_bytes": (c_size_t, [_L, _L]),
    "lthc_lazy_update_bwd": (_I, [_P, _P, _P, _I, _P, _I, _P, _P, _P, _P, c_size_t, _L, _L, _I, _P]),
    "lthc_selftest_umma": (_I, [_P, _P, _P, _I, _I, _P, _P]),
    "lthc_selftest_umma_desc": (_I, [_P, _I, _P, _I, _P, _P, _I, c_uint32, _I, _P, _P, _P]),
    "lthc_branch_lazy_fwd": (_I, [_P, _P, _P, _P, _L, _P, _I, _P, _I, _P, _P, _L, _L, _L, _I, _P]),
    "lthc_branch_lazy_bwd_workspace_bytes": (c_size_t, [_L, _L, _L]),
    "lthc_branch_lazy_bwd": (_I, [_P, _P, _P, _P, _P, _L, _P, _I, _P, _I, _P, _P, _P, _P, _P, _P, c_size_t, _L, _L,
                                  _L, _I, _P]),
    "lthc_patch_embed_read_fwd": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _L, _I, _L, _L, _P]),
    "lthc_final_norm_modulate_fwd": (_I, [_P, _P, _I, _P, _P, _L, _P, _L, _L, _L, c_float, _I, _P]),
    "lthc_final_norm_modulate_bwd_workspace_bytes": (c_size_t, [_L, _L, _L]),
    "lthc_final_norm_modulate_bwd": (_I, [_P, _P, _I, _P, _L, _P, _P, _P, _P, _P, _P, c_size_t, _L, _L, _L,
                                          c_float, _I, _P]),
}

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


class LthcError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        self.func = func
        super().__init__(f"{func}: {STATUS_NAMES.get(status, status)}: {message}")


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load the library (once).  Raises ImportError if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise ImportError(
                f"LTHC CUDA library not found at {p}; build it with "
                "`python -m flowmatching_lthc_b200.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(status: int, func: str) -> None:
    if status != 0:
        msg = load().lthc_last_error_message().decode(errors="replace")
        raise LthcError(status, func, msg)


_fns: dict = {}


def call(func: str, *args) -> None:
    """Call an int-returning entry point and raise LthcError on failure."""
    fn = _fns.get(func)
    if fn is None or _lib is None:
        fn = _fns[func] = getattr(load(), func)
    st = fn(*args)
    if st != 0:
        check(st, func)


def ptr_array(ptrs) -> ctypes.Array:
    return (c_void_p * len(ptrs))(*ptrs)
