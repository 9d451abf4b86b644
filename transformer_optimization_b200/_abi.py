"""ctypes binding of the C ABI in include/tfb200.h (libtfb200.so).

This is the only door to the CUDA kernels. There is no CPU fallback: if the
library is missing or the device is not a B200 (sm_100), every call raises.
The library is loaded from this package directory (built in-tree by
`python -m transformer_optimization_b200.build` or `__graft_entry__.build()`).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

LIB_PATH = Path(__file__).resolve().parent / "libtfb200.so"

# status codes and flags (include/tfb200.h)
TF_OK = 0
TF_ERR_SHAPE = 1
TF_ERR_ALIGN = 2
TF_ERR_LAUNCH = 3
TF_ERR_UNSUPPORTED = 4
TF_ERR_DEVICE = 5
TF_ERR_DRIVER = 6
TF_ERR_TIMEOUT = 7

TF_LN_MASK_DELTA = 1
TF_LN_MASK_X = 2
TF_LN_MASK_OUT = 4
TF_LN_WRITE_X = 8
TF_LN_OUT_F32 = 16
TF_LN_X_F16 = 32
TF_LN_X_BF16 = 64

TF_EPI_BIAS = 0
TF_EPI_BIAS_GELU = 1
TF_EPI_BIAS_GELU_ROUNDED = 2
TF_EPI_W_SPLIT = 16
TF_EPI_BF16 = 32

TF_RES_NO_MASK = 0
TF_RES_MASK_DELTA = 1
TF_RES_MASK_X = 2
TF_RES_X16 = 4
TF_RES_BF16 = 8

TF_ATTN_CAUSAL = 1
TF_ATTN_OUT_F32 = 2
TF_ATTN_EXP_F16X2 = 4
TF_ATTN_BF16 = 8
TF_ATTN_ROUND_SCORES = 16

# every symbol include/tfb200.h declares, with its ctypes signature
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
SIGNATURES = {
    "tf_abi_version": ([], _I),
    "tf_last_error": ([], ctypes.c_char_p),
    "tf_device_status": ([ctypes.POINTER(_I), _P], _I),
    "tf_test_wait_timeout": ([_P, _I64, _P, _P], _I),
    "tf_ln_residual": ([_P, _P, _P, _P, _F, _P, _I64, _I64, _I, _P, _P, _P], _I),
    "tf_gemm": ([_P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I, _P], _I),
    "tf_gemm_tiled": ([_P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _I, _P], _I),
    "tf_gemm_residual": ([_P, _I64, _P, _I64, _P, _P, _P, _I64, _P, _I, _I64, _I64, _I64, _I, _I, _I, _P], _I),
    "tf_gemm_residual_ready": ([_P, _I64, _P, _I64, _P, _P, _P, _I64, _P, _I, _I64, _I64, _I64, _I, _P, _P], _I),
    "tf_ln_ready": ([_P, _P, _P, _F, _P, _I64, _I64, _I, _P, _P, _P], _I),
    "tf_flash_fwd": ([_P, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _P,
                      _I64, _I64, _I64, _I64, _I64, _F, _I64, _I64, _I, _P], _I),
    "tf_attn_merge": ([_P, _P, _P, _P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P], _I),
    "tf_gemm_splitk_workspace": ([_I64, _I64, _I64, _I], _I64),
    "tf_gemm_splitk": ([_P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _P, _I64, _P], _I),
    "tf_gemm_residual_splitk": ([_P, _I64, _P, _I64, _P, _P, _P, _I64, _P, _I, _I64, _I64, _I64, _I, _P, _I64, _P],
                                _I),
    "tf_gemm_splitk_static": ([_P, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _P], _I),
    "tf_gemm_residual_ln_splitk": ([_P, _I64, _P, _I64, _P, _P, _P, _I64, _P, _I, _I64, _I64, _I64, _I, _P, _I64,
                                    _P, _P, _F, _P, _I, _P], _I),
}

_lib: Optional[ctypes.CDLL] = None


class TfError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def load(path: Optional[os.PathLike] = None) -> ctypes.CDLL:
    """Load (once) and return the library with every signature declared."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"CUDA library {p} is missing: build it with `python -m transformer_optimization_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if path is None:
        _lib = lib
    return lib


def check(fn: str, rc: int) -> None:
    if rc != TF_OK:
        msg = load().tf_last_error()
        raise TfError(fn, rc, msg.decode() if msg else "")


def call(fn: str, *args) -> None:
    """Call an ABI function and raise TfError on a non-zero status."""
    check(fn, getattr(load(), fn)(*args))


def call_value(fn: str, *args) -> int:
    """Call an ABI function that returns a value (negative = error)."""
    v = getattr(load(), fn)(*args)
    if v < 0:
        raise TfError(fn, -1, load().tf_last_error().decode())
    return v


def device_status(stream: int = 0) -> int:
    """Synchronise `stream`, return and clear the device status word
    (0 = no kernel wait ran out)."""
    code = ctypes.c_int(0)
    rc = load().tf_device_status(ctypes.byref(code), ctypes.c_void_p(stream))
    if rc not in (TF_OK, TF_ERR_TIMEOUT):
        check("tf_device_status", rc)
    return code.value
