"""ctypes binding of libflashprefill_b200.so (the C ABI in include/flashprefill_b200.h).

The shared library is built in-tree by ``flashprefill_b200.build``.  There is no CPU or
Triton fallback: if the library cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# FLASHPREFILL_B200_LIB selects another build of the same library (e.g. an instrumented one)
LIB_PATH = os.environ.get("FLASHPREFILL_B200_LIB") or os.path.join(_HERE, "libflashprefill_b200.so")

FPB_OK, FPB_EINVAL, FPB_ECUDA, FPB_EDEVICE = 0, 1, 2, 3
FPB_BF16, FPB_FP16 = 0, 1

DEV_ERROR_BITS = {
    1: "pipeline wait timed out",
    2: "cu_seqlens not non-decreasing from 0 to total_tokens",
    4: "a sequence is longer than max_seq_len",
    8: "a block list held an index outside [0, query block]",
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_I64P = ctypes.POINTER(ctypes.c_int64)
_U32P = ctypes.POINTER(ctypes.c_uint32)

# Exported symbols and their signatures (restype, argtypes).
SIGNATURES = {
    "fpb_version": (_I, []),
    "fpb_last_error": (ctypes.c_char_p, []),
    "fpb_dense_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "fpb_varlen_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "fpb_workspace_layout": (_I, [_I, _I, _I, _I, _I, _I, _I, _I64P]),
    "fpb_prefill_dense": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I64P, _I64P,
                               _I, _I, _I, _F, _I, _I, _I, _P, _SZ, _P]),
    "fpb_prefill_dense_peers": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I64P, _I64P,
                                     _I, _I, _I, _F, _I, _I, _I, _P, _SZ, ctypes.POINTER(_P), _I, _P]),
    "fpb_prefill_dense_rows": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I64P, _I64P,
                                    _I, _I, _I, _F, _I, _I, _I, _I, _I, _P, _SZ, _P]),
    "fpb_prefill_dense_chunk": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I64P, _I64P,
                                     _I, _I, _I, _F, _I, _I, _I, _P, _SZ, _P]),
    "fpb_prefill_varlen": (_I, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I64P, _I64P,
                                _I, _I, _I, _F, _I, _I, _P, _SZ, _P]),
    "fpb_search_dense": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I, _I, _I, _F, _I, _I, _I,
                              _P, _SZ, _P]),
    "fpb_search_varlen": (_I, [_P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I, _I, _I, _F, _I, _I,
                               _P, _SZ, _P]),
    "fpb_attention_dense": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I64P, _I64P, _I,
                                 _P, _SZ, _P]),
    "fpb_attention_varlen": (_I, [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I64P, _I64P,
                                  _I, _P, _SZ, _P]),
    "fpb_read_device_error": (_I, [_P, _U32P, _P]),
    "fpb_noalloc_read_device_error": (_I, [_U32P, _P]),
    "fpb_test_set_fault": (_I, [_I, ctypes.c_ulonglong]),
    "fpb_prefill_dense_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I64P, _I64P, _I64P, _I64P,
                                       _I, _I, _I, _F, _I, _I, _I, _P]),
}

_lock = threading.Lock()
_lib = None


class FlashPrefillError(RuntimeError):
    """A CUDA or device-side failure reported by the library."""


def load(path: str = LIB_PATH):
    """Load the library (once) and declare the signatures of every exported symbol."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise ImportError(
                    f"flashprefill_b200: CUDA library not built ({path} missing); run "
                    "`python -m flashprefill_b200.build` (needs nvcc with sm_100a support)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def i64arr(vals):
    return (ctypes.c_int64 * len(vals))(*[int(x) for x in vals])


def check(rc: int) -> None:
    """Raise on a non-zero return code, with the library's message."""
    if rc == FPB_OK:
        return
    msg = load().fpb_last_error().decode(errors="replace")
    if rc == FPB_EINVAL:
        raise ValueError(f"flashprefill_b200: {msg}")
    raise FlashPrefillError(f"flashprefill_b200: {msg}")
