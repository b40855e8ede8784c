"""flashprefill_b200: FlashPrefill's sparse-prefill operator, rebuilt for B200 (sm_100a).

Public entry points keep the reference's signatures (qhfan/FlashPrefill ops/__init__.py):

    from flashprefill_b200 import flash_prefill, flash_prefill_varlen_func

A caller written against the reference's ``ops`` package can call ``install_as_ops()``
once; ``import ops`` then resolves to this package.
"""
from ._lib import FlashPrefillError
from ._ops import check_device_error, get_mean_warps, search_dense, search_varlen, set_mean_warps
from .flashprefill_native_forward import flash_prefill
from .flashprefill_varlen_func import flash_prefill_varlen_func
from . import torch_ops  # registers torch.ops.flashprefill.prefill_dense / prefill_varlen

__all__ = ["flash_prefill", "flash_prefill_varlen_func", "search_dense", "search_varlen", "set_mean_warps",
           "get_mean_warps", "check_device_error", "FlashPrefillError", "install_as_ops"]


def install_as_ops() -> None:
    """Register this package under the reference's import paths ``ops``,
    ``ops.flashprefill_native_forward`` and ``ops.flashprefill_varlen_func`` so that callers
    written against the reference (HF model wrappers, vLLM patches) import it unchanged."""
    import sys
    from . import flashprefill_native_forward, flashprefill_varlen_func
    this = sys.modules[__name__]
    sys.modules["ops"] = this
    sys.modules["ops.flashprefill_native_forward"] = flashprefill_native_forward
    sys.modules["ops.flashprefill_varlen_func"] = flashprefill_varlen_func
