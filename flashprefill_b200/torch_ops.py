"""The operator as registered PyTorch ops: ``torch.ops.flashprefill.prefill_dense`` and
``torch.ops.flashprefill.prefill_varlen``.

They wrap the same C ABI entry points as ``flash_prefill`` / ``flash_prefill_varlen_func``
(``fpb_prefill_dense`` / ``fpb_prefill_varlen``), each writing its output argument in place.
They are registered with fake (meta) implementations, so ``torch.compile`` and other graph
tracing can follow a model that calls them without a graph break.  The reference calls its
Python functions directly; these ops take the same positional arguments.
"""
from __future__ import annotations

import torch

from . import _ops

_NS = "flashprefill"


@torch.library.custom_op(f"{_NS}::prefill_dense", mutates_args=("out",), device_types="cuda")
def prefill_dense(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, block_size: int,
                  attention_sink: int, window_size: int, alpha: float, last_n_block_full: int,
                  min_budget: int) -> None:
    """flash_prefill (ops/flashprefill_native_forward.py:481-499) as a registered op."""
    _ops.prefill_dense(q, k, v, out, block_size, attention_sink, window_size, alpha, last_n_block_full,
                       min_budget)


@prefill_dense.register_fake
def _(q, k, v, out, block_size, attention_sink, window_size, alpha, last_n_block_full, min_budget):
    return None


@torch.library.custom_op(f"{_NS}::prefill_varlen", mutates_args=("o",), device_types="cuda")
def prefill_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, cu_seqlens: torch.Tensor,
                   max_seq_len: int, alpha: float, block_size: int = 128, attention_sink: int = 2,
                   window_size: int = 4, last_n_block: int = 2) -> None:
    """flash_prefill_varlen_func (ops/flashprefill_varlen_func.py:723-743) as a registered op."""
    _ops.prefill_varlen(q, k, v, o, cu_seqlens, max_seq_len, alpha, block_size, attention_sink, window_size,
                        last_n_block)


@prefill_varlen.register_fake
def _(q, k, v, o, cu_seqlens, max_seq_len, alpha, block_size=128, attention_sink=2, window_size=4,
      last_n_block=2):
    return None
