"""Dense entry point with the reference's signature.

Drop-in for ``ops.flashprefill_native_forward.flash_prefill``
(qhfan/FlashPrefill ops/flashprefill_native_forward.py:480-499): same positional
arguments, same meaning, ``out`` written in place, returns None, runs under no_grad.
q: (B, S, Hq, 128), k/v: (B, S, Hk, 128), bfloat16 or float16 CUDA tensors, any strides
(copied only when the last dimension is not contiguous or a stride is not a multiple of
8 elements -- the reference always copies via its ``@contiguous`` decorator).
"""
from __future__ import annotations

import torch

from . import _ops


@torch.no_grad()
def flash_prefill(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    out: torch.Tensor,
    block_size: int,
    attention_sink: int,
    window_size: int,
    alpha: float,
    last_n_block_full: int,
    min_budget: int,
):
    """Block-sparse causal GQA prefill attention (search + sparse attention).

    block_size must be 128 (the reference asserts block_size == k_stride and uses it for
    both; its model code always passes 128).  The softmax scale is 1/sqrt(head_dim), as in
    the reference.  k/v may be longer than q (chunked prefill over a cached prefix): the
    queries are then the last q.shape[1] positions of the k/v sequence, selected with the
    whole sequence's block structure (the reference sends that case to dense attention).  Raises ValueError/TypeError for unsupported shapes or dtypes and
    flashprefill_b200.FlashPrefillError for CUDA failures.
    """
    _ops.prefill_dense(q, k, v, out, block_size, attention_sink, window_size, alpha, last_n_block_full,
                       min_budget)
