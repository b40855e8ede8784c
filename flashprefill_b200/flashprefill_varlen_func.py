"""Packed (varlen) entry point with the reference's signature.

Drop-in for ``ops.flashprefill_varlen_func.flash_prefill_varlen_func``
(qhfan/FlashPrefill ops/flashprefill_varlen_func.py:722-743), called positionally with 11
arguments by the vLLM 0.10 / 0.12 patches (patches/patch_loader_vllm_0_10_0.py:246-258,
patches/patch_loader_vllm_0_12_0.py:187-199).  q: (T, Hq, 128), k/v: (T, Hk, 128), o like q
(written in place), cu_seqlens: int32 CUDA tensor [nseq+1].  No host synchronisation:
cu_seqlens is validated on the device, and every temporary is sized from max_seq_len.
"""
from __future__ import annotations

import torch

from . import _ops


@torch.no_grad()
def flash_prefill_varlen_func(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    o: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seq_len: int,
    alpha: float,
    block_size: int = 128,
    attention_sink: int = 2,
    window_size: int = 4,
    last_n_block: int = 2,
):
    """Block-sparse causal GQA prefill over packed sequences; writes ``o`` in place."""
    _ops.prefill_varlen(q, k, v, o, cu_seqlens, max_seq_len, alpha, block_size, attention_sink, window_size,
                        last_n_block)
