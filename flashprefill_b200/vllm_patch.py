"""vLLM attention-backend shim: prefill batches through ``flash_prefill_varlen_func``.

The reference ships one loader per vLLM version that replaces
``FlashAttentionImpl.forward`` of vLLM's FlashAttention backend with a copy of it whose
prefill branch calls ``flash_prefill_varlen_func`` (patches/patch_loader_vllm_0_12_0.py:47-253,
patches/patch_loader_vllm_0_10_0.py).  Those loaders import modules the installed vLLM
(0.22) no longer has.  In vLLM 0.22 the KV-cache write has moved out of ``forward`` into
``do_kv_cache_update``, so this shim wraps the original method instead of copying it:

* a batch goes to the sparse prefill when it is decoder self-attention on the non-cascade,
  single-DCP path, with no sliding window, ALiBi, soft cap or attention sinks, head size
  128, the default scale 1/sqrt(head_size) (the operator always uses it, as the reference's
  does), 16-bit inputs, and every sequence of the batch is a whole new prefill (its query
  length equals its KV length);
* every other batch (decode steps, cached prefixes, mixed prefill/decode batches, profiling
  runs with no metadata) runs the original ``forward`` unchanged.

The last condition is decided on the host, without a device sync: the patch also wraps
``FlashAttentionMetadataBuilder.build``, which vLLM calls once per batch with the
scheduler's host-side copies of the query start offsets (``query_start_loc_cpu``) and
sequence lengths (``seq_lens_cpu_upper_bound``, exact for prefill rows and never below the
real length); it stores the verdict on the metadata it returns (``fp_whole_prefill``).
A query length equal to the upper bound of its sequence length means the sequence has no
cached prefix.  Metadata without that verdict, and batches traced during CUDA-graph
capture, run vLLM's own ``forward``.  The reference instead takes any batch with
``max_query_len > 1`` as a prefill (patch_loader_vllm_0_12_0.py:167-168), which computes
wrong attention for the decode tokens and cached prefixes such a batch can hold.

Usage, in every worker process before the model runs::

    from flashprefill_b200.vllm_patch import apply_patch_to_worker
    apply_patch_to_worker(config="flashprefill_llama")
"""
from __future__ import annotations

import math

# Selection parameters per model family, as the reference's loader defines them
# (patch_loader_vllm_0_12_0.py:13-42).
ATTENTION_CONFIGS = {
    "flashprefill_llama": {"block_size": 128, "attention_sink": 2, "window_size": 4, "alpha": 0.18,
                           "last_n_full_block": 2},
    "flashprefill_qwen2": {"block_size": 128, "attention_sink": 2, "window_size": 4, "alpha": 0.08,
                           "last_n_full_block": 2},
    "flashprefill_qwen3moe": {"block_size": 128, "attention_sink": 2, "window_size": 4, "alpha": 0.12,
                              "last_n_full_block": 2},
}

_state = {"original": None, "original_build": None, "cfg": None, "calls": 0, "fallbacks": 0}


def _backend():
    import vllm.v1.attention.backends.flash_attn as fa
    return fa


def _static_ok(impl, query, output_scale, output_block_scale) -> bool:
    """Conditions that need no device data."""
    import torch
    fa = _backend()
    if output_scale is not None or output_block_scale is not None:
        return False
    if impl.attn_type != fa.AttentionType.DECODER:
        return False
    if getattr(impl, "dcp_world_size", 1) > 1 or getattr(impl, "kv_sharing_target_layer_name", None) is not None:
        return False
    sw = getattr(impl, "sliding_window", None)
    if sw is not None and tuple(sw) != (-1, -1):
        return False
    if getattr(impl, "alibi_slopes", None) is not None or getattr(impl, "sinks", None) is not None:
        return False
    if getattr(impl, "logits_soft_cap", None) not in (None, 0, 0.0):
        return False
    if impl.head_size != 128 or abs(impl.scale - 1.0 / math.sqrt(impl.head_size)) > 1e-6 / math.sqrt(impl.head_size):
        return False
    return query.dtype in (torch.bfloat16, torch.float16)


def whole_prefill_from_host(common) -> bool | None:
    """Host-side verdict for one batch (CommonAttentionMetadata): True when every sequence is a
    new prefill (query length == sequence length), None when the host copies are missing."""
    qsl = getattr(common, "query_start_loc_cpu", None)
    sl = getattr(common, "seq_lens_cpu_upper_bound", None)
    if sl is None:
        sl = getattr(common, "_seq_lens_cpu", None)
    if qsl is None or sl is None:
        return None
    n = int(common.num_reqs)
    if n < 1 or int(common.max_query_len) <= 1:
        return False
    q_lens = qsl[1:n + 1] - qsl[:n]
    return bool((q_lens.to(sl.dtype) == sl[:n]).all())


def _whole_prefills(attn_metadata) -> bool:
    """True when every sequence of the batch is a new prefill: query length == KV length.
    Uses only host data (the verdict the wrapped metadata builder attached)."""
    import torch
    if attn_metadata.use_cascade or attn_metadata.max_query_len <= 1:
        return False
    if attn_metadata.max_seq_len != attn_metadata.max_query_len:
        return False  # some sequence has KV beyond its queries
    if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
        return False  # a captured graph would freeze this batch's routing
    return getattr(attn_metadata, "fp_whole_prefill", None) is True


def _build(self, common_prefix_len, common_attn_metadata, *args, **kwargs):
    md = _state["original_build"](self, common_prefix_len, common_attn_metadata, *args, **kwargs)
    try:
        md.fp_whole_prefill = whole_prefill_from_host(common_attn_metadata)
    except Exception:  # metadata of an unexpected shape: leave the verdict unset (fallback)
        pass
    return md


def _prefill(query, key, value, output, attn_metadata, cfg) -> None:
    from .flashprefill_varlen_func import flash_prefill_varlen_func
    n = attn_metadata.num_actual_tokens
    flash_prefill_varlen_func(query[:n], key[:n], value[:n], output[:n], attn_metadata.query_start_loc,
                              attn_metadata.max_query_len, cfg["alpha"], cfg["block_size"],
                              cfg["attention_sink"], cfg["window_size"], cfg["last_n_full_block"])


def _forward(self, layer, query, key, value, kv_cache, attn_metadata, output=None, output_scale=None,
             output_block_scale=None):
    cfg = _state["cfg"]
    if (attn_metadata is not None and output is not None and key is not None and value is not None
            and _static_ok(self, query, output_scale, output_block_scale) and _whole_prefills(attn_metadata)):
        _state["calls"] += 1
        # FlashAttentionImpl.forward writes into output[:num_actual_tokens] viewed as
        # [tokens, heads, head_size]; the operator takes the same layout.
        out3 = output.view(output.shape[0], -1, self.head_size) if output.dim() == 2 else output
        _prefill(query, key, value, out3, attn_metadata, cfg)
        return output
    _state["fallbacks"] += 1
    return _state["original"](self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                              output_block_scale)


def apply_patch_to_worker(worker=None, config: str | dict = "flashprefill_llama") -> None:
    """Route eligible prefill batches of vLLM's FlashAttention backend through the sparse
    prefill (reference: patch_loader_vllm_0_12_0.py:47-253, same function name).  ``config``
    names an entry of ATTENTION_CONFIGS or gives the parameters directly.  Idempotent."""
    cfg = dict(ATTENTION_CONFIGS[config]) if isinstance(config, str) else dict(config)
    if cfg.get("block_size", 128) != 128:
        raise ValueError("block_size must be 128")
    fa = _backend()
    if _state["original"] is None:
        _state["original"] = fa.FlashAttentionImpl.forward
        _state["original_build"] = fa.FlashAttentionMetadataBuilder.build
    _state["cfg"] = cfg
    fa.FlashAttentionImpl.forward = _forward
    fa.FlashAttentionMetadataBuilder.build = _build


def remove_patch() -> None:
    """Restore vLLM's own FlashAttentionImpl.forward."""
    if _state["original"] is not None:
        _backend().FlashAttentionImpl.forward = _state["original"]
        _backend().FlashAttentionMetadataBuilder.build = _state["original_build"]
        _state["original"] = None
        _state["original_build"] = None
        _state["cfg"] = None


def stats() -> dict:
    """Batches routed to the sparse prefill and to vLLM's own forward since the patch."""
    return {"sparse_prefill": _state["calls"], "fallback": _state["fallbacks"]}
