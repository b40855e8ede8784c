"""Tensor plumbing between PyTorch and the C ABI: validation, layout, workspace, stream.

PyTorch only provides device memory (the workspace comes from its caching allocator, as
the reference's temporaries do) and the current CUDA stream; all computation happens in
the CUDA kernels of libflashprefill_b200.so.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.FPB_BF16, torch.float16: _lib.FPB_FP16}

# Reduction order of the pooled-key sum: the Triton warp count whose order is reproduced
# (the reference's autotuner picks 4 or 8, ops/flashprefill_native_forward.py:7-20).
_MEAN_WARPS = int(os.environ.get("FLASHPREFILL_B200_MEAN_WARPS", "4"))
# When set, every call synchronises and raises if a kernel reported a device error.
_CHECK = os.environ.get("FLASHPREFILL_B200_CHECK", "0") not in ("", "0")

LAYOUT_KEYS = ["err", "cu_tile", "mk", "cnt", "idx", "total", "tiles", "cap"]


def set_mean_warps(w: int) -> None:
    """Choose the pooled-key summation order (4 or 8 warps of Triton's reduction)."""
    global _MEAN_WARPS
    if w not in (4, 8):
        raise ValueError("mean warps must be 4 or 8")
    _MEAN_WARPS = w


def get_mean_warps() -> int:
    return _MEAN_WARPS


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"flashprefill_b200 supports bfloat16 and float16 inputs (got {t.dtype})") from None


def _tma_ok(t: torch.Tensor) -> bool:
    """Can the kernels address t directly (last dim contiguous, 16-byte strides/base)?"""
    if t.stride(-1) != 1 or t.data_ptr() % 16 != 0:
        return False
    return all(s % 8 == 0 for s in t.stride()[:-1])


def _prep_input(t: torch.Tensor, name: str, ndim: int, device) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dimensions, got shape {tuple(t.shape)}")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (flashprefill_b200 has no CPU path), got {t.device}")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    return t if _tma_ok(t) else t.contiguous()


def _strides(t: torch.Tensor, n: int):
    return _lib.i64arr(t.stride()[:n])


def _P(x):
    return ctypes.c_void_p(x.data_ptr() if isinstance(x, torch.Tensor) else x)


def _finish(ws: torch.Tensor, stream) -> None:
    if _CHECK:
        check_device_error(ws, stream)


def check_device_error(ws: torch.Tensor, stream=None) -> int:
    """Synchronise and raise if the kernels recorded an error in the workspace."""
    lib = _lib.load()
    if stream is None:
        stream = torch.cuda.current_stream(ws.device).cuda_stream
    flags = ctypes.c_uint32(0)
    rc = lib.fpb_read_device_error(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(flags), ctypes.c_void_p(stream))
    if rc == _lib.FPB_EDEVICE:
        what = [m for b, m in _lib.DEV_ERROR_BITS.items() if flags.value & b]
        raise _lib.FlashPrefillError("flashprefill_b200 device error: " + "; ".join(what))
    _lib.check(rc)
    return flags.value


def dense_layout(batch, seqlen, hq, hk):
    out = (ctypes.c_int64 * 8)()
    _lib.check(_lib.load().fpb_workspace_layout(0, batch, seqlen, 0, hq, hk, 128, out))
    return dict(zip(LAYOUT_KEYS, list(out)))


def varlen_layout(nseq, total, max_seq_len, hq, hk):
    out = (ctypes.c_int64 * 8)()
    _lib.check(_lib.load().fpb_workspace_layout(1, nseq, total, max_seq_len, hq, hk, 128, out))
    return dict(zip(LAYOUT_KEYS, list(out)))


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def _views(ws, L, Hq, Hk, dtype):
    tiles, cap = int(L["tiles"]), int(L["cap"])
    cnt = ws[L["cnt"]:L["cnt"] + 4 * Hq * tiles].view(torch.int32).view(Hq, tiles)
    idx = ws[L["idx"]:L["idx"] + 4 * Hq * tiles * cap].view(torch.int32).view(Hq, tiles, cap)
    mk = ws[L["mk"]:L["mk"] + 2 * tiles * Hk * 128].view(dtype).view(tiles, Hk, 128)
    return cnt, idx, mk


# --------------------------------------------------------------------------- dense
def _dense_args(q, k, v, out, allow_chunk=False):
    device = q.device
    q = _prep_input(q, "q", 4, device)
    k = _prep_input(k, "k", 4, device)
    v = _prep_input(v, "v", 4, device) if v is not None else None
    B, S, Hq, D = q.shape
    if k.shape[0] != B or k.shape[3] != D or not (k.shape[1] == S or (allow_chunk and k.shape[1] > S)):
        raise ValueError(f"k shape {tuple(k.shape)} does not match q shape {tuple(q.shape)}")
    if v is not None and v.shape != k.shape:
        raise ValueError(f"v shape {tuple(v.shape)} must equal k shape {tuple(k.shape)}")
    if k.dtype != q.dtype or (v is not None and v.dtype != q.dtype):
        raise TypeError("q, k and v must share one dtype")
    if out is not None:
        if not isinstance(out, torch.Tensor) or out.shape != q.shape or out.dtype != q.dtype or out.device != device:
            raise ValueError("out must be a tensor with q's shape, dtype and device")
    return q, k, v, B, S, Hq, k.shape[2], D


def prefill_dense(q, k, v, out, block_size, attention_sink, window_size, alpha, last_n_block_full, min_budget,
                  workspace: torch.Tensor | None = None, out_peers=None, q_blocks=None):
    """Full operator on (B,S,H,D) tensors; writes ``out`` in place.  Returns the workspace.

    ``out_peers``: device addresses (ints) of the same output slice in other GPUs' copies of
    the output; every output tile is written there too (fpb_prefill_dense_peers).
    ``q_blocks``: (begin, end) query-block range; only those rows are searched and written,
    with the selection rules of the whole sequence (fpb_prefill_dense_rows).
    k/v longer than q: chunked prefill, the queries being the last q.shape[1] positions
    (fpb_prefill_dense_chunk)."""
    lib = _lib.load()
    Skv = k.shape[1] if isinstance(k, torch.Tensor) and k.dim() == 4 else None
    q, k, v, B, S, Hq, Hk, D = _dense_args(q, k, v, out, allow_chunk=True)
    if Skv is not None and Skv != S:
        if out_peers or q_blocks is not None:
            raise ValueError("chunked prefill cannot be combined with out_peers or q_blocks")
        return _prefill_chunk(lib, q, k, v, out, B, S, Skv, Hq, Hk, D, block_size, attention_sink, window_size,
                              alpha, last_n_block_full, min_budget, workspace)
    code = _dtype_code(q)
    tgt = out if _tma_ok(out) else torch.empty_like(q)
    if out_peers and tgt is not out:
        raise ValueError("out must be a TMA-compatible strided view when out_peers is given")
    ws = workspace if workspace is not None else _workspace(lib.fpb_dense_workspace_bytes(B, S, Hq, Hk, D), q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        args = (_P(q), _P(k), _P(v), _P(tgt), code, B, S, Hq, Hk, D, _strides(q, 3), _strides(k, 3), _strides(v, 3),
                _strides(tgt, 3), int(block_size), int(attention_sink), int(window_size), float(alpha),
                int(last_n_block_full), int(min_budget), _MEAN_WARPS, _P(ws), ws.numel())
        if out_peers and q_blocks is not None:
            raise ValueError("out_peers and q_blocks cannot be combined")
        if out_peers:
            peers = (ctypes.c_void_p * len(out_peers))(*[int(p) for p in out_peers])
            rc = lib.fpb_prefill_dense_peers(*args, peers, len(out_peers), _P(stream))
        elif q_blocks is not None:
            rc = lib.fpb_prefill_dense_rows(*args[:21], int(q_blocks[0]), int(q_blocks[1]), *args[21:], _P(stream))
        else:
            rc = lib.fpb_prefill_dense(*args, _P(stream))
    _lib.check(rc)
    if tgt is not out:
        out.copy_(tgt)
    _finish(ws, stream)
    return ws


def _prefill_chunk(lib, q, k, v, out, B, Sq, Skv, Hq, Hk, D, block_size, attention_sink, window_size, alpha,
                   last_n_block_full, min_budget, workspace):
    code = _dtype_code(q)
    tgt = out if _tma_ok(out) else torch.empty_like(q)
    ws = workspace if workspace is not None else _workspace(lib.fpb_dense_workspace_bytes(B, Skv, Hq, Hk, D), q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        rc = lib.fpb_prefill_dense_chunk(_P(q), _P(k), _P(v), _P(tgt), code, B, Sq, Skv, Hq, Hk, D, _strides(q, 3),
                                         _strides(k, 3), _strides(v, 3), _strides(tgt, 3), int(block_size),
                                         int(attention_sink), int(window_size), float(alpha), int(last_n_block_full),
                                         int(min_budget), _MEAN_WARPS, _P(ws), ws.numel(), _P(stream))
    _lib.check(rc)
    if tgt is not out:
        out.copy_(tgt)
    _finish(ws, stream)
    return ws


def search_dense(q, k, block_size=128, attention_sink=2, window_size=4, alpha=0.18, last_n_block_full=2,
                 min_budget=0, workspace: torch.Tensor | None = None):
    """Block search only.  Returns (counts [Hq, B*NB] int32, lists [Hq, B*NB, NB] int32,
    pooled keys [B*NB, Hk, D], workspace); row b*NB + qb of head h lists counts[h, row]
    ascending key-block indices."""
    lib = _lib.load()
    q, k, _, B, S, Hq, Hk, D = _dense_args(q, k, None, None)
    code = _dtype_code(q)
    L = dense_layout(B, S, Hq, Hk)
    ws = workspace if workspace is not None else _workspace(L["total"], q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        rc = lib.fpb_search_dense(_P(q), _P(k), code, B, S, Hq, Hk, D, _strides(q, 3), _strides(k, 3),
                                  int(block_size), int(attention_sink), int(window_size), float(alpha),
                                  int(last_n_block_full), int(min_budget), _MEAN_WARPS, _P(ws), ws.numel(),
                                  _P(stream))
    _lib.check(rc)
    _finish(ws, stream)
    return _views(ws, L, Hq, Hk, q.dtype) + (ws,)


def attention_dense(q, k, v, out, workspace: torch.Tensor, block_size=128):
    """Attention stage only over the block lists held in ``workspace``."""
    lib = _lib.load()
    q, k, v, B, S, Hq, Hk, D = _dense_args(q, k, v, out)
    code = _dtype_code(q)
    tgt = out if _tma_ok(out) else torch.empty_like(q)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        rc = lib.fpb_attention_dense(_P(q), _P(k), _P(v), _P(tgt), code, B, S, Hq, Hk, D, _strides(q, 3),
                                     _strides(k, 3), _strides(v, 3), _strides(tgt, 3), int(block_size),
                                     _P(workspace), workspace.numel(), _P(stream))
    _lib.check(rc)
    if tgt is not out:
        out.copy_(tgt)
    _finish(workspace, stream)


# --------------------------------------------------------------------------- varlen
def _varlen_args(q, k, v, o, cu_seqlens):
    device = q.device
    q = _prep_input(q, "q", 3, device)
    k = _prep_input(k, "k", 3, device)
    v = _prep_input(v, "v", 3, device) if v is not None else None
    T, Hq, D = q.shape
    if k.shape[0] != T or k.shape[2] != D:
        raise ValueError(f"k shape {tuple(k.shape)} does not match q shape {tuple(q.shape)}")
    if v is not None and v.shape != k.shape:
        raise ValueError("v shape must equal k shape")
    if k.dtype != q.dtype or (v is not None and v.dtype != q.dtype):
        raise TypeError("q, k and v must share one dtype")
    if o is not None and (o.shape != q.shape or o.dtype != q.dtype or o.device != device):
        raise ValueError("o must be a tensor with q's shape, dtype and device")
    if not isinstance(cu_seqlens, torch.Tensor) or cu_seqlens.dim() != 1 or cu_seqlens.numel() < 2:
        raise ValueError("cu_seqlens must be a 1-D tensor with at least 2 entries")
    if cu_seqlens.device != device:
        raise ValueError(f"cu_seqlens must be on {device}")
    cu = cu_seqlens if cu_seqlens.dtype == torch.int32 and cu_seqlens.is_contiguous() else \
        cu_seqlens.to(torch.int32).contiguous()
    return q, k, v, cu, T, Hq, k.shape[1], D


def prefill_varlen(q, k, v, o, cu_seqlens, max_seq_len, alpha, block_size=128, attention_sink=2, window_size=4,
                   last_n_block=2, workspace: torch.Tensor | None = None):
    """Full operator on packed (T,H,D) tensors; writes ``o`` in place.  Returns the workspace."""
    lib = _lib.load()
    q, k, v, cu, T, Hq, Hk, D = _varlen_args(q, k, v, o, cu_seqlens)
    code = _dtype_code(q)
    nseq = cu.numel() - 1
    tgt = o if _tma_ok(o) else torch.empty_like(q)
    nbytes = lib.fpb_varlen_workspace_bytes(T, nseq, int(max_seq_len), Hq, Hk, D)
    ws = workspace if workspace is not None else _workspace(nbytes, q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        rc = lib.fpb_prefill_varlen(_P(q), _P(k), _P(v), _P(tgt), code, _P(cu), nseq, T, int(max_seq_len), Hq, Hk,
                                    D, _strides(q, 2), _strides(k, 2), _strides(v, 2), _strides(tgt, 2),
                                    int(block_size), int(attention_sink), int(window_size), float(alpha),
                                    int(last_n_block), _MEAN_WARPS, _P(ws), ws.numel(), _P(stream))
    _lib.check(rc)
    if tgt is not o:
        o.copy_(tgt)
    _finish(ws, stream)
    return ws


def search_varlen(q, k, cu_seqlens, max_seq_len, alpha, block_size=128, attention_sink=2, window_size=4,
                  last_n_block=2, workspace: torch.Tensor | None = None):
    """Block search only.  Returns (counts [Hq, tiles], lists [Hq, tiles, cap], pooled keys,
    cu_tile [nseq+1], workspace)."""
    lib = _lib.load()
    q, k, _, cu, T, Hq, Hk, D = _varlen_args(q, k, None, None, cu_seqlens)
    code = _dtype_code(q)
    nseq = cu.numel() - 1
    L = varlen_layout(nseq, T, int(max_seq_len), Hq, Hk)
    ws = workspace if workspace is not None else _workspace(L["total"], q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        rc = lib.fpb_search_varlen(_P(q), _P(k), code, _P(cu), nseq, T, int(max_seq_len), Hq, Hk, D,
                                   _strides(q, 2), _strides(k, 2), int(block_size), int(attention_sink),
                                   int(window_size), float(alpha), int(last_n_block), _MEAN_WARPS, _P(ws),
                                   ws.numel(), _P(stream))
    _lib.check(rc)
    _finish(ws, stream)
    cnt, idx, mk = _views(ws, L, Hq, Hk, q.dtype)
    cu_tile = ws[L["cu_tile"]:L["cu_tile"] + 4 * (nseq + 1)].view(torch.int32)
    return cnt, idx, mk, cu_tile, ws


def attention_varlen(q, k, v, o, cu_seqlens, max_seq_len, workspace: torch.Tensor, block_size=128):
    """Attention stage only over the block lists (and cu_tile) held in ``workspace``."""
    lib = _lib.load()
    q, k, v, cu, T, Hq, Hk, D = _varlen_args(q, k, v, o, cu_seqlens)
    code = _dtype_code(q)
    nseq = cu.numel() - 1
    tgt = o if _tma_ok(o) else torch.empty_like(q)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        rc = lib.fpb_attention_varlen(_P(q), _P(k), _P(v), _P(tgt), code, _P(cu), nseq, T, int(max_seq_len), Hq,
                                      Hk, D, _strides(q, 2), _strides(k, 2), _strides(v, 2), _strides(tgt, 2),
                                      int(block_size), _P(workspace), workspace.numel(), _P(stream))
    _lib.check(rc)
    if tgt is not o:
        o.copy_(tgt)
    _finish(workspace, stream)
