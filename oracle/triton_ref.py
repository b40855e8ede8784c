"""The reference's own Triton path, run on the GPU as a checker and as a timed baseline.

TEST INFRASTRUCTURE ONLY.  Imported by ``tests/`` (parity against the reference itself) and by
bench.py's Triton baseline leg; the product path (``flashprefill_b200``) never imports it.

The reference operator (qhfan/FlashPrefill ``ops/``) is loaded unmodified from the copy that
``oracle/stage_ref.py`` stages into ``oracle/_ref/ops/``, under a private package name so that it
cannot collide with the ``ops`` aliases ``flashprefill_b200.install_as_ops()`` registers.  Nothing
in it is changed; a few of its module-level launchers are wrapped while a call runs so that
their arguments can be recorded:

* dense (``ops/flashprefill_native_forward.py``): the pooled keys ``mean_k`` at the launch of
  ``compute_block_score`` (native:438), the normalised scores returned by ``normalize_scores``
  (native:455), and ``block_index`` / ``counts`` at the launch of ``_flash_forward`` (native:464);
* varlen (``ops/flashprefill_varlen_func.py``): ``mean_k`` at ``compute_block_score_varlen``
  (varlen:621), the weighted scores at ``compute_block_max_varlen`` (varlen:668) and the CSR lists
  ``out_index`` / ``out_number_cu`` at ``_flash_block_sparse_varlen`` (varlen:705).

The mask comparisons follow the parity rule of the operator: block sets equal, except blocks
whose reference score lies within 1e-3 relative of the row's threshold ``alpha * max score``
(counted as ``near``; any other difference is ``other``).
"""
from __future__ import annotations

import contextlib
import importlib.util
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref", "ops")
_PKG = "flashprefill_reference_ops"


def available() -> bool:
    try:
        import triton  # noqa: F401
        import fla.utils  # noqa: F401
    except Exception:
        return False
    return os.path.isfile(os.path.join(REF_DIR, "__init__.py"))


def _static_compile():
    """The reference wraps two torch helpers in torch.compile.  After a few input shapes
    torch's dynamo would switch them to dynamic shapes, whose inductor build needs a host
    C++/OpenMP toolchain this image lacks; compiling each shape statically (as the first
    call of every shape does anyway) keeps them on the GPU code path."""
    import torch._dynamo.config as dc
    dc.automatic_dynamic_shapes = False
    for name in ("recompile_limit", "cache_size_limit"):
        if hasattr(dc, name):
            setattr(dc, name, max(getattr(dc, name), 256))


def load():
    """Import the staged reference package; returns (native module, varlen module)."""
    _static_compile()
    if _PKG not in sys.modules:
        if not os.path.isfile(os.path.join(REF_DIR, "__init__.py")):
            raise RuntimeError("reference sources are not staged (run oracle/stage_ref.py)")
        spec = importlib.util.spec_from_file_location(_PKG, os.path.join(REF_DIR, "__init__.py"),
                                                      submodule_search_locations=[REF_DIR])
        mod = importlib.util.module_from_spec(spec)
        sys.modules[_PKG] = mod
        spec.loader.exec_module(mod)
    return (sys.modules[_PKG + ".flashprefill_native_forward"], sys.modules[_PKG + ".flashprefill_varlen_func"])


class _Launch:
    """Stands in for a Triton launcher: records chosen arguments of each launch, then launches."""

    def __init__(self, fn, slots, store):
        self.fn, self.slots, self.store = fn, slots, store

    def __getitem__(self, grid):
        launch = self.fn[grid]

        def run(*args, **kw):
            r = launch(*args, **kw)
            for name, i in self.slots.items():
                self.store[name] = args[i].detach().clone()
            return r
        return run

    def __getattr__(self, n):
        return getattr(self.fn, n)


@contextlib.contextmanager
def _patched(mod, wraps):
    saved = {n: getattr(mod, n) for n in wraps}
    try:
        for n, w in wraps.items():
            setattr(mod, n, w(saved[n]))
        yield
    finally:
        for n, f in saved.items():
            setattr(mod, n, f)


def _record_return(store, name):
    def wrap(fn):
        def run(*a, **kw):
            r = fn(*a, **kw)
            store[name] = r.detach().clone()
            return r
        return run
    return wrap


def _mean_warps(kernel) -> int | None:
    cfg = getattr(kernel, "best_config", None)
    return getattr(cfg, "num_warps", None) if cfg is not None else None


def flash_prefill(q, k, v, out, block_size, sink, window, alpha, last_n, min_budget):
    """The reference's dense entry point, unmodified (``ops.flash_prefill``, native:481-499)."""
    nf, _ = load()
    nf.flash_prefill(q, k, v, out, block_size, sink, window, alpha, last_n, min_budget)


def flash_prefill_varlen_func(q, k, v, o, cu, max_seq_len, alpha, block_size=128, sink=2, window=4, last_n=2):
    """The reference's varlen entry point, unmodified (``ops.flash_prefill_varlen_func``, varlen:723-743)."""
    _, vf = load()
    vf.flash_prefill_varlen_func(q, k, v, o, cu, max_seq_len, alpha, block_size, sink, window, last_n)


def run_dense(q, k, v, out, block_size, sink, window, alpha, last_n, min_budget):
    """One reference dense call with its intermediates recorded.  Returns a dict with ``mk``
    (B, NB, Hk, D), ``score`` (B, NB, NB, Hq) fp32 normalised, ``block_index`` (B, NB, NB, Hq)
    int64 ascending padded with NB, ``counts`` (B, NB, Hq) int32 and ``mean_warps``."""
    nf, _ = load()
    st = {}
    with _patched(nf, {"compute_block_score": lambda f: _Launch(f, {"mk": 1}, st),
                       "normalize_scores": _record_return(st, "score"),
                       "_flash_forward": lambda f: _Launch(f, {"block_index": 4, "counts": 5}, st)}):
        nf.flash_prefill(q, k, v, out, block_size, sink, window, alpha, last_n, min_budget)
    st["mean_warps"] = _mean_warps(nf.compute_mean_vector)
    return st


def run_varlen(q, k, v, o, cu, max_seq_len, alpha, block_size=128, sink=2, window=4, last_n=2):
    """One reference varlen call with its intermediates recorded: ``mk`` (sum NB_i, Hk, D),
    ``score`` (sum NB_i^2, Hq) fp32, ``out_index`` (CSR int32, head-major -> sequence -> query
    block), ``out_number_cu`` (Hq * sum NB_i + 1) and ``mean_warps``."""
    _, vf = load()
    st = {}
    with _patched(vf, {"compute_block_score_varlen": lambda f: _Launch(f, {"mk": 1}, st),
                       "compute_block_max_varlen": lambda f: _Launch(f, {"score": 0}, st),
                       "_flash_block_sparse_varlen": lambda f: _Launch(f, {"out_index": 4, "out_number_cu": 5}, st)}):
        vf.flash_prefill_varlen_func(q, k, v, o, cu, max_seq_len, alpha, block_size, sink, window, last_n)
    st["mean_warps"] = _mean_warps(vf.compute_mean_vector_varlen)
    return st


# --------------------------------------------------------------------------- masks
def _band(score, thr):
    return (score - thr).abs() <= 1e-3 * thr.abs()


def dense_mask_diff(ref: dict, cnt: torch.Tensor, idx: torch.Tensor, alpha: float, batch: int = 1):
    """Compare our lists (counts [Hq, B*NB], lists [Hq, B*NB, cap]) with the reference's dense
    block_index / counts; returns {"selected", "exact_rows", "near", "other"}."""
    bi, cn, sc = ref["block_index"], ref["counts"], ref["score"]  # (B,NB,NB,H), (B,NB,H), (B,NB,NB,H)
    B, NB, _, H = bi.shape
    dev = bi.device
    ar = torch.arange(NB, device=dev)
    # reference masks, (B, H, NB, NB+1) with the padding column dropped
    valid = ar.view(1, 1, NB, 1) < cn.unsqueeze(2)  # (B,NB,NB,H): list position j < count
    rm = torch.zeros(B, NB, NB + 1, H, dtype=torch.bool, device=dev)
    rm.scatter_(2, torch.where(valid, bi, torch.full_like(bi, NB)), True)
    rm = rm[:, :, :NB].permute(0, 3, 1, 2)  # (B,H,qb,kb)
    c = cnt[:, :B * NB].view(H, B, NB).permute(1, 0, 2)  # (B,H,NB)
    ix = idx[:, :B * NB, :NB].view(H, B, NB, -1).permute(1, 0, 2, 3).long()
    gv = torch.arange(ix.shape[-1], device=dev).view(1, 1, 1, -1) < c.unsqueeze(-1)
    gm = torch.zeros(B, H, NB, NB + 1, dtype=torch.bool, device=dev)
    gm.scatter_(3, torch.where(gv, ix, torch.full_like(ix, NB)), True)
    gm = gm[..., :NB]
    diff = rm ^ gm
    s = sc.permute(0, 3, 1, 2)  # (B,H,qb,kb)
    thr = alpha * s.max(dim=3, keepdim=True).values
    near = diff & _band(s, thr)
    return {"selected": int(rm.sum()), "near": int(near.sum()), "other": int((diff & ~near).sum()),
            "rows_differing": int(diff.any(-1).sum())}


def varlen_mask_diff(ref: dict, cnt: torch.Tensor, idx: torch.Tensor, seqlens, alpha: float):
    """Compare our varlen lists with the reference's CSR lists (same row numbering:
    row ``h * sum NB + tile``).  Returns {"selected", "near", "other", "rows_differing"}."""
    oi, ocu, sc = ref["out_index"].long(), ref["out_number_cu"].long(), ref["score"]
    dev = oi.device
    nbs = [(L + 127) // 128 for L in seqlens]
    tot = sum(nbs)
    H = cnt.shape[0]
    cap = max(nbs) if nbs else 1
    rows = H * tot
    lens_r = (ocu[1:] - ocu[:-1])
    row_of = torch.repeat_interleave(torch.arange(rows, device=dev), lens_r)
    rm = torch.zeros(rows, cap, dtype=torch.bool, device=dev)
    rm[row_of, oi] = True
    c = cnt[:, :tot].reshape(rows)
    ix = idx[:, :tot, :cap].reshape(rows, -1).long()
    gv = torch.arange(ix.shape[-1], device=dev).view(1, -1) < c.unsqueeze(-1)
    gm = torch.zeros(rows, cap + 1, dtype=torch.bool, device=dev)
    gm.scatter_(1, torch.where(gv, ix, torch.full_like(ix, cap)), True)
    gm = gm[:, :cap]
    diff = rm ^ gm
    # reference score of each (row, kb): score[cu_tile2[s] + qb * NB_s + kb, h]
    s_full = torch.full((rows, cap), float("nan"), device=dev)
    t0 = t2 = 0
    for nb in nbs:
        if nb:
            blk = sc[t2:t2 + nb * nb].view(nb, nb, H).permute(2, 0, 1)  # (H, qb, kb)
            s_full.view(H, tot, cap)[:, t0:t0 + nb, :nb] = blk
        t0 += nb
        t2 += nb * nb
    causal = torch.zeros(H, tot, cap, dtype=torch.bool, device=dev)
    t0 = 0
    for nb in nbs:
        if nb:
            causal[:, t0:t0 + nb, :nb] = torch.ones(nb, nb, dtype=torch.bool, device=dev).tril()
        t0 += nb
    causal = causal.view(rows, cap)
    s_c = torch.where(causal, s_full, torch.full_like(s_full, float("-inf")))
    thr = alpha * s_c.max(dim=1, keepdim=True).values
    near = diff & _band(s_full, thr)
    return {"selected": int(rm.sum()), "near": int(near.sum()), "other": int((diff & ~near).sum()),
            "rows_differing": int(diff.any(-1).sum())}


# --------------------------------------------------------------------------- fp32 recomputation
def recompute_rows(q, k, v, lists, rows):
    """fp32 attention of chosen 128-row query blocks over given key-block lists, on the device.

    q (S, Hq, D), k/v (S, Hk, D) of ONE sequence; ``lists[(h, qb)]`` = key blocks; ``rows`` =
    iterable of (h, qb).  Returns {(h, qb): (rows_in_block, D) fp32}."""
    S, Hq, D = q.shape
    G = Hq // k.shape[1]
    c = 1.0 / (D ** 0.5)
    out = {}
    for h, qb in rows:
        r0, r1 = qb * 128, min(S, qb * 128 + 128)
        kbs = sorted(int(x) for x in lists[(h, qb)])
        if not kbs:
            out[(h, qb)] = torch.zeros(r1 - r0, D, device=q.device)
            continue
        pos = torch.cat([torch.arange(kb * 128, min(S, kb * 128 + 128), device=q.device) for kb in kbs])
        qq = q[r0:r1, h].float()
        kk = k[pos, h // G].float()
        vv = v[pos, h // G].float()
        s = (qq @ kk.T) * c
        qpos = torch.arange(r0, r1, device=q.device).view(-1, 1)
        s = s.masked_fill(pos.view(1, -1) > qpos, float("-inf"))
        p = torch.softmax(s, dim=1)
        p = torch.nan_to_num(p, nan=0.0)
        out[(h, qb)] = p @ vv
    return out
