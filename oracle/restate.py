"""CPU restatement of FlashPrefill's sparse-prefill algorithm (the parity oracle).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` may import this module, and only as the checker or as the
timed CPU baseline.  The product path (``flashprefill_b200``) never calls it.

Every stage restates one piece of the reference (paths relative to the reference
project root):

* ``block_mean``        -- ops/flashprefill_native_forward.py:22-67 (compute_mean_vector),
                           ops/flashprefill_varlen_func.py:35-85 (compute_mean_vector_varlen)
* ``block_scores_head`` -- ops/flashprefill_native_forward.py:88-188 (compute_block_score),
                           ops/flashprefill_varlen_func.py:107-217
* ``select_row``        -- ops/flashprefill_native_forward.py:347-403 (deal_output_score,
                           normalize_scores); ops/flashprefill_varlen_func.py:240-409,656
* ``sparse_attention``  -- ops/flashprefill_native_forward.py:228-344 (_flash_forward),
                           ops/flashprefill_varlen_func.py:449-575

Values of 16-bit dtypes are carried as float32 arrays that hold exactly representable
values; ``round_to`` performs the round-to-nearest-even conversion.

Pooled-K rounding models (the only place where summation order changes selected blocks):

* ``"seq32"``  fp32 sum of rows 0..127 in order, fp32 divide.  This is what the reference
               computes when its Triton kernels run under the interpreter on CPU (numpy
               reduces axis 0 row after row); pinned by the golden fixtures.
* ``"tw4"``/``"tw8"``  the order Triton's reduction uses on the GPU for a 128x128 16-bit
               tile with 4 / 8 warps: each thread sums its rows sequentially (row = rep*2W
               + 2w + l), the lane pair (l=0,1) is combined, then the W warp partials are
               combined by xor shuffles of distance W/2, ..., 1 (W=4: (w0+w2)+(w1+w3)).
               Every add rounds to the input dtype.  Which of the two the reference picks
               depends on its autotuner, so it is a parameter here and in the CUDA kernel
               (default ``"tw4"``).
"""
from __future__ import annotations

import math

import numpy as np

LOG2E = 1.4426950408889634


# --------------------------------------------------------------------------- dtypes
def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def round_to(x: np.ndarray, dt: str) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    if dt == "bf16":
        return round_bf16(x)
    if dt == "fp16":
        return x.astype(np.float16).astype(np.float32)
    if dt == "fp32":
        return x
    raise ValueError(dt)


def scale_log2(head_dim: int) -> np.float32:
    """c = fp32(1/sqrt(D)) * fp32(log2 e), as the reference forms sm_scale (native:144)."""
    return np.float32(np.float32(1.0 / (head_dim ** 0.5)) * np.float32(LOG2E))


# ---------------------------------------------------------------------- sequences
def seq_layout(cu_seqlens, block: int = 128):
    """Per-sequence (start, length, nb, tile_base) and the total block count -- varlen:8-18."""
    cu = [int(x) for x in cu_seqlens]
    out, base = [], 0
    for i in range(len(cu) - 1):
        L = cu[i + 1] - cu[i]
        nb = (L + block - 1) // block
        out.append((cu[i], L, nb, base))
        base += nb
    return out, base


# ------------------------------------------------------------------- pooled keys
def _mean_tiles(x: np.ndarray, n_valid: np.ndarray, dt: str, model: str) -> np.ndarray:
    """Means of tiles x (nt, 128, ...) whose rows >= n_valid[t] are zero -- native:47-58."""
    if model == "seq32":
        acc = x[:, 0].astype(np.float32).copy()
        for r in range(1, x.shape[1]):
            acc = (acc + x[:, r]).astype(np.float32)
        s = acc
    elif model in ("tw4", "tw8"):
        W = 4 if model == "tw4" else 8
        step = 2 * W
        parts = []
        for w in range(W):
            pair = []
            for l in range(2):
                acc = x[:, 2 * w + l].copy()
                for rep in range(1, x.shape[1] // step):
                    acc = round_to(acc + x[:, rep * step + 2 * w + l], dt)
                pair.append(acc)
            parts.append(round_to(pair[0] + pair[1], dt))
        # warp partials are combined with xor shuffles of decreasing distance (W/2, ..., 1)
        n = W // 2
        while n >= 1:
            parts = [round_to(parts[w] + parts[w ^ n], dt) for w in range(W)]
            n //= 2
        s = parts[0]
    else:
        raise ValueError(model)
    nv = n_valid.astype(np.float32).reshape((-1,) + (1,) * (s.ndim - 1))
    with np.errstate(invalid="ignore", divide="ignore"):
        out = round_to(s.astype(np.float32) / nv, dt)
    out[n_valid <= 0] = 0.0
    return out


def block_mean(k: np.ndarray, cu_seqlens, dt: str, model: str, block: int = 128):
    """Pooled keys mk[tile, hk, :] for packed k (T, Hk, D) -- native:22-67, varlen:35-85."""
    layout, ntiles = seq_layout(cu_seqlens, block)
    T, HK, D = k.shape
    mk = np.zeros((ntiles, HK, D), np.float32)
    for (start, L, nb, base) in layout:
        if nb == 0:
            continue
        tiles = np.zeros((nb * block, HK, D), np.float32)
        tiles[:L] = k[start:start + L]
        tiles = tiles.reshape(nb, block, HK, D)
        n_valid = np.minimum(block, L - np.arange(nb) * block)
        mk[base:base + nb] = _mean_tiles(tiles, n_valid, dt, model)
    return mk


# ------------------------------------------------------------------- block scores
def block_scores_head(qh: np.ndarray, mk_h: np.ndarray, nb: int, c: np.float32, qbs=None):
    """(m, p) for the query blocks of one head -- native:129-188.

    qh: (nb*128, D) zero padded queries of the head; mk_h: (nb, D).  Returns m, p of shape
    (nb, nb) with m = -inf, p = 0 for kb > qb.  Row r of block qb is causal for kb iff
    qb*128 + r >= kb*128 + 127 (native:157): the diagonal block sees only row 127, and
    zero-padded rows past the end of the sequence count (their score is 0).
    """
    B = 128
    m = np.full((nb, nb), -np.inf, np.float32)
    p = np.zeros((nb, nb), np.float32)
    qbs = list(range(nb) if qbs is None else qbs)
    for c0 in range(0, len(qbs), 32):
        blk = np.array(qbs[c0:c0 + 32])
        rows = (blk[:, None] * B + np.arange(B)[None, :]).reshape(-1)
        hi = int(blk.max()) + 1
        s = (qh[rows].astype(np.float64) @ mk_h[:hi].astype(np.float64).T).astype(np.float32)
        s = (s * c).astype(np.float32).reshape(len(blk), B, hi)
        kb = np.arange(hi)
        causal = kb[None, :] < blk[:, None]               # off-diagonal: every row counts
        mm = s.max(axis=1)                                 # (nblk, hi)
        diag_val = s[np.arange(len(blk)), B - 1, blk]      # row 127 of the diagonal block
        mm = np.where(causal, mm, -np.inf).astype(np.float32)
        mm[np.arange(len(blk)), blk] = diag_val
        with np.errstate(over="ignore", invalid="ignore"):
            e = np.exp2((s - mm[:, None, :]).astype(np.float32)).astype(np.float32)
        pp = np.where(causal, e.sum(axis=1, dtype=np.float32), 0.0).astype(np.float32)
        pp[np.arange(len(blk)), blk] = 1.0
        m[blk, :hi] = mm
        p[blk, :hi] = pp
    return m, p


# ------------------------------------------------------------------- selection
def select_row(m: np.ndarray, p: np.ndarray, qb: int, nb: int, alpha: float, sink: int,
               window: int, last_n: int, dense: bool, min_budget: int = 0):
    """Selected key blocks of one query-block row -- native:347-403 / varlen:240-409,656.

    m, p: length qb+1 (causal entries).  Returns (sel bool[nb], score f32[nb], thr f32).
    Entries kb > qb score 0 (dense: masked to 0 by normalize_scores; varlen: excluded by
    the causal AND, and the NaNs the reference leaves there are ignored by Triton's max).
    """
    M = m.max()
    w = np.exp2((m - M).astype(np.float32)).astype(np.float32)
    pw = np.zeros(nb, np.float32)
    pw[: qb + 1] = (p * w).astype(np.float32)
    if dense:
        tot = pw.sum(dtype=np.float32)
        score = (pw / np.float32(tot + np.float32(1e-9))).astype(np.float32)
    else:
        score = pw
    top1 = score.max()
    thr = np.float32(top1 * np.float32(alpha))
    sel = score >= thr
    if dense and min_budget > 0:
        k = min(min_budget, nb)
        order = np.lexsort((np.arange(nb), -score.astype(np.float64)))
        sel = sel.copy()
        sel[order[:k]] = True
    kb = np.arange(nb)
    dist = qb - kb
    sel = sel | (kb < sink) | ((dist >= 0) & (dist < window)) | (qb >= nb - last_n)
    sel &= dist >= 0
    return sel, score, thr


def search(q: np.ndarray, k: np.ndarray, cu_seqlens, hq: int, hk: int, *, dt: str, alpha: float,
           sink: int = 2, window: int = 4, last_n: int = 2, dense: bool = True, min_budget: int = 0,
           mean_model: str = "tw4", block: int = 128, rows=None):
    """Block search over packed q (T,Hq,D), k (T,Hk,D).

    Returns a dict with ``mk`` (tiles,Hk,D), per-sequence ``sel`` (Hq,nb,nb) bool,
    ``score`` (Hq,nb,nb) f32, ``thr`` (Hq,nb) f32 and ``near`` (Hq,nb,nb) bool -- blocks
    whose score lies within 1e-3 relative of the row threshold.
    ``rows``: optional set of (seq, h, qb) to restrict work to (CPU-baseline sampling).
    """
    D = q.shape[2]
    G = hq // hk
    c = scale_log2(D)
    mk = block_mean(k, cu_seqlens, dt, mean_model, block)
    layout, _ = seq_layout(cu_seqlens, block)
    res = {"mk": mk, "sel": [], "score": [], "thr": [], "near": []}
    for si, (start, L, nb, base) in enumerate(layout):
        sel = np.zeros((hq, nb, nb), bool)
        score = np.zeros((hq, nb, nb), np.float32)
        thr = np.zeros((hq, nb), np.float32)
        qpad = np.zeros((nb * block, hq, D), np.float32)
        qpad[:L] = q[start:start + L]
        for h in range(hq):
            qbs = None
            if rows is not None:
                qbs = [qb for qb in range(nb) if (si, h, qb) in rows]
                if not qbs:
                    continue
            if nb == 0:
                continue
            m, p = block_scores_head(qpad[:, h], mk[base:base + nb, h // G], nb, c, qbs)
            for qb in (range(nb) if qbs is None else qbs):
                s_, sc, t = select_row(m[qb, :qb + 1], p[qb, :qb + 1], qb, nb, alpha, sink, window, last_n,
                                       dense, min_budget)
                sel[h, qb] = s_
                score[h, qb] = sc
                thr[h, qb] = t
        near = np.abs(score - thr[:, :, None]) <= 1e-3 * np.abs(thr[:, :, None])
        near &= np.tril(np.ones((nb, nb), bool))[None]
        res["sel"].append(sel)
        res["score"].append(score)
        res["thr"].append(thr)
        res["near"].append(near)
    return res


# ------------------------------------------------------------------- attention
def sparse_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_seqlens, sels, hq: int, hk: int,
                     block: int = 128, rows=None) -> np.ndarray:
    """fp32 recomputation of block-sparse causal GQA attention over the given masks.

    Mirrors native:270-344: for each query block the selected key blocks are attended,
    the diagonal block causally; a row with no selected block outputs zeros (the
    reference's l_i starts at 1.0 and acc at 0).  The softmax scale is 1/sqrt(D).
    """
    D = q.shape[2]
    G = hq // hk
    out = np.zeros(q.shape, np.float32)
    layout, _ = seq_layout(cu_seqlens, block)
    sc = 1.0 / math.sqrt(D)
    for si, (start, L, nb, base) in enumerate(layout):
        sel = sels[si]
        for h in range(hq):
            kh = k[start:start + L, h // G].astype(np.float64)
            vh = v[start:start + L, h // G].astype(np.float64)
            for qb in range(nb):
                if rows is not None and (si, h, qb) not in rows:
                    continue
                r0, r1 = qb * block, min(L, (qb + 1) * block)
                kbs = np.nonzero(sel[h, qb])[0]
                if kbs.size == 0:
                    continue
                keys = np.concatenate([np.arange(kb * block, min(L, (kb + 1) * block)) for kb in kbs])
                qq = q[start + r0:start + r1, h].astype(np.float64)
                s = (qq @ kh[keys].T) * sc
                qi = np.arange(r0, r1)[:, None]
                s = np.where(keys[None, :] <= qi, s, -np.inf)
                s -= s.max(axis=1, keepdims=True)
                e = np.exp(s)
                out[start + r0:start + r1, h] = ((e @ vh[keys]) / e.sum(axis=1, keepdims=True)).astype(np.float32)
    return out


def prefill(q, k, v, cu_seqlens, hq, hk, *, dt, alpha, sink=2, window=4, last_n=2, dense=True,
            min_budget=0, mean_model="tw4"):
    """search + sparse_attention over packed inputs; returns (out, search_result)."""
    res = search(q, k, cu_seqlens, hq, hk, dt=dt, alpha=alpha, sink=sink, window=window, last_n=last_n,
                 dense=dense, min_budget=min_budget, mean_model=mean_model)
    out = sparse_attention(q, k, v, cu_seqlens, res["sel"], hq, hk)
    return out, res
