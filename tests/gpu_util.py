"""Helpers shared by the GPU parity tests: oracle runs on the same inputs and mask diffs."""
from __future__ import annotations

import math

import numpy as np
import torch

from flashprefill_b200.synthetic import make_sequence
from oracle import restate

DT_NAME = {torch.bfloat16: "bf16", torch.float16: "fp16"}

# Output tolerance against an fp32 recomputation over the same block mask.
MAX_ABS = 2e-2
MEAN_ABS = 1e-3


def make_packed(lens, hq, hk, dtype, seed0=0, rope_base=500000.0, heavy=0.01):
    seqs = [make_sequence(L, hq, hk, 128, rope_base, heavy, seed0 + i, dtype) for i, L in enumerate(lens)]
    q = torch.cat([s[0] for s in seqs])
    k = torch.cat([s[1] for s in seqs])
    v = torch.cat([s[2] for s in seqs])
    cu = np.zeros(len(lens) + 1, np.int64)
    cu[1:] = np.cumsum(lens)
    return q, k, v, cu


def lists_to_masks(cnt, idx, cu, hq):
    """GPU block lists -> per-sequence boolean masks (hq, nb, nb)."""
    cnt = cnt.cpu().numpy()
    idx = idx.cpu().numpy()
    layout, _ = restate.seq_layout(cu)
    out = []
    for (start, L, nb, base) in layout:
        m = np.zeros((hq, nb, nb), bool)
        for h in range(hq):
            for qb in range(nb):
                c = int(cnt[h, base + qb])
                assert 0 <= c <= qb + 1, (h, qb, c)
                lst = idx[h, base + qb, :c]
                assert np.all(np.diff(lst) > 0), "block list not strictly ascending"
                m[h, qb, lst] = True
        out.append(m)
    return out


def mask_diff(gpu_masks, res):
    """(#mismatches outside the 1e-3 threshold band, #inside, #selected by the oracle)."""
    bad = near = tot = 0
    for g, o, nr in zip(gpu_masks, res["sel"], res["near"]):
        d = g ^ o
        bad += int((d & ~nr).sum())
        near += int((d & nr).sum())
        tot += int(o.sum())
    return bad, near, tot


def ref_attention_rows(q, k, v, cu, masks, hq, hk, rows=None):
    """fp32 recomputation over the given masks (optionally only some (seq, h, qb) rows)."""
    f = lambda t: t.float().cpu().numpy()
    return restate.sparse_attention(f(q), f(k), f(v), cu, masks, hq, hk, rows=rows)


def out_err(out, ref):
    e = np.abs(out.float().cpu().numpy() - ref)
    return float(e.max()), float(e.mean())


def causal_reference(q, k, v):
    """Dense causal GQA attention in fp32 on the GPU; q (S,Hq,D), k/v (S,Hk,D)."""
    S, hq, d = q.shape
    g = hq // k.shape[1]
    qf = q.float().transpose(0, 1)
    kf = k.float().repeat_interleave(g, 1).transpose(0, 1)
    vf = v.float().repeat_interleave(g, 1).transpose(0, 1)
    s = (qf @ kf.transpose(1, 2)) / math.sqrt(d)
    s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    return (s.softmax(-1) @ vf).transpose(0, 1)
