"""Parity of the CUDA path (through the public API and the C ABI) with the CPU oracle.

Block lists must equal the oracle's exactly, except blocks whose score lies within 1e-3
relative of the row threshold (counted, reported, allowed).  Outputs must agree with an
fp32 recomputation over the same mask: max-abs <= 2e-2 and mean-abs <= 1e-3.
"""
import numpy as np
import pytest
import torch

import flashprefill_b200 as fp
from flashprefill_b200 import _ops
from oracle import restate
from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _oracle(q, k, cu, hq, hk, dtype, alpha, sink, window, last_n, dense, min_budget=0, warps=4):
    f = lambda t: t.float().cpu().numpy()
    return restate.search(f(q), f(k), cu, hq, hk, dt=gu.DT_NAME[dtype], alpha=alpha, sink=sink, window=window,
                          last_n=last_n, dense=dense, min_budget=min_budget, mean_model=f"tw{warps}")


def _check_masks(gmasks, res, label):
    bad, near, tot = gu.mask_diff(gmasks, res)
    print(f"{label}: selected={tot} mismatches_outside_band={bad} near_threshold_flips={near}")
    assert bad == 0, f"{label}: {bad} block(s) differ outside the 1e-3 threshold band"


DENSE_CASES = [
    # S,    B, hq, hk, alpha, sink, window, last_n, budget, dtype,          warps
    (1000, 1, 4, 2, 0.18, 2, 4, 2, 0, torch.bfloat16, 4),
    (4096, 1, 8, 2, 0.05, 2, 4, 2, 0, torch.bfloat16, 4),
    (4096, 1, 8, 2, 0.02, 1, 1, 0, 0, torch.bfloat16, 8),
    (2048, 1, 4, 1, 0.3, 2, 4, 2, 3, torch.bfloat16, 4),
    (3000, 1, 4, 4, 0.1, 0, 0, 0, 0, torch.float16, 4),
    (1536, 2, 4, 1, 0.18, 2, 4, 2, 0, torch.bfloat16, 4),
    (100, 1, 2, 1, 0.18, 2, 4, 2, 0, torch.bfloat16, 4),
    (8192, 1, 4, 1, 0.18, 2, 4, 2, 0, torch.bfloat16, 4),
]


@pytest.mark.parametrize("S,B,hq,hk,alpha,sink,window,last_n,budget,dtype,warps", DENSE_CASES)
def test_dense_matches_oracle(S, B, hq, hk, alpha, sink, window, last_n, budget, dtype, warps):
    q, k, v, cu = gu.make_packed([S] * B, hq, hk, dtype, seed0=S + hq)
    res = _oracle(q, k, cu, hq, hk, dtype, alpha, sink, window, last_n, True, budget, warps)
    qd, kd, vd = (t.view(B, S, -1, 128).to(DEV) for t in (q, k, v))
    prev = fp.get_mean_warps()
    fp.set_mean_warps(warps)
    try:
        cnt, idx, mk, ws = fp.search_dense(qd, kd, 128, sink, window, alpha, last_n, budget)
        torch.cuda.synchronize()
        assert fp.check_device_error(ws) == 0
        # pooled keys: bit-exact with the oracle's model of the reference's reduction
        np.testing.assert_array_equal(mk.float().cpu().numpy(), res["mk"])
        gmasks = gu.lists_to_masks(cnt, idx, cu, hq)
        _check_masks(gmasks, res, f"dense S={S} B={B} {hq}/{hk} alpha={alpha}")
        out = torch.empty_like(qd)
        fp.flash_prefill(qd, kd, vd, out, 128, sink, window, alpha, last_n, budget)
        torch.cuda.synchronize()
    finally:
        fp.set_mean_warps(prev)
    ref = gu.ref_attention_rows(q, k, v, cu, gmasks, hq, hk)
    mx, mean = gu.out_err(out.view(B * S, hq, 128), ref)
    print(f"  out max-abs {mx:.3e} mean-abs {mean:.3e}")
    assert mx <= gu.MAX_ABS and mean <= gu.MEAN_ABS


VARLEN_CASES = [
    ([300, 640, 129, 1], 4, 2, 0.18, 2, 4, 2, torch.bfloat16),
    ([1024, 0, 513], 4, 1, 0.05, 3, 1, 1, torch.bfloat16),
    ([8192, 4096, 100, 2048], 8, 2, 0.18, 2, 4, 2, torch.bfloat16),
    ([777, 1500], 4, 4, 0.02, 2, 4, 2, torch.float16),
]


@pytest.mark.parametrize("lens,hq,hk,alpha,sink,window,last_n,dtype", VARLEN_CASES)
def test_varlen_matches_oracle(lens, hq, hk, alpha, sink, window, last_n, dtype):
    q, k, v, cu = gu.make_packed(lens, hq, hk, dtype, seed0=sum(lens))
    res = _oracle(q, k, cu, hq, hk, dtype, alpha, sink, window, last_n, False)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    cud = torch.tensor(cu, dtype=torch.int32, device=DEV)
    cnt, idx, mk, cu_tile, ws = fp.search_varlen(qd, kd, cud, max(lens), alpha, 128, sink, window, last_n)
    torch.cuda.synchronize()
    assert fp.check_device_error(ws) == 0
    layout, ntiles = restate.seq_layout(cu)
    np.testing.assert_array_equal(cu_tile.cpu().numpy(), [0] + list(np.cumsum([x[2] for x in layout])))
    np.testing.assert_array_equal(mk[:ntiles].float().cpu().numpy(), res["mk"])
    gmasks = gu.lists_to_masks(cnt, idx, cu, hq)
    _check_masks(gmasks, res, f"varlen {lens} {hq}/{hk} alpha={alpha}")
    o = torch.zeros_like(qd)
    # positional 11-argument call, exactly as the vLLM patches make it
    fp.flash_prefill_varlen_func(qd, kd, vd, o, cud, max(lens), alpha, 128, sink, window, last_n)
    torch.cuda.synchronize()
    ref = gu.ref_attention_rows(q, k, v, cu, gmasks, hq, hk)
    mx, mean = gu.out_err(o, ref)
    print(f"  out max-abs {mx:.3e} mean-abs {mean:.3e}")
    assert mx <= gu.MAX_ABS and mean <= gu.MEAN_ABS


@pytest.mark.parametrize("S,hq,hk", [(640, 4, 2), (700, 2, 1), (1024, 8, 8)])
def test_full_mask_equals_causal_attention(S, hq, hk):
    """alpha = 0 selects every causal block: the output must be plain causal attention."""
    q, k, v, _ = gu.make_packed([S], hq, hk, torch.bfloat16, seed0=7)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out = torch.empty_like(qd)[None]
    fp.flash_prefill(qd[None], kd[None], vd[None], out, 128, 2, 4, 0.0, 2, 0)
    ref = gu.causal_reference(qd, kd, vd)
    err = (out[0].float() - ref).abs()
    assert err.max().item() <= gu.MAX_ABS and err.mean().item() <= gu.MEAN_ABS, (err.max(), err.mean())


def test_strided_views_match_contiguous():
    """HF callers pass q.transpose(1, 2) views of (B,H,S,D) buffers; no copy is needed."""
    S, hq, hk = 1536, 4, 2
    q, k, v, _ = gu.make_packed([S], hq, hk, torch.bfloat16, seed0=11)
    qd, kd, vd = (t[None].to(DEV) for t in (q, k, v))
    out_c = torch.empty_like(qd)
    fp.flash_prefill(qd, kd, vd, out_c, 128, 2, 4, 0.1, 2, 0)
    qt = qd.transpose(1, 2).contiguous().transpose(1, 2)
    kt = kd.transpose(1, 2).contiguous().transpose(1, 2)
    vt = vd.transpose(1, 2).contiguous().transpose(1, 2)
    assert not qt.is_contiguous()
    out_t = torch.empty(1, hq, S, 128, dtype=torch.bfloat16, device=DEV).transpose(1, 2)
    fp.flash_prefill(qt, kt, vt, out_t, 128, 2, 4, 0.1, 2, 0)
    torch.cuda.synchronize()
    assert torch.equal(out_c, out_t)


def test_cfg1_full_size_mask_parity():
    """BASELINE configs[1] (32K, 32/8, alpha 0.18): masks vs oracle at full size, output
    checked on a sample of query-block rows (plus a global finiteness check)."""
    S, hq, hk = 32768, 32, 8
    q, k, v, cu = gu.make_packed([S], hq, hk, torch.bfloat16, seed0=1000)
    res = _oracle(q, k, cu, hq, hk, torch.bfloat16, 0.18, 2, 4, 2, True)
    qd, kd, vd = (t[None].to(DEV) for t in (q, k, v))
    cnt, idx, mk, ws = fp.search_dense(qd, kd, 128, 2, 4, 0.18, 2, 0)
    torch.cuda.synchronize()
    gmasks = gu.lists_to_masks(cnt, idx, cu, hq)
    _check_masks(gmasks, res, "cfg1 32K")
    print(f"  density {gmasks[0].sum() / (hq * 256 * 257 / 2):.4f}")
    out = torch.empty_like(qd)
    fp.flash_prefill(qd, kd, vd, out, 128, 2, 4, 0.18, 2, 0)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    rng = np.random.default_rng(0)
    rows = {(0, int(h), int(b)) for h, b in zip(rng.integers(0, hq, 24), rng.integers(0, 256, 24))}
    rows |= {(0, 0, 255), (0, 31, 254), (0, 5, 0)}
    ref = gu.ref_attention_rows(q, k, v, cu, gmasks, hq, hk, rows=rows)
    o = out[0].float().cpu().numpy()
    for (_, h, b) in rows:
        e = np.abs(o[b * 128:(b + 1) * 128, h] - ref[b * 128:(b + 1) * 128, h])
        assert e.max() <= gu.MAX_ABS and e.mean() <= gu.MEAN_ABS, (h, b, e.max(), e.mean())


def test_bad_cu_seqlens_reported_on_device():
    """Malformed cu_seqlens is detected on the device (no host sync on the call path) and
    reported through the error word; nothing is read or written out of bounds."""
    q, k, v, _ = gu.make_packed([512], 2, 1, torch.bfloat16)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    cud = torch.tensor([0, 300, 200, 512], dtype=torch.int32, device=DEV)
    o = torch.zeros_like(qd)
    ws = _ops.prefill_varlen(qd, kd, vd, o, cud, 512, 0.1)
    with pytest.raises(fp.FlashPrefillError, match="cu_seqlens"):
        fp.check_device_error(ws)


@pytest.mark.parametrize("lens,varlen", [([20000], False), ([20000, 3000], True)])
def test_split_long_rows_match_oracle(lens, varlen, monkeypatch):
    """Rows longer than 64 listed blocks (here the last-N rows, 157 blocks) are processed as
    parallel chunks whose partial results are merged; their output must match the fp32
    recomputation like every other row, with and without the split."""
    hq, hk, alpha, dtype = 4, 1, 0.05, torch.bfloat16
    q, k, v, cu = gu.make_packed(lens, hq, hk, dtype, seed0=sum(lens) + 7)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    cud = torch.tensor(cu, dtype=torch.int32, device=DEV)
    if varlen:
        cnt, idx, _, _, ws = fp.search_varlen(qd, kd, cud, max(lens), alpha, 128, 2, 4, 2)
    else:
        cnt, idx, _, ws = fp.search_dense(qd[None], kd[None], 128, 2, 4, alpha, 2, 0)
    gmasks = gu.lists_to_masks(cnt, idx, cu, hq)
    layout, _ = restate.seq_layout(cu)
    rng = np.random.default_rng(0)
    rows = set()
    for si, (_, _, nb, _) in enumerate(layout):
        for h in range(hq):
            for qb in [nb - 1, nb - 2] + list(rng.integers(0, nb, 3)):
                rows.add((si, h, int(qb)))
    assert max(int(m.sum(-1).max()) for m in gmasks) > 64, "the case must contain rows to split"
    ref = gu.ref_attention_rows(q, k, v, cu, gmasks, hq, hk, rows=rows)
    sel = np.zeros(ref.shape[:2], bool)
    for si, h, qb in rows:
        start, L, _, _ = layout[si]
        sel[start + qb * 128:start + min(L, (qb + 1) * 128), h] = True
    for split in (True, False):
        if split:
            monkeypatch.delenv("FLASHPREFILL_B200_NO_SPLIT", raising=False)
        else:
            monkeypatch.setenv("FLASHPREFILL_B200_NO_SPLIT", "1")
        o = torch.zeros_like(qd)
        if varlen:
            fp.flash_prefill_varlen_func(qd, kd, vd, o, cud, max(lens), alpha, 128, 2, 4, 2)
        else:
            fp.flash_prefill(qd[None], kd[None], vd[None], o[None], 128, 2, 4, alpha, 2, 0)
        torch.cuda.synchronize()
        err = np.abs(o.float().cpu().numpy() - ref)[sel]
        print(f"  split={split} rows={len(rows)} max-abs {err.max():.3e} mean-abs {err.mean():.3e}")
        assert err.max() <= gu.MAX_ABS and err.mean() <= gu.MEAN_ABS


def test_prefill_peers_writes_every_copy():
    """fpb_prefill_dense_peers: one rank of a head-sharded layer (heads 4-7 of 8) writes its
    output slice into its own full output and into two 'peer' copies (other buffers on this
    GPU stand in for other GPUs' memory).  Every copy of the slice equals the plain prefill
    bit for bit, and the other heads are left alone.  20,000 tokens: split rows and a
    partial last block go through the peer path too."""
    S, hq, hk, HQ = 20000, 4, 1, 8
    q, k, v, cu = gu.make_packed([S], hq, hk, torch.bfloat16, seed0=77)
    qd, kd, vd = (t[None].to(DEV) for t in (q, k, v))
    ref = torch.empty_like(qd)
    fp.flash_prefill(qd, kd, vd, ref, 128, 2, 4, 0.05, 2, 0)
    fulls = [torch.full((1, S, HQ, 128), 7.0, dtype=torch.bfloat16, device=DEV) for _ in range(3)]
    slices = [f[:, :, 4:8] for f in fulls]
    _ops.prefill_dense(qd, kd, vd, slices[0], 128, 2, 4, 0.05, 2, 0,
                       out_peers=[slices[1].data_ptr(), slices[2].data_ptr()])
    torch.cuda.synchronize()
    for i, (f, sl) in enumerate(zip(fulls, slices)):
        assert torch.equal(sl, ref), f"copy {i} differs from the plain prefill"
        assert bool((f[:, :, :4] == 7.0).all()), f"copy {i}: heads outside the slice were written"


def test_query_block_ranges_partition_the_layer():
    """fpb_prefill_dense_rows over a partition of the query blocks (the 2-D split of one layer
    over GPUs) gives the block lists of the whole-layer call for every row in its range, the
    same outputs, and leaves the rows outside its range untouched."""
    S, hq, hk, alpha = 20000, 4, 1, 0.05
    q, k, v, cu = gu.make_packed([S], hq, hk, torch.bfloat16, seed0=31337)
    qd, kd, vd = (t[None].to(DEV) for t in (q, k, v))
    nb = (S + 127) // 128
    full = torch.empty_like(qd)
    ws_full = _ops.prefill_dense(qd, kd, vd, full, 128, 2, 4, alpha, 2, 0)
    L = _ops.dense_layout(1, S, hq, hk)
    cnt_f, idx_f, _ = _ops._views(ws_full, L, hq, hk, qd.dtype)
    parts = torch.full_like(qd, float("nan"))
    for lo, hi in [(0, 90), (90, 150), (150, nb)]:
        piece = torch.full_like(qd, float("nan"))
        ws = _ops.prefill_dense(qd, kd, vd, piece, 128, 2, 4, alpha, 2, 0, q_blocks=(lo, hi))
        torch.cuda.synchronize()
        assert fp.check_device_error(ws) == 0
        cnt, idx, _ = _ops._views(ws, L, hq, hk, qd.dtype)
        assert torch.equal(cnt[:, lo:hi], cnt_f[:, lo:hi])
        for h in range(hq):
            for qb in range(lo, hi):
                c = int(cnt_f[h, qb])
                assert torch.equal(idx[h, qb, :c], idx_f[h, qb, :c]), (h, qb)
        r0, r1 = lo * 128, min(S, hi * 128)
        assert torch.isnan(piece[:, :r0].float()).all() and torch.isnan(piece[:, r1:].float()).all()
        parts[:, r0:r1] = piece[:, r0:r1]
    d = (parts.float() - full.float()).abs()
    assert d.max().item() <= gu.MAX_ABS and d.mean().item() <= 1e-4, (d.max().item(), d.mean().item())
    with pytest.raises(ValueError):
        _ops.prefill_dense(qd, kd, vd, parts, 128, 2, 4, alpha, 2, 0, q_blocks=(5, 5))


@pytest.mark.parametrize("kv_len,q_len", [(3000, 1000), (4096, 1024), (1000, 1000), (2200, 37)])
def test_chunked_prefill_matches_oracle(kv_len, q_len):
    """Chunked prefill: queries are the last q_len positions of a kv_len-token sequence.  The
    oracle runs the whole sequence with the query rows before the chunk set to zero (the
    operator's definition: missing rows score as zero rows); block lists of the chunk's query
    blocks must match it and the chunk's outputs must match the fp32 recomputation."""
    hq, hk, alpha = 4, 1, 0.1
    q, k, v, cu = gu.make_packed([kv_len], hq, hk, torch.bfloat16, seed0=kv_len + q_len)
    q_off = kv_len - q_len
    qz = q.clone()
    qz[:q_off] = 0
    res = _oracle(qz, k, cu, hq, hk, torch.bfloat16, alpha, 2, 4, 2, True)
    qd = q[q_off:][None].to(DEV)
    kd, vd = k[None].to(DEV), v[None].to(DEV)
    out = torch.full_like(qd, float("nan"))
    ws = _ops.prefill_dense(qd, kd, vd, out, 128, 2, 4, alpha, 2, 0)
    torch.cuda.synchronize()
    assert fp.check_device_error(ws) == 0
    L = _ops.dense_layout(1, kv_len, hq, hk)
    cnt, idx, _ = _ops._views(ws, L, hq, hk, torch.bfloat16)
    nb = (kv_len + 127) // 128
    qb0 = q_off // 128
    sel = res["sel"][0]
    near = res["near"][0]
    got = np.zeros_like(sel)
    cnt_h, idx_h = cnt.cpu().numpy(), idx.cpu().numpy()
    for h in range(hq):
        for qb in range(qb0, nb):
            got[h, qb, idx_h[h, qb, :cnt_h[h, qb]]] = True
    diff = (got ^ sel)[:, qb0:]
    assert int((diff & ~near[:, qb0:]).sum()) == 0
    ref = gu.ref_attention_rows(qz, k, v, cu, [got], hq, hk)
    e = np.abs(out[0].float().cpu().numpy() - ref[q_off:])
    print(f"chunk kv={kv_len} q={q_len}: max-abs {e.max():.3e} mean-abs {e.mean():.3e}")
    assert e.max() <= gu.MAX_ABS and e.mean() <= gu.MEAN_ABS
    if q_off % 128 == 0:  # whole query blocks: the same rows of the full prefill, bit for bit
        full = torch.empty_like(kd.expand(-1, -1, hq, -1).contiguous())
        fp.flash_prefill(q[None].to(DEV), kd, vd, full, 128, 2, 4, alpha, 2, 0)
        torch.cuda.synchronize()
        assert torch.equal(full[:, q_off:], out)
