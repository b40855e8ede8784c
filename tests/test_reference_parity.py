"""Parity with the reference implementation itself, on the GPU.

The reference's own operator (qhfan/FlashPrefill ``ops/``, Python + Triton, staged
unmodified by oracle/stage_ref.py) runs on the same bf16/fp16 inputs as this library:

* pooled keys: bit-identical to the reference's ``mean_k`` (its bf16 ``tl.sum`` order; the
  library reproduces the order of the warp count the reference's autotuner picks);
* block sets: identical, except blocks whose reference score lies within 1e-3 relative of
  the row threshold (counted and reported, allowed);
* outputs: within bf16 tolerance of an fp32 recomputation over the reference's mask
  (max-abs <= 2e-2, mean-abs <= 1e-3) on sampled query blocks, for both implementations,
  and close to the reference's own output everywhere.

Covers the BASELINE configurations at full size (32K Llama-shaped, the 128K headline
layer, the 8K/16K/32K/64K varlen batch, the 256K Qwen2.5-shaped layer with G = 7) and
small edge cases (ragged, batch 2, min_budget, threshold-only selection, G = 2/7/8,
zero- and one-token sequences).  fp16 and further small shapes are covered against the CPU
oracle (test_gpu_parity.py), whose fp32 model is pinned to the reference's own kernels.
"""
import math

import numpy as np
import pytest
import torch

import bench
import flashprefill_b200 as fp
from oracle import triton_ref as tr
from tests import gpu_util as gu

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not tr.available(), reason="reference sources not staged (oracle/stage_ref.py)")]

DEV = torch.device("cuda:0")
# ours vs the reference's own bf16 output: each is within MAX_ABS of the fp32 result
PAIR_MAX_ABS = 2 * gu.MAX_ABS


def _with_warps(w, fn):
    prev = fp.get_mean_warps()
    fp.set_mean_warps(w or 4)
    try:
        return fn()
    finally:
        fp.set_mean_warps(prev)


def _check_rows(q, k, v, out, ref_out, lists, rows, label):
    """Both outputs against the fp32 recomputation over the reference's lists."""
    exact = tr.recompute_rows(q, k, v, lists, rows)
    for (h, qb), o32 in exact.items():
        r0 = qb * 128
        for name, o in (("ours", out), ("reference", ref_out)):
            e = (o[r0:r0 + o32.shape[0], h].float() - o32).abs()
            assert e.max().item() <= gu.MAX_ABS and e.mean().item() <= gu.MEAN_ABS, \
                (label, name, h, qb, e.max().item(), e.mean().item())


def _dense_lists(ref, b=0):
    bi, cn = ref["block_index"][b].cpu(), ref["counts"][b].cpu()  # (NB,NB,H), (NB,H)
    return lambda h, qb: bi[qb, :int(cn[qb, h]), h].tolist()


def _run_dense(q, k, v, alpha, sink=2, window=4, last_n=2, budget=0, nrows=24, label=""):
    """q (B,S,Hq,D) etc. on the device.  Returns the mask report."""
    B, S, Hq, _ = q.shape
    ref_out = torch.zeros_like(q)
    ref = tr.run_dense(q, k, v, ref_out, 128, sink, window, alpha, last_n, budget)
    res = _with_warps(ref["mean_warps"], lambda: (fp.search_dense(q, k, 128, sink, window, alpha, last_n, budget),))
    cnt, idx, mk, ws = res[0]
    torch.cuda.synchronize()
    NB = ref["mk"].shape[1]
    assert torch.equal(mk[:B * NB].reshape(-1), ref["mk"].reshape(-1)), f"{label}: pooled keys differ"
    rep = tr.dense_mask_diff(ref, cnt, idx, alpha, B)
    print(f"{label}: mean_warps={ref['mean_warps']} {rep}")
    assert rep["other"] == 0, f"{label}: {rep['other']} block(s) differ outside the 1e-3 band"
    out = torch.zeros_like(q)
    _with_warps(ref["mean_warps"], lambda: fp.flash_prefill(q, k, v, out, 128, sink, window, alpha, last_n, budget))
    torch.cuda.synchronize()
    d = (out.float() - ref_out.float()).abs()
    print(f"  ours vs reference output: max-abs {d.max().item():.3e} mean-abs {d.mean().item():.3e}")
    assert d.max().item() <= PAIR_MAX_ABS and d.mean().item() <= gu.MEAN_ABS
    rng = np.random.default_rng(S + Hq)
    NBs = math.ceil(S / 128)
    for b in range(B):
        lst = _dense_lists(ref, b)
        rows = {(int(h), int(qb)) for h, qb in zip(rng.integers(0, Hq, nrows), rng.integers(0, NBs, nrows))}
        rows |= {(0, NBs - 1), (Hq - 1, 0)}
        _check_rows(q[b], k[b], v[b], out[b], ref_out[b], {r: lst(*r) for r in rows}, rows, label)
    return rep


def _run_varlen(q, k, v, lens, alpha, sink=2, window=4, last_n=2, nrows=8, label=""):
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32, device=DEV)
    Hq = q.shape[1]
    ref_out = torch.zeros_like(q)
    ref = tr.run_varlen(q, k, v, ref_out, cu, max(lens), alpha, 128, sink, window, last_n)
    cnt, idx, mk, cu_tile, ws = _with_warps(
        ref["mean_warps"], lambda: fp.search_varlen(q, k, cu, max(lens), alpha, 128, sink, window, last_n))
    torch.cuda.synchronize()
    n = ref["mk"].shape[0]
    assert torch.equal(mk[:n], ref["mk"]), f"{label}: pooled keys differ"
    rep = tr.varlen_mask_diff(ref, cnt, idx, lens, alpha)
    print(f"{label}: mean_warps={ref['mean_warps']} {rep}")
    assert rep["other"] == 0, f"{label}: {rep['other']} block(s) differ outside the 1e-3 band"
    out = torch.zeros_like(q)
    _with_warps(ref["mean_warps"], lambda: fp.flash_prefill_varlen_func(q, k, v, out, cu, max(lens), alpha, 128,
                                                                      sink, window, last_n))
    torch.cuda.synchronize()
    d = (out.float() - ref_out.float()).abs()
    print(f"  ours vs reference output: max-abs {d.max().item():.3e} mean-abs {d.mean().item():.3e}")
    assert d.max().item() <= PAIR_MAX_ABS and d.mean().item() <= gu.MEAN_ABS
    # reference CSR lists of sampled rows (row h * sum NB + tile)
    oi, ocu = ref["out_index"].cpu(), ref["out_number_cu"].cpu()
    nbs = [math.ceil(L / 128) for L in lens]
    tot = sum(nbs)
    rng = np.random.default_rng(sum(lens))
    start = base = 0
    for L, nb in zip(lens, nbs):
        if L:
            rows = {(int(h), int(qb)) for h, qb in zip(rng.integers(0, Hq, nrows), rng.integers(0, nb, nrows))}
            rows |= {(0, nb - 1)}
            lists = {(h, qb): oi[ocu[h * tot + base + qb]:ocu[h * tot + base + qb + 1]].tolist() for h, qb in rows}
            sl = slice(start, start + L)
            _check_rows(q[sl], k[sl], v[sl], out[sl], ref_out[sl], lists, rows, f"{label} seq len {L}")
        start += L
        base += nb
    return rep


def _device_layer(name):
    w = bench.workload(name)
    q, k, v = bench.device_inputs(w, 0, w.hk, DEV, seed=w.config_index * 1000 + 1)
    return w, q, k, v


@pytest.mark.parametrize("name", ["cfg1", "l128k", "cfg3"])
def test_full_size_dense_configs_match_reference(name):
    """BASELINE configs[1] (32K, 32/8), the 128K headline layer and configs[3] (256K, 28/4,
    G = 7, RoPE base 1e6, alpha 0.08, 0.5% heavy keys), at full size."""
    w, q, k, v = _device_layer(name)
    _run_dense(q[None], k[None], v[None], w.alpha, label=name)
    torch.cuda.empty_cache()


def test_full_size_varlen_config_matches_reference():
    """8K + 16K + 32K + 64K packed, 32/8 heads."""
    w, q, k, v = _device_layer("cfg2")
    _run_varlen(q, k, v, w.seqlens, w.alpha, label="cfg2")
    torch.cuda.empty_cache()


# Small cases share one shape per group (1000 tokens, 4/2 heads; 4096 tokens, 8/1 heads) so
# that the reference's autotuner benchmarks each shape once.
DENSE_EDGE = [
    # S,    B, hq, hk, alpha, sink, window, last_n, budget, dtype, rope, heavy
    (1000, 1, 4, 2, 0.18, 2, 4, 2, 0, torch.bfloat16, 500000.0, 0.01),   # ragged last block, G = 2
    (1000, 2, 4, 2, 0.05, 1, 2, 1, 0, torch.bfloat16, 500000.0, 0.01),   # batch 2, low alpha
    (1000, 1, 4, 2, 0.3, 2, 4, 2, 3, torch.bfloat16, 500000.0, 0.01),    # min_budget 3
    (1000, 1, 4, 2, 0.5, 0, 0, 0, 0, torch.bfloat16, 500000.0, 0.01),    # threshold only
    (4096, 1, 8, 1, 0.18, 2, 4, 2, 0, torch.bfloat16, 500000.0, 0.01),   # G = 8
]


@pytest.mark.parametrize("S,B,hq,hk,alpha,sink,window,last_n,budget,dtype,rope,heavy", DENSE_EDGE)
def test_dense_edge_cases_match_reference(S, B, hq, hk, alpha, sink, window, last_n, budget, dtype, rope, heavy):
    q, k, v, _ = gu.make_packed([S] * B, hq, hk, dtype, seed0=S + 31 * hq, rope_base=rope, heavy=heavy)
    qd, kd, vd = (t.view(B, S, -1, 128).to(DEV) for t in (q, k, v))
    _run_dense(qd, kd, vd, alpha, sink, window, last_n, budget, nrows=6, label=f"dense S={S} B={B} {hq}/{hk}")


VARLEN_EDGE = [
    ([1024, 0, 513, 1], 14, 2, 0.08, 3, 1, 1, torch.bfloat16),  # zero- and one-token sequences, G = 7
]


@pytest.mark.parametrize("lens,hq,hk,alpha,sink,window,last_n,dtype", VARLEN_EDGE)
def test_varlen_edge_cases_match_reference(lens, hq, hk, alpha, sink, window, last_n, dtype):
    q, k, v, _ = gu.make_packed(lens, hq, hk, dtype, seed0=sum(lens) + 3)
    _run_varlen(q.to(DEV), k.to(DEV), v.to(DEV), lens, alpha, sink, window, last_n, nrows=4,
                label=f"varlen {lens} {hq}/{hk}")
