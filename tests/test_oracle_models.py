"""Properties of the oracle's building blocks (dtype rounding, pooled-key models, rules)."""
import numpy as np
import torch

from oracle import restate


def test_round_bf16_matches_torch():
    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 100
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(restate.round_bf16(x), ref)


def test_mean_models_exact_on_integers():
    # integer keys: every partial sum is exact in bf16 (|sum| < 256), so all orders agree
    rng = np.random.default_rng(1)
    x = rng.integers(-1, 2, size=(3, 128, 2, 128)).astype(np.float32)
    nv = np.array([128, 128, 77])
    x[2, 77:] = 0
    for m in ("tw4", "tw8", "seq32"):
        got = restate._mean_tiles(x, nv, "bf16", m)
        exact = restate.round_bf16(x.sum(axis=1) / nv[:, None, None].astype(np.float32))
        np.testing.assert_array_equal(got, exact)


def test_mean_models_differ_on_random_bf16():
    rng = np.random.default_rng(2)
    x = restate.round_bf16(rng.standard_normal((64, 128, 1, 128)).astype(np.float32) * 3)
    nv = np.full(64, 128)
    a = restate._mean_tiles(x, nv, "bf16", "tw4")
    b = restate._mean_tiles(x, nv, "bf16", "tw8")
    c = restate.round_bf16(x.sum(axis=1) / 128)
    assert (a != b).mean() > 0.05 and (a != c).mean() > 0.05


def test_structural_rules():
    nb, qb = 10, 6
    m = np.zeros(qb + 1, np.float32)
    p = np.ones(qb + 1, np.float32)
    sel, _, _ = restate.select_row(m, p, qb, nb, alpha=2.0, sink=2, window=3, last_n=0, dense=True)
    assert sel.nonzero()[0].tolist() == [0, 1, 4, 5, 6]
    sel, _, _ = restate.select_row(np.zeros(10, np.float32), np.ones(10, np.float32), 9, nb, alpha=2.0, sink=0,
                                   window=0, last_n=1, dense=True)
    assert sel.all()
    sel, _, _ = restate.select_row(m, p, qb, nb, alpha=0.0, sink=0, window=0, last_n=0, dense=False)
    assert sel[:qb + 1].all() and not sel[qb + 1:].any()


def test_min_budget_forces_topk():
    m = np.zeros(5, np.float32)
    p = np.array([5, 1, 4, 3, 1], np.float32)
    sel, _, _ = restate.select_row(m, p, 4, 5, alpha=0.9, sink=0, window=0, last_n=0, dense=True, min_budget=3)
    assert sel.nonzero()[0].tolist() == [0, 2, 3]


def test_search_small_bf16_is_causal_and_structural():
    from flashprefill_b200.synthetic import make_sequence
    q, k, v = make_sequence(700, 4, 2, 128, 500000.0, 0.01, 3, torch.bfloat16)
    f = lambda t: t.float().numpy()
    res = restate.search(f(q), f(k), [0, 700], 4, 2, dt="bf16", alpha=0.18)
    sel = res["sel"][0]
    assert not np.triu(sel, 1).any()
    assert sel[:, :, 0].all()                         # sink
    assert sel[:, np.arange(6), np.arange(6)].all()  # window includes the diagonal
