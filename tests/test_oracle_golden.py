"""Pins the CPU oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by running the reference's Triton kernels under the Triton
interpreter in fp32 (tests/golden/make_golden.py).  The oracle must reproduce the pooled
keys bit-exactly (model "seq32"), the selected block sets exactly except for blocks whose
score lies within 1e-3 relative of the row threshold, and the outputs to fp32 accuracy.
"""
import numpy as np
import pytest

from oracle import restate
from tests import golden_util as gu

NAMES = gu.golden_names()


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_golden(name):
    meta, z = gu.load(name)
    q, k, v, cu = gu.regenerate(meta)
    dense = meta["kind"] == "dense"
    res = restate.search(q, k, cu, meta["hq"], meta["hk"], dt="fp32", alpha=meta["alpha"], sink=meta["sink"],
                         window=meta["window"], last_n=meta["last_n"], dense=dense,
                         min_budget=meta["min_budget"], mean_model="seq32")
    # pooled keys: bit-exact
    np.testing.assert_array_equal(res["mk"], z["mk"])
    # selected blocks: exact outside the 1e-3 threshold band
    gsel = gu.golden_sels(meta, z)
    for si in range(len(gsel)):
        diff = res["sel"][si] ^ gsel[si]
        assert not (diff & ~res["near"][si]).any(), f"seq {si}: {int(diff.sum())} mismatched blocks"
    # outputs: fp32 recompute over the reference's own mask
    out = restate.sparse_attention(q, k, v, cu, gsel, meta["hq"], meta["hk"])
    rows = z["out_rows"]
    err = np.abs(out[rows] - z["out"])
    assert err.max() < 5e-4 and err.mean() < 1e-5, (err.max(), err.mean())
