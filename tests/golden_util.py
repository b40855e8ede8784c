"""Loading of the golden fixtures made by tests/golden/make_golden.py (reference runs)."""
import glob
import hashlib
import json
import os

import numpy as np
import torch

from flashprefill_b200.synthetic import make_sequence

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    return meta, z


def regenerate(meta, dtype=torch.float32):
    """Re-create the fixture's inputs; returns packed q, k, v (numpy f32) and cu_seqlens."""
    seqs = [make_sequence(L, meta["hq"], meta["hk"], 128, 500000.0, 0.01, meta["seed0"] + i, torch.float32)
            for i, L in enumerate(meta["lens"])]
    h = hashlib.sha256()
    for q, k, v in seqs:
        for t in (q, k, v):
            h.update(t.contiguous().numpy().tobytes())
    assert h.hexdigest() == meta["sha"], "generator no longer reproduces the golden inputs"
    q = torch.cat([s[0] for s in seqs]).numpy()
    k = torch.cat([s[1] for s in seqs]).numpy()
    v = torch.cat([s[2] for s in seqs]).numpy()
    cu = np.zeros(len(seqs) + 1, np.int64)
    cu[1:] = np.cumsum(meta["lens"])
    return q, k, v, cu


def golden_sels(meta, z):
    out = []
    for si, nb in enumerate(meta["nbs"]):
        bits = np.unpackbits(z[f"sel_bits_{si}"])[: meta["hq"] * nb * nb]
        out.append(bits.reshape(meta["hq"], nb, nb).astype(bool))
    return out
