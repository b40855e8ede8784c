"""Generate the golden fixtures by running the REFERENCE implementation itself.

The reference (qhfan/FlashPrefill, ``ops/``) is pure Triton and has no CPU path; its own
kernels run on the CPU under Triton's interpreter (``TRITON_INTERPRET=1``) in fp32.  This
script imports the reference from a checkout (argument ``--ref``), runs its two public
entry points on seeded inputs from ``flashprefill_b200.synthetic`` and records, per case:

* ``mk``       -- the pooled keys the reference computed (captured at the launch of its
                  score kernel, native:438 / varlen:621),
* ``sel_bits`` -- the selected block sets (captured at the launch of its attention kernel,
                  from block_index+counts native:464 or out_index+out_number_cu varlen:705),
* ``out``      -- attention output rows (every ``stride``-th token, all heads),
* ``sha``      -- SHA-256 of the generated fp32 inputs, so the tests can check that the
                  generator still reproduces the exact inputs the fixture was made from.

Interpreter shims (the reference needs a GPU otherwise): fla's ``custom_device_ctx`` becomes
a null context, each autotuner keeps a single config (the score kernel the widest K tile, so
that every varlen score entry of a row is computed), and torch.compile is disabled.

Run in an environment where the reference and fla are importable:
    python tests/golden/make_golden.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import contextlib
import hashlib
import json
import os
import sys
import time
import warnings

os.environ["TRITON_INTERPRET"] = "1"
os.environ["TORCHDYNAMO_DISABLE"] = "1"
warnings.filterwarnings("ignore")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from flashprefill_b200.synthetic import make_sequence  # noqa: E402

# Each case: dense cases are a batch of equal-length sequences; varlen cases are packed.
CASES = [
    dict(name="dense_ragged_g2", kind="dense", lens=[1000], hq=4, hk=2, alpha=0.18, sink=2, window=4, last_n=2,
         min_budget=0, seed0=100),
    dict(name="dense_batch2_lowalpha", kind="dense", lens=[768, 768], hq=4, hk=1, alpha=0.05, sink=1, window=2,
         last_n=1, min_budget=0, seed0=200),
    dict(name="dense_budget3", kind="dense", lens=[1024], hq=2, hk=1, alpha=0.3, sink=2, window=4, last_n=2,
         min_budget=3, seed0=300),
    dict(name="dense_single_partial", kind="dense", lens=[100], hq=2, hk=1, alpha=0.18, sink=2, window=4, last_n=2,
         min_budget=0, seed0=400),
    dict(name="dense_threshold_only_g1", kind="dense", lens=[640], hq=4, hk=4, alpha=0.5, sink=0, window=0,
         last_n=0, min_budget=0, seed0=500),
    dict(name="dense_alpha002", kind="dense", lens=[896], hq=4, hk=1, alpha=0.02, sink=2, window=4, last_n=2,
         min_budget=0, seed0=600),
    dict(name="varlen_ragged", kind="varlen", lens=[300, 640, 129, 1], hq=4, hk=2, alpha=0.18, sink=2, window=4,
         last_n=2, min_budget=0, seed0=700),
    dict(name="varlen_zero_len", kind="varlen", lens=[1024, 0, 513], hq=4, hk=1, alpha=0.05, sink=3, window=1,
         last_n=1, min_budget=0, seed0=800),
    dict(name="cfg0", kind="dense", lens=[4096], hq=4, hk=1, alpha=0.18, sink=2, window=4, last_n=2, min_budget=0,
         seed0=0, out_stride=17),
]


def gen_inputs(case):
    seqs = [make_sequence(L, case["hq"], case["hk"], 128, 500000.0, 0.01, case["seed0"] + i, torch.float32)
            for i, L in enumerate(case["lens"])]
    return seqs


def input_sha(seqs) -> str:
    h = hashlib.sha256()
    for q, k, v in seqs:
        for t in (q, k, v):
            h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


def setup_reference(ref):
    sys.path.insert(0, ref)
    import fla.utils as fu
    fu.custom_device_ctx = lambda i: contextlib.nullcontext()
    from triton.runtime.autotuner import Autotuner
    import ops.flashprefill_native_forward as nf
    import ops.flashprefill_varlen_func as vf
    for mod in (nf, vf):
        for n in dir(mod):
            a = getattr(mod, n)
            if isinstance(a, Autotuner):
                if n.startswith("compute_block_score"):
                    best = max(a.configs, key=lambda c: c.kwargs.get("K_TILE_SIZE", 0))
                    a.configs = [best]
                else:
                    a.configs = [a.configs[0]]
    return nf, vf


class _Capture:
    """Wraps a Triton launcher so the arguments of its launch can be recorded."""

    def __init__(self, fn, slots, store):
        self.fn, self.slots, self.store = fn, slots, store

    def __getitem__(self, grid):
        def run(*args, **kw):
            for name, i in self.slots.items():
                self.store[name] = args[i].detach().clone()
            return self.fn[grid](*args, **kw)
        return run


def run_case(nf, vf, case):
    seqs = gen_inputs(case)
    hq, hk = case["hq"], case["hk"]
    cap = {}
    lens = case["lens"]
    nbs = [(L + 127) // 128 for L in lens]
    t0 = time.time()
    if case["kind"] == "dense":
        S = lens[0]
        q = torch.stack([s[0] for s in seqs])
        k = torch.stack([s[1] for s in seqs])
        v = torch.stack([s[2] for s in seqs])
        out = torch.zeros_like(q)
        orig_s, orig_a = nf.compute_block_score, nf._flash_forward
        nf.compute_block_score = _Capture(orig_s, {"mk": 1}, cap)
        nf._flash_forward = _Capture(orig_a, {"idx": 4, "cnt": 5}, cap)
        try:
            nf.flash_prefill(q, k, v, out, 128, case["sink"], case["window"], case["alpha"], case["last_n"],
                             case["min_budget"])
        finally:
            nf.compute_block_score, nf._flash_forward = orig_s, orig_a
        B, NB = len(lens), nbs[0]
        mk = cap["mk"].reshape(B * NB, hk, 128).numpy()
        sel = np.zeros((B, hq, NB, NB), bool)
        idx, cnt = cap["idx"], cap["cnt"]  # (B,NB,NB,H) int64, (B,NB,H)
        for b in range(B):
            for h in range(hq):
                for qb in range(NB):
                    c = int(cnt[b, qb, h])
                    sel[b, h, qb, idx[b, qb, :c, h].numpy()] = True
        sels = [sel[b] for b in range(B)]
        out_packed = out.reshape(B * S, hq, 128).numpy()
    else:
        q = torch.cat([s[0] for s in seqs])
        k = torch.cat([s[1] for s in seqs])
        v = torch.cat([s[2] for s in seqs])
        cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(torch.tensor(lens), 0)
        out = torch.zeros_like(q)
        orig_s, orig_a = vf.compute_block_score_varlen, vf._flash_block_sparse_varlen
        vf.compute_block_score_varlen = _Capture(orig_s, {"mk": 1}, cap)
        vf._flash_block_sparse_varlen = _Capture(orig_a, {"idx": 4, "cu": 5}, cap)
        try:
            vf.flash_prefill_varlen_func(q, k, v, out, cu, max(lens), case["alpha"], 128, case["sink"],
                                         case["window"], case["last_n"])
        finally:
            vf.compute_block_score_varlen, vf._flash_block_sparse_varlen = orig_s, orig_a
        mk = cap["mk"].numpy()
        tot = sum(nbs)
        idx, cuo = cap["idx"].numpy(), cap["cu"].numpy()
        sels = []
        base = 0
        for si, NB in enumerate(nbs):
            sel = np.zeros((hq, NB, NB), bool)
            for h in range(hq):
                for qb in range(NB):
                    r = h * tot + base + qb
                    sel[h, qb, idx[cuo[r]:cuo[r + 1]]] = True
            sels.append(sel)
            base += NB
        out_packed = out.numpy()
    dt = time.time() - t0
    stride = case.get("out_stride", 5)
    rows = np.arange(0, out_packed.shape[0], stride)
    arrays = {
        "mk": mk.astype(np.float32),
        "out_rows": rows.astype(np.int64),
        "out": out_packed[rows].astype(np.float32),
    }
    for si, s in enumerate(sels):
        arrays[f"sel_bits_{si}"] = np.packbits(s.reshape(-1))
    meta = dict(case)
    meta["sha"] = input_sha(seqs)
    meta["nbs"] = nbs
    meta["interp_seconds"] = round(dt, 2)
    meta["generator"] = "flashprefill_b200.synthetic.make_sequence(L, hq, hk, 128, 500000.0, 0.01, seed0+i, fp32)"
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    return arrays, dt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of a reference checkout (contains ops/)")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    nf, vf = setup_reference(a.ref)
    for case in CASES:
        if a.only and case["name"] != a.only:
            continue
        arrays, dt = run_case(nf, vf, case)
        path = os.path.join(HERE, f"{case['name']}.npz")
        np.savez_compressed(path, **arrays)
        print(f"{case['name']}: {dt:.1f}s -> {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
