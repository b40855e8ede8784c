"""The reference's own kernels on the CPU (Triton interpreter), timed on one whole layer.

TEST INFRASTRUCTURE ONLY: bench.py runs this file in a subprocess as its timed CPU baseline of
kind "reference".  The reference (qhfan/FlashPrefill ``ops/``, staged unmodified by
oracle/stage_ref.py) has no CPU path of its own; its Triton kernels run on the host under
``TRITON_INTERPRET=1`` in fp32, which is BASELINE configs[0] (S=4096, 4 query / 1 KV head,
D=128, alpha 0.18, sink 2, window 4, last_n 2).  Shims needed only because no GPU driver is
used: fla's device context becomes a null context, every autotuner keeps one configuration
(the score kernel the widest key tile, so that every score of a row is computed) and
torch.compile is disabled (the reference's two compiled helpers run eagerly).

    python oracle/interp_ref.py [--seq 4096] [--hq 4] [--hk 1]

Prints one JSON line: {"seconds": ..., "threads": ..., "selected_blocks": ...}.
"""
from __future__ import annotations

import os

os.environ["TRITON_INTERPRET"] = "1"
os.environ["TORCHDYNAMO_DISABLE"] = "1"
os.environ.setdefault("CUDA_VISIBLE_DEVICES", "")

import argparse  # noqa: E402
import contextlib  # noqa: E402
import json  # noqa: E402
import sys  # noqa: E402
import time  # noqa: E402
import warnings  # noqa: E402

warnings.filterwarnings("ignore")

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--hq", type=int, default=4)
    ap.add_argument("--hk", type=int, default=1)
    ap.add_argument("--alpha", type=float, default=0.18)
    a = ap.parse_args()

    import torch
    import fla.utils as fu
    fu.custom_device_ctx = lambda i: contextlib.nullcontext()
    from triton.runtime.autotuner import Autotuner

    from flashprefill_b200.synthetic import make_sequence
    from oracle import triton_ref

    nf, _ = triton_ref.load()
    for n in dir(nf):
        obj = getattr(nf, n)
        if isinstance(obj, Autotuner):
            if n.startswith("compute_block_score"):
                obj.configs = [max(obj.configs, key=lambda c: c.kwargs.get("K_TILE_SIZE", 0))]
            else:
                obj.configs = [obj.configs[0]]
    q, k, v = make_sequence(a.seq, a.hq, a.hk, 128, 500000.0, 0.01, 0, torch.float32)
    q, k, v = q[None], k[None], v[None]
    out = torch.zeros_like(q)
    t0 = time.perf_counter()
    st = triton_ref.run_dense(q, k, v, out, 128, 2, 4, a.alpha, 2, 0)
    dt = time.perf_counter() - t0
    print(json.dumps({"seconds": round(dt, 3), "threads": torch.get_num_threads(),
                      "selected_blocks": int(st["counts"].sum()), "seq": a.seq, "hq": a.hq, "hk": a.hk}))


if __name__ == "__main__":
    main()
