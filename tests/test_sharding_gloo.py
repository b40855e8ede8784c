"""Head sharding across two ranks (gloo, CPU): each rank runs the CPU restatement of the
operator on its KV-head group of the same layer; the gathered per-rank outputs and block sets
must equal the unsharded run exactly (the path has no cross-head dependency, so bench.py's
multi-GPU layout needs no collective on the data path)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashprefill_b200.sharding import head_shard
from flashprefill_b200.synthetic import make_sequence
from oracle import restate

S, HQ, HK = 640, 8, 4
ARGS = dict(dt="bf16", alpha=0.18, sink=2, window=4, last_n=2, dense=True)


def _inputs():
    q, k, v = make_sequence(S, HQ, HK, seed=11)
    return q.float().numpy(), k.float().numpy(), v.float().numpy()


def _rank_main(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, k, v = _inputs()
    hk0, hk1, hq0, hq1 = head_shard(HQ, HK, rank, world)
    cu = np.array([0, S])
    out, res = restate.prefill(q[:, hq0:hq1], k[:, hk0:hk1], v[:, hk0:hk1], cu, hq1 - hq0, hk1 - hk0, **ARGS)
    sel = torch.from_numpy(res["sel"][0].astype(np.uint8))
    o = torch.from_numpy(np.ascontiguousarray(out))
    outs = [torch.empty_like(o) for _ in range(world)]
    sels = [torch.empty_like(sel) for _ in range(world)]
    dist.all_gather(outs, o)
    dist.all_gather(sels, sel)
    if rank == 0:
        np.save(os.path.join(outdir, "out.npy"), torch.cat(outs, dim=1).numpy())
        np.save(os.path.join(outdir, "sel.npy"), torch.cat(sels, dim=0).numpy())
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_shard_ranges():
    assert head_shard(32, 8, 0, 8) == (0, 1, 0, 4)
    assert head_shard(32, 8, 3, 4) == (6, 8, 24, 32)
    with pytest.raises(ValueError):
        head_shard(32, 8, 0, 3)


def test_two_rank_shards_equal_unsharded(tmp_path):
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    q, k, v = _inputs()
    out, res = restate.prefill(q, k, v, np.array([0, S]), HQ, HK, **ARGS)
    np.testing.assert_array_equal(np.load(tmp_path / "sel.npy").astype(bool), res["sel"][0])
    np.testing.assert_array_equal(np.load(tmp_path / "out.npy"), out)
