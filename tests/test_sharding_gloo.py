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

from flashprefill_b200.sharding import head_shard, layer_shard, row_ranges, row_work
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


def _rank_main_2d(rank, world, port, outdir):
    """2-D split: HK2 KV heads over `world` ranks, each KV group cut into query-block ranges.
    Each rank produces only the rows of its range for its heads; rank 0 assembles them."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, k, v = _inputs2()
    nb = (S + 127) // 128
    hk0, hk1, hq0, hq1, qb0, qb1 = layer_shard(HQ2, HK2, nb, rank, world)
    cu = np.array([0, S])
    out, res = restate.prefill(q[:, hq0:hq1], k[:, hk0:hk1], v[:, hk0:hk1], cu, hq1 - hq0, hk1 - hk0, **ARGS)
    piece = np.full((S, HQ2, 128), np.nan, np.float32)
    r0, r1 = qb0 * 128, min(S, qb1 * 128)
    piece[r0:r1, hq0:hq1] = out[r0:r1]
    sel = np.zeros((HQ2, nb, nb), np.uint8)
    sel[hq0:hq1, qb0:qb1] = res["sel"][0][:, qb0:qb1]
    pieces = [torch.empty(S, HQ2, 128) for _ in range(world)]
    sels = [torch.empty(HQ2, nb, nb, dtype=torch.uint8) for _ in range(world)]
    dist.all_gather(pieces, torch.from_numpy(piece))
    dist.all_gather(sels, torch.from_numpy(sel))
    if rank == 0:
        full = torch.stack(pieces).nan_to_num(0.0).sum(0)
        covered = sum((~torch.isnan(p)).int() for p in pieces)
        np.save(os.path.join(outdir, "out2d.npy"), full.numpy())
        np.save(os.path.join(outdir, "cover2d.npy"), covered.numpy())
        np.save(os.path.join(outdir, "sel2d.npy"), torch.stack(sels).sum(0).numpy())
    dist.destroy_process_group()


HQ2, HK2 = 4, 2


def _inputs2():
    q, k, v = make_sequence(S, HQ2, HK2, seed=12)
    return q.float().numpy(), k.float().numpy(), v.float().numpy()


def test_row_ranges_balance_and_partition():
    for nb, parts in [(2048, 2), (1024, 2), (157, 3), (5, 5)]:
        b = row_ranges(nb, parts)
        assert b[0] == 0 and b[-1] == nb and all(x < y for x, y in zip(b, b[1:])) and len(b) == parts + 1
    w = row_work(2048)
    b = row_ranges(2048, 2)
    assert abs(sum(w[:b[1]]) - sum(w[b[1]:])) <= max(w)
    # Qwen2.5-7B-shaped layer (4 KV heads) over 8 GPUs: 4 groups x 2 query-block ranges
    shards = [layer_shard(28, 4, 2048, r, 8) for r in range(8)]
    assert [s_[:4] for s_ in shards[:2]] == [(0, 1, 0, 7)] * 2
    assert shards[0][4:] == (0, b[1]) and shards[1][4:] == (b[1], 2048)
    assert layer_shard(32, 8, 1024, 5, 8) == (5, 6, 20, 24, 0, 1024)
    with pytest.raises(ValueError):
        layer_shard(28, 4, 2048, 0, 6)


def test_four_rank_2d_split_equals_unsharded(tmp_path):
    """2 KV heads over 4 ranks: each rank one KV head and half of its query blocks."""
    world = 4
    mp.spawn(_rank_main_2d, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    q, k, v = _inputs2()
    out, res = restate.prefill(q, k, v, np.array([0, S]), HQ2, HK2, **ARGS)
    assert (np.load(tmp_path / "cover2d.npy") == 1).all(), "every output element written by exactly one rank"
    np.testing.assert_array_equal(np.load(tmp_path / "sel2d.npy").astype(bool), res["sel"][0])
    np.testing.assert_array_equal(np.load(tmp_path / "out2d.npy"), out)
