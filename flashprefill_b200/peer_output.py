"""Full-output copies on every GPU of a head-sharded layer, written in place by each rank.

Each rank of a head-sharded layer computes the output of its own heads
(:mod:`flashprefill_b200.sharding`).  A caller that needs the whole (T, Hq, D) output on
every GPU would otherwise gather the head shards after the layer, e.g. with an NCCL
all-gather.  Instead, every rank holds a full output tensor, and the attention epilogue
writes each output tile into all of them (``fpb_prefill_dense_peers``).

This module maps the other ranks' output tensors into this process with CUDA IPC memory
handles: plain peer mappings over NVLink, no multicast object.  It uses the cuda-python
runtime bindings.  The ranks run on GPUs of one node, one process per GPU, in a
``torch.distributed`` process group.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _rt():
    from cuda.bindings import driver, runtime
    return runtime, driver


def _ok(res):
    err = res[0]
    if int(err) != 0:
        raise RuntimeError(f"CUDA call failed: {err}")
    return res[1:] if len(res) > 2 else (res[1] if len(res) == 2 else None)


class PeerOutputs:
    """Opens every other rank's copy of ``full`` (same shape, dtype and layout on each rank).

    ``peer_ptrs(offset_bytes)`` gives the device addresses, in this process, of the byte
    ``offset_bytes`` of every other rank's tensor (the rank's own slice of the output).
    ``close()`` unmaps them.  Collective: every rank of ``group`` calls the constructor.
    """

    def __init__(self, full: torch.Tensor, group=None):
        if not full.is_cuda or not full.is_contiguous():
            raise ValueError("full must be a contiguous CUDA tensor")
        rt, drv = _rt()
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        ptr = full.data_ptr()
        base, _size = _ok(drv.cuMemGetAddressRange(ptr))
        base = int(base)
        handle = _ok(rt.cudaIpcGetMemHandle(base))
        mine = (bytes(handle.reserved), ptr - base, full.numel() * full.element_size())
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        if any(e[2] != mine[2] for e in everyone):
            raise ValueError("the full output tensors differ in size across ranks")
        self._bases = {}
        self._offsets = {}
        for r, (hb, off, _n) in enumerate(everyone):
            if r == self.rank:
                continue
            h = rt.cudaIpcMemHandle_t()
            h.reserved = hb
            pbase = _ok(rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess))
            self._bases[r] = int(pbase)
            self._offsets[r] = off
        self.full = full

    def peer_ranks(self):
        return sorted(self._bases)

    def peer_ptrs(self, offset_bytes: int = 0):
        return [self._bases[r] + self._offsets[r] + offset_bytes for r in self.peer_ranks()]

    def close(self):
        rt, _ = _rt()
        for b in self._bases.values():
            _ok(rt.cudaIpcCloseMemHandle(b))
        self._bases.clear()
