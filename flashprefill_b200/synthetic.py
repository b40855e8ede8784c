"""Seeded synthetic attention-layer inputs with the shapes and value structure of the
FlashPrefill benchmark configurations.

The reference evaluates on long-context suites (RULER, InfiniteBench, Video-MME) whose
data is not available here; these inputs stand in for them.  The recipe plants the
structures the block search is meant to find: a shared offset vector added to every
query and key row and rotated by RoPE (local/diagonal structure), four "sink" keys
scaled x8 and a random fraction of "heavy" keys scaled x4 (vertical structure).

Draw order per sequence (CPU ``torch.Generator`` seeded with ``seed``):
  q ~ N(0,1) (S,Hq,D); k ~ N(0,1) (S,Hk,D); v ~ N(0,1) (S,Hk,D); off = 2*N(0,1) (D,);
  q,k += off; RoPE (HF rotate-half, positions 0..S-1) on q and k; k[0:4] *= 8;
  k[randperm(S)[:round(f*S)]] *= 4; cast to the working dtype.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


def rope(x: torch.Tensor, base: float) -> torch.Tensor:
    """HF rotate-half RoPE on an (S, H, D) fp32 tensor, positions 0..S-1."""
    S, _, D = x.shape
    inv = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    pos = torch.arange(S, dtype=torch.float64)
    f = torch.outer(pos, inv)
    emb = torch.cat([f, f], -1)
    cos = emb.cos().float()[:, None, :]
    sin = emb.sin().float()[:, None, :]
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    return x * cos + torch.cat([-x2, x1], -1) * sin


def make_sequence(S: int, hq: int, hk: int, d: int = 128, rope_base: float = 500000.0,
                  heavy_frac: float = 0.01, seed: int = 0, dtype=torch.bfloat16):
    """One sequence of the seeded generator: returns q (S,hq,d), k (S,hk,d), v (S,hk,d)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(S, hq, d, generator=g)
    k = torch.randn(S, hk, d, generator=g)
    v = torch.randn(S, hk, d, generator=g)
    off = 2.0 * torch.randn(d, generator=g)
    q = rope(q + off, rope_base)
    k = rope(k + off, rope_base)
    k[:4] *= 8.0
    nh = int(round(heavy_frac * S))
    if nh > 0:
        idx = torch.randperm(S, generator=g)[:nh]
        k[idx] *= 4.0
    return q.to(dtype), k.to(dtype), v.to(dtype)


@dataclass
class Workload:
    """A named benchmark/parity configuration (one attention layer)."""
    name: str
    seqlens: list
    hq: int
    hk: int
    d: int = 128
    rope_base: float = 500000.0
    heavy_frac: float = 0.01
    alpha: float = 0.18
    dtype: torch.dtype = torch.bfloat16
    varlen: bool = False
    config_index: int = 0
    attention_sink: int = 2
    window_size: int = 4
    last_n_block: int = 2
    block_size: int = 128
    extra: dict = field(default_factory=dict)

    def seed(self, i: int) -> int:
        return self.config_index * 1000 + i

    def make(self):
        """Generate all sequences; returns lists of per-sequence (q, k, v)."""
        return [make_sequence(L, self.hq, self.hk, self.d, self.rope_base, self.heavy_frac,
                              self.seed(i), self.dtype) for i, L in enumerate(self.seqlens)]

    def make_dense(self):
        """(1,S,hq,d), (1,S,hk,d), (1,S,hk,d) for a single-sequence workload."""
        assert len(self.seqlens) == 1
        q, k, v = self.make()[0]
        return q[None], k[None], v[None]

    def make_packed(self):
        """Packed (T,h,d) tensors plus int32 cu_seqlens for a varlen workload."""
        seqs = self.make()
        q = torch.cat([s[0] for s in seqs])
        k = torch.cat([s[1] for s in seqs])
        v = torch.cat([s[2] for s in seqs])
        cu = torch.zeros(len(seqs) + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(torch.tensor(self.seqlens, dtype=torch.int64), 0).to(torch.int32)
        return q, k, v, cu


def workloads():
    """The BASELINE configurations (cfg0..cfg3) plus the 128K Llama-shaped headline layer."""
    return {
        "cfg0": Workload("cfg0_dense_4k_fp32", [4096], 4, 1, dtype=torch.float32, config_index=0),
        "cfg1": Workload("cfg1_llama3_8b_32k", [32768], 32, 8, config_index=1),
        "cfg2": Workload("cfg2_varlen_8k_16k_32k_64k", [8192, 16384, 32768, 65536], 32, 8,
                         varlen=True, config_index=2),
        "cfg3": Workload("cfg3_qwen2.5_7b_256k", [262144], 28, 4, rope_base=1e6, heavy_frac=0.005,
                         alpha=0.08, config_index=3),
        "l128k": Workload("llama3_8b_layer_128k", [131072], 32, 8, config_index=4),
    }


def causal_block_pairs(seqlens, block: int = 128) -> int:
    """P = sum over sequences of NB(NB+1)/2 causal (query-block, key-block) pairs, per head."""
    tot = 0
    for L in seqlens:
        nb = math.ceil(L / block)
        tot += nb * (nb + 1) // 2
    return tot
