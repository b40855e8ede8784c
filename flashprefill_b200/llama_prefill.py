"""End-to-end prefill of a Llama-3-8B-architecture model with FlashPrefill attention in every layer.

The reference applies FlashPrefill inside HF / vLLM Llama models (ruler/models/llama.py:260-334:
the attention layer projects q/k/v, applies RoPE, and calls ``flash_prefill`` on (B, S, H, D)
tensors during prefill).  This module is that caller for one process per GPU with tensor
parallelism over the attention heads and the MLP (Megatron-style):

* q/k/v projection column-parallel: rank r owns KV heads [r*Hk/N, (r+1)*Hk/N) and their query
  heads, so its attention call needs no exchange (the operator shards by KV-head group);
* o_proj row-parallel, followed by one all-reduce of the hidden state;
* MLP gate/up column-parallel, down row-parallel, followed by one all-reduce;
* embedding, norms and the LM head replicated; only the last position's logits are produced.

Weights are random (normal, std 0.02, bf16) and seeded per matrix, so every rank holds exactly its
slice of one and the same full model for any number of ranks.  The GEMMs run on cuBLAS through
torch (plain library GEMMs); the attention runs the library's CUDA kernels; RMSNorm, RoPE and SiLU
are torch element-wise ops.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class LlamaConfig:
    """Llama-3-8B: 32 layers, hidden 4096, 32 query / 8 KV heads of 128, SwiGLU FFN 14336,
    RMSNorm eps 1e-5, RoPE base 500000, vocabulary 128256."""
    layers: int = 32
    hidden: int = 4096
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_base: float = 500000.0
    eps: float = 1e-5
    init_std: float = 0.02
    # FlashPrefill selection parameters for Llama models (patches/patch_loader_vllm_0_12_0.py:17-24)
    alpha: float = 0.18
    attention_sink: int = 2
    window: int = 4
    last_n: int = 2


def _seeded_normal(shape, seed, std, device, dtype):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def rope_tables(S: int, d: int, base: float, device):
    inv = 1.0 / (base ** (torch.arange(0, d, 2, device=device, dtype=torch.float64) / d))
    f = torch.outer(torch.arange(S, device=device, dtype=torch.float64), inv)
    emb = torch.cat([f, f], -1)
    return emb.cos().float(), emb.sin().float()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """HF rotate-half RoPE on (S, H, D), computed in fp32, returned in x's dtype."""
    d = x.shape[-1]
    xf = x.float()
    x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
    return (xf * cos[:, None] + torch.cat([-x2, x1], -1) * sin[:, None]).to(x.dtype)


class TPLlamaPrefill:
    """One rank's shard of the model.  ``attention(q, k, v, out, cfg)`` runs the attention of
    one layer on (1, S, H, D) tensors; by default the library's ``flash_prefill``."""

    def __init__(self, cfg: LlamaConfig, rank: int = 0, world: int = 1, device="cuda", dtype=torch.bfloat16,
                 seed: int = 0, attention=None, all_reduce=None):
        if cfg.kv_heads % world or cfg.ffn % world:
            raise ValueError(f"{world} ranks do not divide {cfg.kv_heads} KV heads and FFN {cfg.ffn}")
        self.cfg, self.rank, self.world = cfg, rank, world
        self.device, self.dtype = torch.device(device), dtype
        self.attention = attention or _flash_prefill_attention
        self.all_reduce = all_reduce
        G = cfg.q_heads // cfg.kv_heads
        self.hk_l = cfg.kv_heads // world
        self.hq_l = self.hk_l * G
        self.f_l = cfg.ffn // world
        H, D = cfg.hidden, cfg.head_dim
        mk = lambda shape, s: _seeded_normal(shape, seed * 1_000_003 + s, cfg.init_std, self.device, dtype)
        hq0, hk0 = rank * self.hq_l, rank * self.hk_l
        self.embed = mk((cfg.vocab, H), 1)
        self.lm_head = mk((cfg.vocab, H), 2)
        self.final_norm = torch.ones(H, device=self.device, dtype=dtype)
        self.layers = []
        for i in range(cfg.layers):
            base = 100 + 10 * i
            wq = mk((cfg.q_heads * D, H), base)[hq0 * D:(hq0 + self.hq_l) * D]
            wk = mk((cfg.kv_heads * D, H), base + 1)[hk0 * D:(hk0 + self.hk_l) * D]
            wv = mk((cfg.kv_heads * D, H), base + 2)[hk0 * D:(hk0 + self.hk_l) * D]
            wo = mk((H, cfg.q_heads * D), base + 3)[:, hq0 * D:(hq0 + self.hq_l) * D]
            wg = mk((cfg.ffn, H), base + 4)[rank * self.f_l:(rank + 1) * self.f_l]
            wu = mk((cfg.ffn, H), base + 5)[rank * self.f_l:(rank + 1) * self.f_l]
            wd = mk((H, cfg.ffn), base + 6)[:, rank * self.f_l:(rank + 1) * self.f_l]
            self.layers.append({
                "attn_norm": torch.ones(H, device=self.device, dtype=dtype),
                "mlp_norm": torch.ones(H, device=self.device, dtype=dtype),
                "wqkv": torch.cat([wq, wk, wv]).contiguous(),
                "wo": wo.contiguous(),
                "wgu": torch.cat([wg, wu]).contiguous(),
                "wd": wd.contiguous(),
            })
            del wq, wk, wv, wo, wg, wu, wd
        torch.cuda.empty_cache() if self.device.type == "cuda" else None

    def _reduce(self, x):
        if self.world > 1:
            (self.all_reduce or torch.distributed.all_reduce)(x)
        return x

    @torch.no_grad()
    def forward(self, tokens: torch.Tensor, events=None) -> torch.Tensor:
        """Prefill of one sequence of token ids (S,); returns the last position's logits (vocab,)
        in fp32.  ``events``: optional list that receives (start, end) CUDA event pairs around
        every attention call."""
        cfg = self.cfg
        S, D = tokens.shape[0], cfg.head_dim
        cos, sin = rope_tables(S, D, cfg.rope_base, self.device)
        x = self.embed[tokens]
        nq, nk = self.hq_l * D, self.hk_l * D
        attn = torch.empty(1, S, self.hq_l, D, device=self.device, dtype=self.dtype)
        for L in self.layers:
            h = rms_norm(x, L["attn_norm"], cfg.eps)
            qkv = h @ L["wqkv"].t()
            q = apply_rope(qkv[:, :nq].view(S, self.hq_l, D), cos, sin)
            k = apply_rope(qkv[:, nq:nq + nk].view(S, self.hk_l, D), cos, sin)
            v = qkv[:, nq + nk:].view(S, self.hk_l, D)
            del qkv
            if events is not None:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            self.attention(q[None], k[None], v[None], attn, cfg)
            if events is not None:
                e1.record()
                events.append((e0, e1))
            del q, k, v
            o = attn.view(S, nq) @ L["wo"].t()
            x = x + self._reduce(o)
            del o
            h = rms_norm(x, L["mlp_norm"], cfg.eps)
            gu = h @ L["wgu"].t()
            a = torch.nn.functional.silu(gu[:, :self.f_l]) * gu[:, self.f_l:]
            del gu
            y = a @ L["wd"].t()
            del a
            x = x + self._reduce(y)
            del y
        last = rms_norm(x[-1:], self.final_norm, cfg.eps)
        return (last.float() @ self.lm_head.float().t())[0]


def _flash_prefill_attention(q, k, v, out, cfg: LlamaConfig):
    from .flashprefill_native_forward import flash_prefill
    flash_prefill(q, k, v, out, 128, cfg.attention_sink, cfg.window, cfg.alpha, cfg.last_n, 0)


def prefill_flops(cfg: LlamaConfig, S: int) -> float:
    """GEMM FLOPs of one prefill of S tokens (projections, MLP and the last-token LM head)."""
    H, D = cfg.hidden, cfg.head_dim
    per_layer = 2 * S * H * ((cfg.q_heads + 2 * cfg.kv_heads) * D + cfg.q_heads * D + 3 * cfg.ffn)
    return cfg.layers * per_layer + 2 * H * cfg.vocab


def _check_world(cfg: LlamaConfig, world: int) -> None:
    if world < 1 or cfg.kv_heads % world:
        raise ValueError(f"tensor parallelism over {world} ranks needs a divisor of {cfg.kv_heads}")
    if math.gcd(cfg.ffn, world) != world:
        raise ValueError(f"FFN {cfg.ffn} does not split over {world} ranks")
