"""End-to-end Llama prefill harness (flashprefill_b200.llama_prefill): tensor-parallel sharding
on CPU ranks (gloo) equals the unsharded model, and on the GPU the model with FlashPrefill
attention at alpha = 0 (every causal block selected) matches the same model with dense causal
attention."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashprefill_b200.llama_prefill import LlamaConfig, TPLlamaPrefill, prefill_flops

SMALL = dict(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=128, ffn=512, vocab=1000)


def dense_causal(q, k, v, out, cfg):
    """Reference attention for the tests: dense causal GQA in fp32 (1, S, H, D)."""
    G = q.shape[2] // k.shape[2]
    qf = q[0].float().transpose(0, 1)
    kf = k[0].float().repeat_interleave(G, 1).transpose(0, 1)
    vf = v[0].float().repeat_interleave(G, 1).transpose(0, 1)
    o = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=True)
    out[0].copy_(o.transpose(0, 1).to(out.dtype))


def _rank(rank, world, port, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = LlamaConfig(**SMALL)
    m = TPLlamaPrefill(cfg, rank, world, device="cpu", dtype=torch.float32, seed=3, attention=dense_causal)
    tokens = torch.randint(0, cfg.vocab, (300,), generator=torch.Generator().manual_seed(1))
    logits = m.forward(tokens)
    if rank == 0:
        torch.save(logits, path)
    dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_tensor_parallel_equals_one_rank(tmp_path):
    cfg = LlamaConfig(**SMALL)
    m = TPLlamaPrefill(cfg, 0, 1, device="cpu", dtype=torch.float32, seed=3, attention=dense_causal)
    tokens = torch.randint(0, cfg.vocab, (300,), generator=torch.Generator().manual_seed(1))
    ref = m.forward(tokens)
    path = str(tmp_path / "logits.pt")
    mp.spawn(_rank, args=(2, _port(), path), nprocs=2, join=True)
    got = torch.load(path)
    assert torch.allclose(got, ref, atol=1e-4, rtol=1e-4), (got - ref).abs().max()


def test_shards_are_slices_of_one_model():
    cfg = LlamaConfig(**SMALL)
    full = TPLlamaPrefill(cfg, 0, 1, device="cpu", dtype=torch.float32, seed=5, attention=dense_causal)
    half = TPLlamaPrefill(cfg, 1, 2, device="cpu", dtype=torch.float32, seed=5, attention=dense_causal)
    D = cfg.head_dim
    assert torch.equal(half.layers[0]["wo"], full.layers[0]["wo"][:, 2 * D:4 * D])
    assert torch.equal(half.layers[1]["wd"], full.layers[1]["wd"][:, 256:512])
    assert prefill_flops(LlamaConfig(), 131072) > 1e15


@pytest.mark.gpu
def test_flashprefill_full_mask_matches_dense_attention_model():
    cfg = LlamaConfig(layers=2, hidden=1024, q_heads=8, kv_heads=2, head_dim=128, ffn=2048, vocab=4096, alpha=0.0)
    dev = "cuda:0"
    tokens = torch.randint(0, cfg.vocab, (2048,), generator=torch.Generator().manual_seed(2)).to(dev)
    m = TPLlamaPrefill(cfg, 0, 1, device=dev, seed=7)
    got = m.forward(tokens)
    m.attention = dense_causal
    ref = m.forward(tokens)
    torch.cuda.synchronize()
    err = (got - ref).abs().max().item() / ref.abs().max().item()
    assert err < 2e-2, err
