"""vLLM backend shim: installation and dispatch (CPU; the sparse prefill and vLLM's own
forward are replaced by recorders, so no kernel runs).  Reference behaviour:
patches/patch_loader_vllm_0_12_0.py:47-253."""
import math
from types import SimpleNamespace

import pytest
import torch

fa = pytest.importorskip("vllm.v1.attention.backends.flash_attn")

from flashprefill_b200 import vllm_patch as vp  # noqa: E402


def _impl(**kw):
    d = dict(attn_type=fa.AttentionType.DECODER, dcp_world_size=1, kv_sharing_target_layer_name=None,
             sliding_window=(-1, -1), alibi_slopes=None, sinks=None, logits_soft_cap=None, head_size=128,
             scale=1.0 / math.sqrt(128), num_kv_heads=2)
    d.update(kw)
    return SimpleNamespace(**d)


def _common(q_lens, kv_lens, upper=None):
    """CommonAttentionMetadata stand-in with the host copies vLLM's scheduler provides."""
    qsl = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    return SimpleNamespace(num_reqs=len(q_lens), max_query_len=max(q_lens), query_start_loc_cpu=qsl,
                           seq_lens_cpu_upper_bound=torch.tensor(upper or kv_lens, dtype=torch.int32))


def _meta(q_lens, kv_lens, cascade=False, verdict="host"):
    qsl = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    m = SimpleNamespace(num_actual_tokens=int(sum(q_lens)), max_query_len=max(q_lens), query_start_loc=qsl,
                        max_seq_len=max(kv_lens), seq_lens=torch.tensor(kv_lens, dtype=torch.int32),
                        use_cascade=cascade)
    if verdict == "host":  # what the wrapped metadata builder attaches
        m.fp_whole_prefill = vp.whole_prefill_from_host(_common(q_lens, kv_lens))
    return m


@pytest.fixture
def patched(monkeypatch):
    calls = {"sparse": [], "orig": []}
    orig = fa.FlashAttentionImpl.forward

    def fake_orig(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                  output_block_scale=None):
        calls["orig"].append(attn_metadata)
        return output

    monkeypatch.setattr(fa.FlashAttentionImpl, "forward", fake_orig)
    monkeypatch.setattr(vp, "_prefill", lambda q, k, v, o, m, cfg: calls["sparse"].append((q, k, v, o, m, cfg)))
    vp.apply_patch_to_worker(config="flashprefill_qwen2")
    yield calls
    vp.remove_patch()
    assert fa.FlashAttentionImpl.forward is fake_orig
    monkeypatch.setattr(fa.FlashAttentionImpl, "forward", orig)


def _call(impl, meta, dtype=torch.bfloat16):
    T = meta.num_actual_tokens if meta is not None else 8
    q = torch.zeros(T + 3, 4, 128, dtype=dtype)  # padded past num_actual_tokens, as vLLM does
    k = torch.zeros(T + 3, 2, 128, dtype=dtype)
    out = torch.empty(T + 3, 4, 128, dtype=dtype)
    return fa.FlashAttentionImpl.forward(impl, None, q, k, k, None, meta, out)


def test_install_and_remove(patched):
    assert fa.FlashAttentionImpl.forward is vp._forward
    vp.apply_patch_to_worker(config="flashprefill_llama")  # idempotent, switches the config
    assert vp._state["cfg"]["alpha"] == 0.18
    with pytest.raises(ValueError):
        vp.apply_patch_to_worker(config={"block_size": 64, "alpha": 0.1})


def test_whole_prefills_go_sparse(patched):
    m = _meta([300, 129, 1000], [300, 129, 1000])
    _call(_impl(), m)
    assert len(patched["sparse"]) == 1 and not patched["orig"]
    q, k, v, o, meta, cfg = patched["sparse"][0]
    assert meta is m and cfg["alpha"] == 0.08 and o.shape == (m.num_actual_tokens + 3, 4, 128)


@pytest.mark.parametrize("case", ["decode", "prefix", "mixed", "cascade", "profiling", "no_verdict",
                                  "prefix_same_max"])
def test_other_batches_fall_back(patched, case):
    m = {"decode": _meta([1, 1], [500, 77]),
         "prefix": _meta([200], [700]),
         "mixed": _meta([1000, 1], [1000, 40]),
         "cascade": _meta([300, 300], [300, 300], cascade=True),
         "profiling": None,
         # metadata not made by the wrapped builder: no host verdict, so no sparse prefill
         "no_verdict": _meta([300], [300], verdict=None),
         # equal maxima, but the second sequence has a cached prefix (host check per sequence)
         "prefix_same_max": _meta([1000, 200], [1000, 700])}[case]
    _call(_impl(), m)
    assert not patched["sparse"] and len(patched["orig"]) == 1


def test_host_verdict():
    assert vp.whole_prefill_from_host(_common([300, 129], [300, 129])) is True
    assert vp.whole_prefill_from_host(_common([300, 1], [300, 40])) is False
    # an upper bound above the real length (async speculative decode) never passes as a prefill
    assert vp.whole_prefill_from_host(_common([300, 5], [300, 5], upper=[300, 9])) is False
    assert vp.whole_prefill_from_host(_common([1, 1], [1, 1])) is False  # max_query_len 1: decode
    assert vp.whole_prefill_from_host(SimpleNamespace(num_reqs=1, max_query_len=4)) is None


def test_builder_wrapper_attaches_the_verdict(patched, monkeypatch):
    made = SimpleNamespace()
    monkeypatch.setitem(vp._state, "original_build", lambda self, cpl, common, *a, **kw: made)
    md = vp._build(None, 0, _common([300], [300]))
    assert md is made and md.fp_whole_prefill is True
    md = vp._build(None, 0, _common([300], [700]))
    assert md.fp_whole_prefill is False


def test_capture_falls_back(patched, monkeypatch):
    """A batch traced while a CUDA graph is being captured keeps vLLM's own forward."""
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    _call(_impl(), _meta([300], [300]))
    assert not patched["sparse"] and len(patched["orig"]) == 1


def test_no_device_reads_in_dispatch():
    """The dispatch path holds no .item() / bool(tensor) host syncs on device data."""
    import inspect
    src = inspect.getsource(vp._whole_prefills) + inspect.getsource(vp._forward)
    assert ".item()" not in src and ".all()" not in src


@pytest.mark.parametrize("kw", [dict(sliding_window=(1023, 0)), dict(alibi_slopes=torch.zeros(4)),
                                dict(logits_soft_cap=30.0), dict(sinks=torch.zeros(4)), dict(head_size=64),
                                dict(scale=0.5), dict(dcp_world_size=2),
                                dict(kv_sharing_target_layer_name="model.layers.0.attn")])
def test_unsupported_layers_fall_back(patched, kw):
    _call(_impl(**kw), _meta([300], [300]))
    assert not patched["sparse"] and len(patched["orig"]) == 1


def test_fp32_falls_back(patched):
    _call(_impl(), _meta([300], [300]), dtype=torch.float32)
    assert not patched["sparse"] and len(patched["orig"]) == 1


@pytest.mark.gpu
def test_patched_forward_runs_the_sparse_prefill_on_gpu():
    """Through vLLM's FlashAttentionImpl.forward (patched), a whole-prefill batch gives exactly
    what flash_prefill_varlen_func gives on the same tensors."""
    import flashprefill_b200 as fp
    from tests import gpu_util as gu

    lens = [700, 1500]
    q, k, v, cu = gu.make_packed(lens, 4, 2, torch.bfloat16, seed0=5)
    dev = torch.device("cuda:0")
    q, k, v = q.to(dev), k.to(dev), v.to(dev)
    meta = _meta(lens, lens)
    meta.query_start_loc = meta.query_start_loc.to(dev)
    meta.seq_lens = meta.seq_lens.to(dev)
    out = torch.empty_like(q)
    vp.apply_patch_to_worker(config="flashprefill_llama")
    try:
        before = vp.stats()["sparse_prefill"]
        fa.FlashAttentionImpl.forward(_impl(), None, q, k, v, None, meta, out)
        assert vp.stats()["sparse_prefill"] == before + 1
    finally:
        vp.remove_patch()
    ref = torch.empty_like(q)
    fp.flash_prefill_varlen_func(q, k, v, ref, meta.query_start_loc, max(lens), 0.18, 128, 2, 4, 2)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
