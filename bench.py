"""Benchmark of the sparse-prefill operator on B200 (one attention layer per step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload l128k|cfg1|cfg2|cfg3]
                    [--impl ours|reference]

Default workload: the 128K-token Llama-3-8B-shaped layer the headline metric is quoted on
(S=131072, 32 query / 8 KV heads, head_dim 128, bf16, alpha 0.18, sink 2, window 4,
last_n 2).  Under torchrun (N>1) every rank generates the same seeded layer and keeps a
contiguous group of KV heads (and their query heads) -- heads shard with no cross-GPU
dependency -- so total work is fixed and the reported ms/layer is the max over ranks
("scaling": "strong").

Timed region (``value``): K steps of the operator on inputs already in HBM (1.6 GB at
128K, larger than the 126 MB L2, so no extra flush), CUDA events on the launching stream,
barrier + synchronize on both sides, max over ranks.  ``e2e``: the same step through the
public API ``flash_prefill`` with the inputs copied from pinned host memory and the output
copied back inside the timed region.  ``roofline``: the attention kernel (dominant) against
the measured dense bf16 peak; ``roofline_search``: the search stage against measured HBM
bandwidth.

Baselines (rank 0, N=1), none of them on the product path:
  ``triton_baseline``: the reference's own Triton implementation (qhfan/FlashPrefill ops/,
      staged unmodified by oracle/stage_ref.py) on this GPU, same inputs, autotune warmed;
      with the comparison of its block masks and pooled keys with ours;
  ``cpu_baseline``: the CPU restatement (oracle) on a bounded sample of the same layer,
      extrapolated to the whole layer;
  ``cpu_baseline_interpreter``: the reference's own kernels under the Triton interpreter on
      the host, one complete BASELINE configs[0] layer (fp32, S=4096), not extrapolated.

``--impl reference``: the reference has no CPU implementation of its own (its Triton kernels
run on the host only through the interpreter, far too slowly for this layer), so this arm
times the CPU restatement of the reference algorithm (``oracle/``) with every host thread on
a bounded sample of the same layer, extrapolated to ms/layer (``"extrapolated": true``).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sparse-prefill attn ms/layer @128K on 1/8 B200; TC util; mask exactness"
UNIT = "ms/layer"
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu capture of
# each kernel on the full single-GPU workload (1 pass; the commands and figures are in
# profiles/dram_traffic.md and profiles/sparse_attn2_cfg1_full.md: sparse_attn2_kernel and
# block_search_persistent_kernel).  Reported as roofline traffic for those workloads on one GPU
# with all heads; other runs (shards, N > 1, other workloads) report null.
NCU_TRAFFIC = {
    "llama3_8b_layer_128k": {"attention": 2139156224 + 1015631104,
                             "search": 1074930688 + 4879104},
    "cfg1_llama3_8b_32k": {"attention": 504537344 + 221985536,
                           "search": 267095552 + 3992320},
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [v for v in (num(r[1]) for r in rows) if v is not None]
        mx = [v for v in (num(r[2]) for r in rows) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        load = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------- workloads
def workload(name):
    from flashprefill_b200.synthetic import workloads
    return workloads()[name]


def device_inputs(w, hk0, hk1, device, seed):
    """Inputs of KV heads [hk0, hk1) (and their query heads), generated on the device with
    the recipe of flashprefill_b200.synthetic (same distribution, device RNG)."""
    import torch
    G = w.hq // w.hk
    nh_q, nh_k = (hk1 - hk0) * G, hk1 - hk0
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    T = sum(w.seqlens)
    D = w.d
    q = torch.randn(T, nh_q, D, device=device, generator=g)
    k = torch.randn(T, nh_k, D, device=device, generator=g)
    v = torch.randn(T, nh_k, D, device=device, generator=g)
    gc = torch.Generator(device=device)
    gc.manual_seed(w.config_index * 1000 + 17)  # offset vector shared by every head and rank
    off = 2.0 * torch.randn(D, device=device, generator=gc)
    inv = 1.0 / (w.rope_base ** (torch.arange(0, D, 2, device=device, dtype=torch.float64) / D))
    a = 0
    for L in w.seqlens:
        b = a + L
        pos = torch.arange(L, device=device, dtype=torch.float64)
        f = torch.outer(pos, inv)
        emb = torch.cat([f, f], -1)
        cos, sin = emb.cos().float()[:, None, :], emb.sin().float()[:, None, :]
        for t in (q, k):
            x = t[a:b] + off
            x1, x2 = x[..., : D // 2], x[..., D // 2:]
            t[a:b] = x * cos + torch.cat([-x2, x1], -1) * sin
        k[a:a + 4] *= 8.0
        nh = int(round(w.heavy_frac * L))
        if nh:
            idx = torch.randperm(L, device=device, generator=g)[:nh] + a
            k[idx] *= 4.0
        a = b
    return q.to(w.dtype), k.to(w.dtype), v.to(w.dtype)


def algorithmic(w, hq, hk, E):
    """Algorithmic bytes of the search and FLOPs of search / attention for hq/hk local heads."""
    T = sum(w.seqlens)
    D = w.d
    nbs = [math.ceil(L / 128) for L in w.seqlens]
    search_bytes = 2 * (T * hq * D + T * hk * D) + 4 * E + 4 * hq * sum(nbs)
    attn_flops = E * 4 * 128 * 128 * D
    search_flops = hq * sum(nb * (nb + 1) // 2 for nb in nbs) * 2 * 128 * D
    return search_bytes, attn_flops, search_flops


# --------------------------------------------------------------------------- CPU arm
def split_plan_runs_dense(seqlen, hq, cap, sms, sink=2, window=4, last_n=2):
    """Whether fpb_prefill_dense runs the long-row split plan: it skips it when even a
    full-length row is within the split threshold (1.2x the listed blocks per attention
    pipeline) for the fewest blocks the search can list (its structural blocks)."""
    nb = -(-seqlen // 128)
    if cap <= 64:
        return False
    lb = 0
    for qb in range(nb):
        if qb >= nb - last_n:
            lb += qb + 1
        else:
            s_end, w_lo = min(sink, qb + 1), max(0, qb - window + 1)
            lb += s_end + (qb + 1 - w_lo) - max(0, s_end - w_lo)
    grid = min(sms, nb * hq)
    return not (min(cap, nb) * 5 * 2 * grid <= lb * hq * 6)


def cpu_sample(w, seconds_budget=20.0):
    """Time the CPU restatement on a bounded sample of the layer and extrapolate.

    Sample: KV head 0 with its query heads of the longest sequence; pooled keys for the
    whole sequence; search on random query blocks of head 0; attention on the selected
    block pairs of those rows.  Search time scales with the number of (head, query block)
    rows of the layer, attention time with the executed block pairs (estimated from the
    sampled rows' density).  Returns (ms_per_layer, info)."""
    import numpy as np
    import torch

    from flashprefill_b200.synthetic import make_sequence
    from oracle import restate

    L = max(w.seqlens)
    G = w.hq // w.hk
    q, k, v = make_sequence(L, G, 1, w.d, w.rope_base, w.heavy_frac, w.seed(0), torch.bfloat16)
    f = lambda t: t.float().numpy()
    qn, kn, vn = f(q), f(k), f(v)
    nb = math.ceil(L / 128)
    cu = np.array([0, L])
    t0 = time.perf_counter()
    mk = restate.block_mean(kn, cu, "bf16", "tw4")
    t_mean = time.perf_counter() - t0
    c = restate.scale_log2(w.d)
    qpad = np.zeros((nb * 128, G, w.d), np.float32)
    qpad[:L] = qn
    order = np.random.default_rng(0).permutation(nb)
    done, t_search, sel_rows, near_rows = 0, 0.0, {}, {}
    while done < nb and t_search < seconds_budget * 0.5:
        chunk = sorted(order[done:done + 16].tolist())
        t1 = time.perf_counter()
        m, p = restate.block_scores_head(qpad[:, 0], mk[:, 0], nb, c, chunk)
        for qb in chunk:
            s_, score, thr = restate.select_row(m[qb, :qb + 1], p[qb, :qb + 1], qb, nb, w.alpha, 2, 4, 2, True)
            sel_rows[qb] = s_
            near_rows[qb] = np.abs(score - thr) <= 1e-3 * abs(thr)
        t_search += time.perf_counter() - t1
        done += len(chunk)
    sel = np.zeros((1, nb, nb), bool)
    for qb, s_ in sel_rows.items():
        sel[0, qb] = s_
    pairs, t_attn = 0, 0.0
    for qb in sorted(sel_rows):
        if t_attn > seconds_budget * 0.5:
            break
        t1 = time.perf_counter()
        restate.sparse_attention(qn[:, :1], kn, vn, cu, [sel], 1, 1, rows={(0, 0, qb)})
        t_attn += time.perf_counter() - t1
        pairs += int(sel[0, qb].sum())
    dens = sum(int(s.sum()) for s in sel_rows.values()) / max(1, done)
    total_rows = w.hq * sum(math.ceil(x / 128) for x in w.seqlens)
    E_est = dens * total_rows
    ms = 1e3 * (t_mean * w.hk * (sum(w.seqlens) / L) + t_search / done * total_rows
                + (t_attn / max(1, pairs)) * E_est)
    info = {"sample_seconds": t_mean + t_search + t_attn,
            "sample": f"KV head 0 + its {G} query heads of one {L}-token sequence: pooled keys of all {nb} "
                      f"blocks, search on {done} random query blocks of one head, attention on {pairs} block "
                      f"pairs; extrapolated to {total_rows} (head, block) rows and E~{int(E_est)} pairs",
            "cores": os.cpu_count(),
            "mask_sample": (q, k, sel_rows, near_rows)}
    return ms, info


def mask_exactness(w, sample, dev):
    """Block sets of the GPU search against the CPU restatement on the sampled rows (same
    inputs): rows compared, selected blocks, flips inside the 1e-3 threshold band, other flips."""
    import numpy as np

    import flashprefill_b200 as fp

    q, k, sel_rows, near_rows = sample
    qd, kd = q.to(dev), k.to(dev)
    cnt, idx, _, _ = fp.search_dense(qd[None], kd[None], 128, 2, 4, w.alpha, 2, 0)
    cnt, idx = cnt.cpu().numpy(), idx.cpu().numpy()
    nb = idx.shape[2]
    near = other = blocks = 0
    for qb, ref in sel_rows.items():
        got = np.zeros(nb, bool)
        got[idx[0, qb, :cnt[0, qb]]] = True
        diff = got ^ ref
        near += int((diff & near_rows[qb]).sum())
        other += int((diff & ~near_rows[qb]).sum())
        blocks += int(ref.sum())
    return {"rows": len(sel_rows), "blocks_selected": blocks, "near_threshold_flips": near, "other_flips": other,
            "sample": "the CPU baseline's rows (query head 0 of KV head 0, one sequence, same inputs)"}


def triton_baseline(w, q, k, v, cu, maxlen, ws, L, steps, ours_ms):
    """Time the reference's Triton path (qhfan/FlashPrefill ops/, staged unmodified by
    oracle/stage_ref.py) on this GPU on the same inputs, and compare its block masks with the
    lists our last search left in ``ws``.  Not part of the product path."""
    import torch

    try:
        from oracle import triton_ref as tr
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"import failed: {e}"}
    if not tr.available():
        return {"unavailable": "reference sources not staged (oracle/stage_ref.py) or triton/fla missing"}
    from flashprefill_b200 import _ops
    hq, hk = q.shape[1], k.shape[1]
    cnt = ws[L["cnt"]:L["cnt"] + 4 * hq * L["tiles"]].view(torch.int32).view(hq, L["tiles"])
    idx = ws[L["idx"]:L["idx"] + 4 * hq * L["tiles"] * L["cap"]].view(torch.int32).view(hq, L["tiles"], L["cap"])
    ref_out = torch.zeros_like(q)
    t0 = time.perf_counter()
    if w.varlen:
        call = lambda: tr.flash_prefill_varlen_func(q, k, v, ref_out, cu, maxlen, w.alpha, 128, 2, 4, 2)
        st = tr.run_varlen(q, k, v, ref_out, cu, maxlen, w.alpha, 128, 2, 4, 2)
        mk = ws[L["mk"]:L["mk"] + 2 * st["mk"].numel()].view(q.dtype).view(st["mk"].shape)
        rep = tr.varlen_mask_diff(st, cnt, idx, w.seqlens, w.alpha)
    else:
        q4, k4, v4, o4 = q[None], k[None], v[None], ref_out[None]
        call = lambda: tr.flash_prefill(q4, k4, v4, o4, 128, 2, 4, w.alpha, 2, 0)
        st = tr.run_dense(q4, k4, v4, o4, 128, 2, 4, w.alpha, 2, 0)
        mk = ws[L["mk"]:L["mk"] + 2 * st["mk"].numel()].view(q.dtype).view(st["mk"].shape)
        rep = tr.dense_mask_diff(st, cnt, idx, w.alpha)
    torch.cuda.synchronize()
    first_s = time.perf_counter() - t0
    mk_equal = bool(torch.equal(mk, st["mk"]))
    warps = st["mean_warps"]
    del st
    ours_out = torch.empty_like(q)
    if w.varlen:
        _ops.prefill_varlen(q, k, v, ours_out, cu, maxlen, w.alpha, 128, 2, 4, 2)
    else:
        _ops.prefill_dense(q[None], k[None], v[None], ours_out[None], 128, 2, 4, w.alpha, 2, 0)
    torch.cuda.synchronize()
    d = (ours_out.float() - ref_out.float()).abs()
    dmax, dmean = d.max().item(), d.mean().item()
    del d, ours_out
    for _ in range(2):
        call()
    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    for e0, e1 in evs:
        e0.record(stream)
        call()
        e1.record(stream)
    torch.cuda.synchronize()
    t = sorted(e0.elapsed_time(e1) for e0, e1 in evs)
    ref_ms = sum(t) / len(t)
    torch.cuda.empty_cache()
    return {"value": round(ref_ms, 4), "unit": UNIT, "median_ms": round(t[len(t) // 2], 4), "steps": steps,
            "ours_ms": round(ours_ms, 4), "speedup": round(ref_ms / ours_ms, 3),
            "what": "reference ops.flash_prefill / flash_prefill_varlen_func (Triton, unmodified) on this GPU, "
                    "same inputs, autotune cache warmed, CUDA events per call",
            "first_call_s": round(first_s, 1), "mean_warps_autotuned": warps,
            "pooled_keys_bit_identical": mk_equal,
            "masks": {**rep, "rule": "ours vs the reference's lists; near = reference score within 1e-3 "
                                     "relative of its row threshold"},
            "output_vs_reference": {"max_abs": dmax, "mean_abs": dmean}}


def interpreter_baseline():
    """The reference's own kernels under the Triton interpreter on the host cores, one whole
    cfg0 layer (fp32), timed end to end (oracle/interp_ref.py)."""
    path = os.path.join(ROOT, "oracle", "interp_ref.py")
    try:
        r = subprocess.run([sys.executable, path], capture_output=True, text=True, timeout=600,
                           env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
        d = json.loads(r.stdout.strip().splitlines()[-1])
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"interpreter run failed: {e}"}
    return {"value": round(d["seconds"] * 1e3, 1), "unit": UNIT, "cores": d["threads"], "kind": "reference",
            "workload": "cfg0_dense_4k_fp32 (S=4096, 4/1 heads, fp32)", "extrapolated": False,
            "sample": "the complete cfg0 layer: the reference's Triton kernels under TRITON_INTERPRET=1 on the "
                      f"host, {d['selected_blocks']} blocks selected"}


# --------------------------------------------------------------------------- cfg4
def run_cfg4(a, rank, world, local):
    """prefill of one 131072-token sequence of uniform random token ids
    through a random-init Llama-3-8B (32 layers, bf16 weights ~ N(0, 0.02)), FlashPrefill
    attention in every layer, tensor parallel over the ranks (one NCCL all-reduce after o_proj
    and one after the MLP).  A step is one whole prefill (32 layers + last-token logits)."""
    import datetime

    import torch
    import torch.distributed as dist

    from flashprefill_b200.llama_prefill import LlamaConfig, TPLlamaPrefill, prefill_flops

    if a.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no runnable CPU path for a "
                              "32-layer 131072-token prefill (its Triton kernels need a GPU or the interpreter)"}))
        return
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"),
                                timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    cfg = LlamaConfig()
    S = 131072
    model = TPLlamaPrefill(cfg, rank, world, device=dev, seed=4)
    g = torch.Generator(device=dev)
    g.manual_seed(4004)
    tokens = torch.randint(0, cfg.vocab, (S,), device=dev, generator=g)
    for _ in range(max(1, a.warmup)):
        model.forward(tokens)
    steps = max(1, a.steps)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs, attn_evs = [], []
    with ClockSampler(local) as clk:
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            logits = model.forward(tokens, events=attn_evs)
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = sum(x.elapsed_time(y) for x, y in evs) / steps
    attn_ms = sum(x.elapsed_time(y) for x, y in attn_evs) / steps
    t = torch.tensor([ms, attn_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    finite = bool(torch.isfinite(logits).all().item())
    if rank == 0:
        hbm, tflops, tfl_sus, peak_kind = load_peaks()
        fl = prefill_flops(cfg, S)
        line = {"metric": "llama3_8b prefill ms @128K (FlashPrefill in every layer, tensor parallel)",
                "value": round(float(t[0]), 2), "unit": "ms/prefill", "n_gpus": world, "steps": steps,
                "warmup": max(1, a.warmup), "ms_per_step": round(float(t[0]), 2), "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (uniform random token ids, random-init weights N(0, 0.02))",
                "config": {"workload": "cfg4_llama3_8b_prefill_128k", "seq_len": S, "layers": cfg.layers,
                           "parallelism": f"tensor parallel x{world} (heads, MLP)"},
                "attention_ms_per_prefill": round(float(t[1]), 2),
                "attention_share": round(float(t[1] / t[0]), 4),
                "gemm_tflops": round(fl / (float(t[0] - t[1]) * 1e-3) / 1e12 / world, 1),
                "gemm_tflops_note": "projection/MLP GEMM FLOPs per GPU over the non-attention time",
                "tokens_per_s": round(S / (float(t[0]) * 1e-3), 1), "logits_finite": finite,
                "clocks": clk.summary(), "peak_bf16_tflops": tflops, "peak_kind": peak_kind}
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


# --------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="l128k",
                    help="l128k (default), cfg1, cfg2, cfg3, or cfg4: end-to-end Llama-3-8B prefill of 131072 "
                         "tokens, tensor parallel over the ranks")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-triton", action="store_true",
                    help="skip the reference's Triton path on this GPU (timed baseline + mask comparison)")
    ap.add_argument("--no-gather", action="store_true",
                    help="N>1: skip the separately timed gathers of the head shards into the full output")
    ap.add_argument("--shard", default=None, help="R/N: run rank R's share of an N-GPU job alone on one GPU "
                    "(no process group; for studying the per-rank work)")
    a = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    shard = tuple(int(x) for x in a.shard.split("/")) if a.shard else None
    if a.workload == "cfg4":
        return run_cfg4(a, rank, world, local)
    w = workload(a.workload)

    if a.impl == "reference":
        if rank != 0:
            return
        ms, info = cpu_sample(w, seconds_budget=max(10.0, 60.0 / max(1, a.steps)))
        line = {"metric": METRIC, "value": round(ms, 3), "unit": UNIT, "n_gpus": a.gpus, "steps": 1,
                "warmup": 0, "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded generator, BASELINE recipe)",
                "impl": "reference",
                "config": {"workload": w.name, "seq_len": sum(w.seqlens), "q_heads": w.hq, "kv_heads": w.hk,
                           "head_dim": w.d, "alpha": w.alpha, "l2": "inputs larger than L2"},
                "cpu_baseline": {"value": round(ms, 3), "unit": UNIT, "cores": info["cores"], "kind": "port",
                                 "sample": info["sample"]},
                "e2e": {"value": round(ms, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "extrapolated": True, "sample_seconds": round(info["sample_seconds"], 2),
                "note": "the reference has no CPU path of its own; this is the CPU restatement of its algorithm "
                        "timed on a bounded sample of the layer and extrapolated to the whole layer"}
        print(json.dumps(line))
        return

    import torch
    import torch.distributed as dist

    import flashprefill_b200 as fp
    from flashprefill_b200 import _ops

    if world > 1:
        import datetime
        # a collective that one rank never joins fails in two minutes instead of NCCL's ten
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"),
                                timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    from flashprefill_b200.sharding import layer_shard
    nb_max = math.ceil(max(w.seqlens) / 128)
    r_, n_ = shard if shard else (rank, world)
    if w.varlen and n_ > w.hk:
        raise SystemExit(f"varlen workloads shard by KV head only ({w.hk} KV heads, {n_} ranks)")
    try:
        hk0, hk1, hq0, hq1, qb0, qb1 = layer_shard(w.hq, w.hk, nb_max, r_, n_)
    except ValueError as e:
        raise SystemExit(str(e))
    hq_l, hk_l = hq1 - hq0, hk1 - hk0
    # 2-D split (more ranks than KV heads): this rank runs query blocks [qb0, qb1) of its heads
    rows2d = (qb0, qb1) != (0, nb_max)

    # every rank generates the same seeded layer and keeps its heads, so any N times the same layer
    q, k, v = device_inputs(w, 0, w.hk, dev, seed=w.config_index * 1000 + 1)
    if (hq0, hq1) != (0, w.hq):
        q, k, v = q[:, hq0:hq1].contiguous(), k[:, hk0:hk1].contiguous(), v[:, hk0:hk1].contiguous()
        torch.cuda.empty_cache()
    T = q.shape[0]
    cu = torch.tensor([0] + torch.tensor(w.seqlens).cumsum(0).tolist(), dtype=torch.int32, device=dev)
    maxlen = max(w.seqlens)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)
    if w.varlen:
        L = _ops.varlen_layout(len(w.seqlens), T, maxlen, hq_l, hk_l)
    else:
        L = _ops.dense_layout(1, T, hq_l, hk_l)
    ws = torch.empty(L["total"], dtype=torch.uint8, device=dev)

    def step(mid_event=None):
        if w.varlen:
            fp.search_varlen(q, k, cu, maxlen, w.alpha, 128, 2, 4, 2, workspace=ws)
        else:
            fp.search_dense(q[None], k[None], 128, 2, 4, w.alpha, 2, 0, workspace=ws)
        if mid_event is not None:
            mid_event.record(stream)
        if w.varlen:
            _ops.attention_varlen(q, k, v, out, cu, maxlen, ws)
        else:
            _ops.attention_dense(q[None], k[None], v[None], out[None], ws)

    def api_step():  # the call a user makes (flash_prefill / flash_prefill_varlen_func)
        if w.varlen:
            _ops.prefill_varlen(q, k, v, out, cu, maxlen, w.alpha, 128, 2, 4, 2, workspace=ws)
        else:
            _ops.prefill_dense(q[None], k[None], v[None], out[None], 128, 2, 4, w.alpha, 2, 0, workspace=ws,
                               q_blocks=(qb0, qb1) if rows2d else None)

    for _ in range(max(3, a.warmup)):
        api_step()
        if not rows2d:
            step()
    torch.cuda.synchronize()
    fp.check_device_error(ws)
    # the count rows past the layout's real tiles (varlen reserves an upper bound) are unused
    cnt = ws[L["cnt"]:L["cnt"] + 4 * hq_l * L["tiles"]].view(torch.int32).view(hq_l, L["tiles"])
    real_tiles = sum(math.ceil(x / 128) for x in w.seqlens)
    E_local = int((cnt[:, qb0:qb1] if rows2d else cnt[:, :real_tiles]).sum().item())

    # ---- timed region (device-resident inputs): the public entry point, one call per step
    evh = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(2)) for _ in range(a.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_wall = time.perf_counter()
        for e0, e2 in evh:
            e0.record(stream)
            api_step()
            e2.record(stream)
        torch.cuda.synchronize()
        t_wall = time.perf_counter() - t_wall
    if world > 1:
        dist.barrier()
    clocks = clk.summary()
    t_step = sum(e0.elapsed_time(e2) for e0, e2 in evh) / a.steps
    # ---- breakdown (not the headline): search and attention entry points, an event between.
    # A 2-D split rank has no separate range-restricted stage entries: its whole step stands in.
    if rows2d:
        t_search, t_attn = t_step, t_step
    else:
        evs = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(a.steps)]
        torch.cuda.synchronize()
        for e0, e1, e2 in evs:
            e0.record(stream)
            step(e1)
            e2.record(stream)
        torch.cuda.synchronize()
        t_search = sum(e0.elapsed_time(e1) for e0, e1, e2 in evs) / a.steps
        t_attn = sum(e1.elapsed_time(e2) for e0, e1, e2 in evs) / a.steps
    stats = torch.tensor([t_step, t_search, t_attn, E_local], dtype=torch.float64, device=dev)
    mx, tot = stats.clone(), stats.clone()
    if world > 1:
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    ms = float(mx[0])
    E_total = int(tot[3])

    # ---- end-to-end through the public API with host buffers
    e2e = None
    if not a.no_e2e:
        hq_, hk_, hv_ = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
        hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        # Steps are pipelined over three streams (upload, compute, download) with double-buffered
        # device inputs and outputs: step i's output download (device -> host) overlaps step i+1's
        # input upload (host -> device) on the full-duplex PCIe link and the compute of either.
        # Every step still moves all of its inputs in and its whole output out.
        bufs = [(torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(out))
                for _ in range(2)]
        s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_cmp = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        started = [False, False]

        def e2e_step(i):
            b = i % 2
            dq, dk, dv, dout = bufs[b]
            with torch.cuda.stream(s_in):
                if started[b]:
                    s_in.wait_event(ev_cmp[b])  # the compute of step i-2 has read these inputs
                dq.copy_(hq_, non_blocking=True)
                dk.copy_(hk_, non_blocking=True)
                dv.copy_(hv_, non_blocking=True)
                ev_in[b].record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(ev_in[b])
                if started[b]:
                    s_cmp.wait_event(ev_out[b])  # the download of step i-2 has read this output
                if w.varlen:
                    fp.flash_prefill_varlen_func(dq, dk, dv, dout, cu, maxlen, w.alpha, 128, 2, 4, 2)
                else:
                    fp.flash_prefill(dq[None], dk[None], dv[None], dout[None], 128, 2, 4, w.alpha, 2, 0)
                ev_cmp[b].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_cmp[b])
                hout.copy_(dout, non_blocking=True)
                ev_out[b].record(s_out)
            started[b] = True

        for i in range(2):
            e2e_step(i)
        # all --steps steps: the timed region ends with the last step's compute and download
        # (the pipeline's drain), which the whole-job figure includes
        n_e2e = max(2, a.steps)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(s_in)
        for i in range(2, 2 + n_e2e):
            e2e_step(i)
        s_in.wait_stream(s_out)
        s1.record(s_in)
        torch.cuda.synchronize()
        e2e_ms = torch.tensor([s0.elapsed_time(s1) / n_e2e], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        # the link's floor for one step: the same uploads and download, concurrent, no compute
        dq, dk, dv, dout = bufs[0]
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        f0.record(s_in)
        s_out.wait_event(f0)
        for _ in range(3):
            with torch.cuda.stream(s_in):
                dq.copy_(hq_, non_blocking=True)
                dk.copy_(hk_, non_blocking=True)
                dv.copy_(hv_, non_blocking=True)
            with torch.cuda.stream(s_out):
                hout.copy_(dout, non_blocking=True)
        s_in.wait_stream(s_out)
        f1.record(s_in)
        torch.cuda.synchronize()
        link_ms = f0.elapsed_time(f1) / 3
        e2e = {"value": round(float(e2e_ms), 3), "unit": UNIT,
               "link_floor_ms": round(link_ms, 3),
               "h2d_bytes_per_step": int((q.numel() + k.numel() + v.numel()) * q.element_size() * world),
               "d2h_bytes_per_step": int(out.numel() * out.element_size() * world), "steps": n_e2e,
               "pipelined": "upload / compute / download on three streams, device buffers double-buffered"}

    # ---- optional output gather (N>1), timed on its own.  The headline value excludes it; a
    # caller whose next operator is row-parallel over heads (o_proj under tensor parallelism)
    # never needs it.  Two ways, both leaving the full (T, Hq, D) output on every rank:
    #   nccl:  the layer as above, then an NCCL all-gather of the head shards into a rank-major
    #          buffer and one reorder copy;
    #   fused: the attention epilogue writes every output tile into all ranks' full outputs
    #          over NVLink (fpb_prefill_dense_peers, peers mapped by CUDA IPC), then a
    #          one-element all-reduce orders the ranks (a stream-ordered cross-GPU barrier).
    gather = None
    if world > 1 and not a.no_gather and not rows2d:
        stage = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=dev)
        full = torch.empty((T, world * hq_l, w.d), dtype=out.dtype, device=dev)

        def nccl_step():
            api_step()
            dist.all_gather_into_tensor(stage, out)
            full.view(T, world, hq_l, w.d).copy_(stage.permute(1, 0, 2, 3))

        def timed(fn):
            for _ in range(3):
                fn()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            dist.barrier()
            torch.cuda.synchronize()
            g0.record(stream)
            for _ in range(a.steps):
                fn()
            g1.record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([g0.elapsed_time(g1) / a.steps], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t)

        recv = (world - 1) * out.numel() * out.element_size()
        t_nccl = timed(nccl_step)
        gather = {"nvlink_bytes_in_per_rank": recv,
                  "nccl": {"ms_per_layer_with_gather": round(t_nccl, 4), "gather_ms": round(t_nccl - ms, 4),
                           "how": "layer, then NCCL all_gather_into_tensor + reorder copy to (T, Hq, D)"}}
        if not w.varlen:
            from flashprefill_b200.peer_output import PeerOutputs
            full2 = torch.full((T, world * hq_l, w.d), float("nan"), dtype=out.dtype, device=dev)
            mine = full2[:, hq0:hq1]
            peers = PeerOutputs(full2)
            pptr = peers.peer_ptrs((mine.data_ptr() - full2.data_ptr()))
            flag = torch.zeros(1, dtype=torch.float32, device=dev)

            def fused_step():
                _ops.prefill_dense(q[None], k[None], v[None], mine[None], 128, 2, 4, w.alpha, 2, 0,
                                   workspace=ws, out_peers=pptr)
                dist.all_reduce(flag)

            t_fused = timed(fused_step)
            torch.cuda.synchronize()
            dist.barrier()
            same = torch.tensor([1.0 if torch.equal(full2, full) else 0.0], device=dev)
            dist.all_reduce(same, op=dist.ReduceOp.MIN)
            peers.close()
            gather["fused"] = {"ms_per_layer_with_gather": round(t_fused, 4),
                               "gather_ms": round(t_fused - ms, 4),
                               "equals_nccl_gather_on_all_ranks": bool(same.item() == 1.0),
                               "how": "attention epilogue stores every tile to all ranks' full outputs "
                                      "(16-byte peer stores over NVLink, CUDA IPC mappings), then a "
                                      "1-element all-reduce as barrier"}
    # ---- CPU baseline (rank 0, N=1 only)
    cpu = None
    exact = None
    if rank == 0 and world == 1 and not a.no_cpu:
        cms, info = cpu_sample(w, seconds_budget=20.0)
        cpu = {"value": round(cms, 3), "unit": UNIT, "cores": info["cores"], "kind": "port", "sample": info["sample"]}
        if not w.varlen:
            exact = mask_exactness(w, info["mask_sample"], dev)

    # ---- the reference's own Triton path on this GPU (rank 0, N=1): the bar to beat, and
    # the reference's block masks compared with ours on the same inputs
    triton = None
    if rank == 0 and world == 1 and not shard and not a.no_triton:
        triton = triton_baseline(w, q, k, v, cu, maxlen, ws, L, a.steps, ms)
    interp = None
    if rank == 0 and world == 1 and not a.no_cpu:
        interp = interpreter_baseline()

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    hbm, tflops, _, peak_kind = load_peaks()
    whole = world == 1 and not shard and not os.environ.get("FLASHPREFILL_B200_NO_SPLIT")
    traffic = NCU_TRAFFIC.get(w.name, {}) if whole else {}
    sb, af, sf = algorithmic(w, hq_l, hk_l, E_local)
    t_a, t_s = float(mx[2]), float(mx[1])
    ach = af / (t_a * 1e-3) / 1e12
    roof = {"bound": "tensor", "achieved": round(ach, 2), "peak": tflops, "unit": "TFLOP/s",
            "frac": round(ach / tflops, 4), "traffic": traffic.get("attention"),
            "kernel": "sparse_attn2_kernel", "ms": round(t_a, 4),
            "algorithmic": f"E*4*128*128*128 FLOP, E={E_local} executed block pairs on this rank"
                           + (" (2-D split rank: time of the whole step, search included)" if rows2d else ""),
            "peak_kind": f"{peak_kind} burst bf16 (of measured)" if peak_kind == "measured" else "fallback"}
    sach = sb / (t_s * 1e-3) / 1e9
    roof_s = {"bound": "hbm", "achieved": round(sach, 1), "peak": hbm, "unit": "GB/s", "frac": round(sach / hbm, 4),
              "ms": round(t_s, 4), "mma_tflops": round(sf / (t_s * 1e-3) / 1e12, 1),
              "kernels": "block_mean_kernel + block_search_kernel",
              "traffic_search_kernel": traffic.get("search"),
              "algorithmic": "2*(S*Hq*D + S*Hk*D) + 4*E + 4*Hq*NB bytes", "peak_kind": f"{peak_kind} HBM copy"}
    nbs = [math.ceil(L_ / 128) for L_ in w.seqlens]
    P_pairs = w.hq * sum(nb * (nb + 1) // 2 for nb in nbs)
    # kernels one public call launches: pooled keys, search, attention; varlen adds its prep
    # kernel; the long-row split plan adds two unless the dense entry rules it out on the host
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    plan = L["cap"] > 64 and not os.environ.get("FLASHPREFILL_B200_NO_SPLIT")
    if plan and not w.varlen:
        plan = split_plan_runs_dense(T, hq_l, L["cap"], sms)
    launches = 3 + (1 if w.varlen else 0) + (2 if plan else 0)
    line = {"metric": METRIC, "value": round(ms, 4), "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": max(3, a.warmup), "ms_per_step": round(ms, 4), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (BASELINE generator recipe, device RNG)",
            "config": {"workload": w.name, "seq_len": sum(w.seqlens), "seqlens": w.seqlens, "q_heads": w.hq,
                       "kv_heads": w.hk, "head_dim": w.d, "alpha": w.alpha, "sink": 2, "window": 4, "last_n": 2,
                       "parallelism": (f"kv-head groups x{w.hk} x query-block ranges x{world // w.hk}" if rows2d
                                       else f"kv-head groups x{world}"), "l2": "inputs larger than L2 (no flush)"},
            "search_ms": round(t_s, 4), "attention_ms": round(t_a, 4),
            "executed_pairs": E_total, "density": round(E_total / P_pairs, 5),
            "roofline": roof, "roofline_search": roof_s, "e2e": e2e, "cpu_baseline": cpu,
            "cpu_baseline_interpreter": interp, "triton_baseline": triton,
            "mask_exactness": exact,
            "gpu_launches": a.steps * launches, "output_gather": gather,
            "clocks": clocks, "wall_s_timed": round(t_wall, 3)}
    print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
