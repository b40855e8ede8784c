"""C ABI checks that need no GPU: the library loads, exports every symbol the header
declares, sizes its workspace consistently, and rejects invalid arguments on the host
before any CUDA call is made."""
import ctypes
import os
import re

import pytest

from flashprefill_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flashprefill_b200.h")


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from flashprefill_b200 import build
        build.build()
    return _lib.load()


def header_symbols():
    txt = open(HEADER).read()
    return set(re.findall(r"FPB_API\s+[\w\s\*]+?\b(fpb_\w+)\s*\(", txt))


def test_every_declared_symbol_is_exported(lib):
    syms = header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in the header but not exported"
    assert syms == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_version(lib):
    assert lib.fpb_version() >= 100


def _layout(lib, varlen, a, b, c, hq, hk):
    out = (ctypes.c_int64 * 8)()
    assert lib.fpb_workspace_layout(varlen, a, b, c, hq, hk, 128, out) == 0
    return list(out)


def test_dense_workspace_layout(lib):
    err, cu, mk, cnt, idx, total, tiles, cap = _layout(lib, 0, 2, 1000, 0, 8, 2)
    assert tiles == 2 * 8 and cap == 8
    assert err == 0 and cu < mk < cnt < idx < total
    assert cnt - mk >= tiles * 2 * 128 * 2
    assert idx - cnt >= 8 * tiles * 4
    assert total - idx >= 8 * tiles * cap * 4
    assert all(x % 256 == 0 for x in (cu, mk, cnt, idx, total))
    assert lib.fpb_dense_workspace_bytes(2, 1000, 8, 2, 128) == total


def test_varlen_workspace_bound(lib):
    # 4 sequences of 8K/16K/32K/64K: true block count 960, bound ceil(T/128)+nseq
    T = 8192 + 16384 + 32768 + 65536
    *_, total, tiles, cap = _layout(lib, 1, 4, T, 65536, 32, 8)
    assert tiles == T // 128 + 4 and cap == 512
    assert lib.fpb_varlen_workspace_bytes(T, 4, 65536, 32, 8, 128) == total


def _call_dense(lib, **over):
    a = dict(q=256, k=512, v=768, o=1024, dtype=0, B=1, S=1024, hq=4, hk=2, d=128, bs=128, ws=4096,
             wsb=1 << 30, model=4)
    a.update(over)
    st = _lib.i64arr([1024 * 4 * 128, 4 * 128, 128])
    sk = _lib.i64arr([1024 * 2 * 128, 2 * 128, 128])
    P = ctypes.c_void_p
    return lib.fpb_prefill_dense(P(a["q"]), P(a["k"]), P(a["v"]), P(a["o"]), a["dtype"], a["B"], a["S"], a["hq"],
                                 a["hk"], a["d"], st, sk, sk, st, a["bs"], 2, 4, 0.1, 2, 0, a["model"], P(a["ws"]),
                                 a["wsb"], None)


@pytest.mark.parametrize("over,msg", [
    (dict(d=64), "head_dim"),
    (dict(bs=64), "block_size"),
    (dict(hq=6, hk=4), "multiple"),
    (dict(dtype=7), "dtype"),
    (dict(q=0), "q is NULL"),
    (dict(k=520), "16-byte"),
    (dict(S=0), "seqlen"),
    (dict(wsb=100), "workspace too small"),
    (dict(ws=4100), "256-byte"),
    (dict(model=5), "mean_model"),
])
def test_invalid_arguments_rejected_before_launch(lib, over, msg):
    rc = _call_dense(lib, **over)
    assert rc == _lib.FPB_EINVAL
    assert msg in lib.fpb_last_error().decode()


@pytest.mark.parametrize("peers,n,msg", [
    ([4096], 8, "n_peers"),
    (None, 1, "out_peers is NULL"),
    ([0], 1, "out_peers[0]"),
    ([4096, 4104], 2, "out_peers[1]"),
])
def test_peer_entry_rejects_bad_peers(lib, peers, n, msg):
    """fpb_prefill_dense_peers checks its peer list on the host before anything runs."""
    st = _lib.i64arr([1024 * 4 * 128, 4 * 128, 128])
    sk = _lib.i64arr([1024 * 2 * 128, 2 * 128, 128])
    P = ctypes.c_void_p
    arr = (P * len(peers))(*peers) if peers is not None else None
    rc = lib.fpb_prefill_dense_peers(P(256), P(512), P(768), P(1024), 0, 1, 1024, 4, 2, 128, st, sk, sk, st, 128,
                                     2, 4, 0.1, 2, 0, 4, P(4096), 1 << 30, arr, n, None)
    assert rc == _lib.FPB_EINVAL
    assert msg in lib.fpb_last_error().decode()


def test_python_rejects_cpu_tensors():
    import torch
    import flashprefill_b200 as fp
    q = torch.zeros(1, 256, 2, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 256, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        fp.flash_prefill(q, k, k, torch.empty_like(q), 128, 2, 4, 0.1, 2, 0)
    with pytest.raises(ValueError, match="CUDA"):
        fp.flash_prefill_varlen_func(q[0], k[0], k[0], torch.empty_like(q[0]),
                                     torch.tensor([0, 256], dtype=torch.int32), 256, 0.1)


def test_install_as_ops_aliases_reference_import_paths():
    import sys
    import flashprefill_b200 as fp
    keys = ("ops", "ops.flashprefill_native_forward", "ops.flashprefill_varlen_func")
    saved = {k: sys.modules.get(k) for k in keys}
    try:
        fp.install_as_ops()
        from ops import flash_prefill_varlen_func
        from ops.flashprefill_native_forward import flash_prefill
        assert flash_prefill is fp.flash_prefill and flash_prefill_varlen_func is fp.flash_prefill_varlen_func
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


def test_chunk_and_range_entries_reject_bad_sizes_on_the_host(lib):
    """fpb_prefill_dense_chunk (q_len must be in [1, kv_len]) and fpb_prefill_dense_rows (the
    query-block range must be non-empty and inside the sequence) refuse before any CUDA call;
    the timeout test hook refuses limits outside [1 ms, 1 s]; the tile-count bounds refuse
    problems whose lists would overflow the workspace indexing."""
    P = ctypes.c_void_p
    st = _lib.i64arr([1024 * 4 * 128, 4 * 128, 128])
    sk = _lib.i64arr([1024 * 2 * 128, 2 * 128, 128])
    for q_len, kv_len in [(0, 1024), (2048, 1024)]:
        rc = lib.fpb_prefill_dense_chunk(P(256), P(512), P(768), P(1024), 0, 1, q_len, kv_len, 4, 2, 128, st, sk, sk,
                                         st, 128, 2, 4, 0.1, 2, 0, 4, P(4096), 1 << 30, None)
        assert rc == _lib.FPB_EINVAL and "q_len" in lib.fpb_last_error().decode()
    for b, e in [(3, 3), (-1, 2), (0, 9)]:
        rc = lib.fpb_prefill_dense_rows(P(256), P(512), P(768), P(1024), 0, 1, 1024, 4, 2, 128, st, sk, sk, st, 128,
                                        2, 4, 0.1, 2, 0, 4, b, e, P(4096), 1 << 30, None)
        assert rc == _lib.FPB_EINVAL and "query-block range" in lib.fpb_last_error().decode()
    assert lib.fpb_test_set_fault(0, 10) == _lib.FPB_EINVAL
    assert lib.fpb_test_set_fault(0, 5_000_000_000) == _lib.FPB_EINVAL
    rc = lib.fpb_prefill_dense(P(256), P(512), P(768), P(1024), 0, 1 << 20, 1 << 20, 4, 2, 128, st, sk, sk, st,
                               128, 2, 4, 0.1, 2, 0, 4, P(4096), 1 << 30, None)
    assert rc == _lib.FPB_EINVAL and "too large" in lib.fpb_last_error().decode()
