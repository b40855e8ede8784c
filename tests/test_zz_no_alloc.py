"""The no-allocation dense prefill, called through the C ABI.

fpb_prefill_dense_noalloc exists for callers that cannot allocate device memory or hand
over a workspace (runtimes that forbid allocation on their hot path, C hosts without a
device allocator); it keeps its scratch in a fixed 32 MiB array inside the library.  This
test checks its output against the workspace entry point fpb_prefill_dense, bit for bit
(both run the same kernels), on calls in a row: first a 16K-token case whose last rows
are long enough to be split into chunks (the split area inside the array is used), then
smaller cases that reuse the scratch the earlier calls left behind.  It also checks that
a problem too large for the array is rejected, and that a device-side error of a
no-allocation call is visible through fpb_noalloc_read_device_error.  It lives in its
own file, collected last.
"""
import ctypes

import pytest
import torch

from flashprefill_b200 import _lib
from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _args(q, k, v, out):
    B, S, hq, d = q.shape
    hk = k.shape[2]
    P = ctypes.c_void_p
    return (P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(out.data_ptr()), _lib.FPB_BF16, B, S, hq, hk, d,
            _lib.i64arr(q.stride()[:3]), _lib.i64arr(k.stride()[:3]), _lib.i64arr(v.stride()[:3]),
            _lib.i64arr(out.stride()[:3]), 128, 2, 4, 0.18, 2, 0, 4)


def test_noalloc_matches_workspace_entry_point_twice():
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    for seed, (S, hq, hk) in enumerate([(16384, 8, 2), (4096, 8, 2), (3000, 4, 1)]):
        q, k, v, _ = gu.make_packed([S], hq, hk, torch.bfloat16, seed0=900 + seed)
        qd, kd, vd = (t[None].to(DEV) for t in (q, k, v))
        ref = torch.empty_like(qd)
        ws = torch.empty(lib.fpb_dense_workspace_bytes(1, S, hq, hk, 128), dtype=torch.uint8, device=DEV)
        _lib.check(lib.fpb_prefill_dense(*_args(qd, kd, vd, ref), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                         stream))
        out = torch.full_like(qd, float("nan"))
        _lib.check(lib.fpb_prefill_dense_noalloc(*_args(qd, kd, vd, out), stream))
        torch.cuda.synchronize()
        flags = ctypes.c_uint32(0)
        assert lib.fpb_noalloc_read_device_error(ctypes.byref(flags), stream) == _lib.FPB_OK and flags.value == 0
        assert torch.equal(out, ref), f"S={S}: no-allocation output differs from fpb_prefill_dense"


def test_noalloc_rejects_problems_beyond_its_scratch():
    lib = _lib.load()
    # 128K tokens, 32/8 heads needs ~136 MB of scratch, more than the 32 MiB array
    st = _lib.i64arr([131072 * 32 * 128, 32 * 128, 128])
    sk = _lib.i64arr([131072 * 8 * 128, 8 * 128, 128])
    P = ctypes.c_void_p
    rc = lib.fpb_prefill_dense_noalloc(P(256), P(256), P(256), P(256), 0, 1, 131072, 32, 8, 128, st, sk, sk, st,
                                       128, 2, 4, 0.18, 2, 0, 4, None)
    assert rc == _lib.FPB_EINVAL
    assert "32 MiB" in lib.fpb_last_error().decode()


def test_noalloc_device_error_is_visible():
    """A wait that runs out inside a no-allocation call (test hook: the attention kernel's
    first CTA withholds a key load, waits limited to 20 ms) is reported by
    fpb_noalloc_read_device_error; the next call on the same context succeeds and clears it."""
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    S, hq, hk = 2048, 4, 1
    q, k, v, _ = gu.make_packed([S], hq, hk, torch.bfloat16, seed0=950)
    qd, kd, vd = (t[None].to(DEV) for t in (q, k, v))
    out = torch.empty_like(qd)
    torch.cuda.synchronize()
    _lib.check(lib.fpb_test_set_fault(1, 20_000_000))
    try:
        _lib.check(lib.fpb_prefill_dense_noalloc(*_args(qd, kd, vd, out), stream))
        flags = ctypes.c_uint32(0)
        rc = lib.fpb_noalloc_read_device_error(ctypes.byref(flags), stream)
    finally:
        _lib.check(lib.fpb_test_set_fault(0, 1_000_000_000))
    assert rc == _lib.FPB_EDEVICE and flags.value & 1, (rc, flags.value)
    ref = torch.empty_like(qd)
    ws = torch.empty(lib.fpb_dense_workspace_bytes(1, S, hq, hk, 128), dtype=torch.uint8, device=DEV)
    _lib.check(lib.fpb_prefill_dense(*_args(qd, kd, vd, ref), ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream))
    _lib.check(lib.fpb_prefill_dense_noalloc(*_args(qd, kd, vd, out), stream))
    flags = ctypes.c_uint32(0)
    assert lib.fpb_noalloc_read_device_error(ctypes.byref(flags), stream) == _lib.FPB_OK and flags.value == 0
    assert torch.equal(out, ref)
