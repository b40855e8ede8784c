"""Device-side failure detection without a GPU fault.

Every wait inside the kernels is bounded; a wait that runs out makes the CTA stop issuing,
drain its in-flight copies and MMAs, free its tensor memory and set FPB_DEV_WAIT_TIMEOUT in
the workspace error word, which the host reads.  The test hook fpb_test_set_fault shortens
the wait limit to 20 ms and makes the attention kernel's first CTA withhold one key load
(a barrier that nothing completes), so the timeout path runs for real; the next normal call
on the same CUDA context must succeed and match a call made before the fault.
"""
import ctypes

import pytest
import torch

import flashprefill_b200 as fp
from flashprefill_b200 import _lib, _ops
from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.mark.parametrize("varlen", [False, True])
def test_wait_timeout_reported_and_context_survives(varlen):
    lib = _lib.load()
    lens = [3000] if not varlen else [2000, 1100]
    q, k, v, cu = gu.make_packed(lens, 4, 1, torch.bfloat16, seed0=4242)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    cud = torch.tensor(cu, dtype=torch.int32, device=DEV)

    def call(o):
        if varlen:
            return _ops.prefill_varlen(qd, kd, vd, o, cud, max(lens), 0.1)
        return _ops.prefill_dense(qd[None], kd[None], vd[None], o[None], 128, 2, 4, 0.1, 2, 0)

    ref = torch.zeros_like(qd)
    ws = call(ref)
    assert fp.check_device_error(ws) == 0
    torch.cuda.synchronize()
    _lib.check(lib.fpb_test_set_fault(1, 20_000_000))
    try:
        bad = torch.zeros_like(qd)
        ws = call(bad)
        with pytest.raises(fp.FlashPrefillError, match="wait timed out"):
            fp.check_device_error(ws)
    finally:
        _lib.check(lib.fpb_test_set_fault(0, 1_000_000_000))
    torch.cuda.synchronize()  # the context is still usable
    again = torch.zeros_like(qd)
    ws = call(again)
    assert fp.check_device_error(ws) == 0
    assert torch.equal(again, ref)


def test_fault_hook_rejects_out_of_range_limits():
    lib = _lib.load()
    assert lib.fpb_test_set_fault(0, 10) == _lib.FPB_EINVAL
    assert lib.fpb_test_set_fault(0, 5_000_000_000) == _lib.FPB_EINVAL
