"""The registered PyTorch ops: schema with an in-place output, fake implementations (CPU),
and on the GPU the same result as the Python entry points."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import flashprefill_b200 as fp  # noqa: F401  (registers the ops)


def test_ops_registered_with_mutable_outputs():
    for name, mut in (("prefill_dense", "out"), ("prefill_varlen", "o")):
        schema = getattr(torch.ops.flashprefill, name).default._schema
        args = {a.name: a for a in schema.arguments}
        assert args[mut].alias_info is not None and args[mut].alias_info.is_write
        assert len(schema.returns) == 0


def test_fake_tensor_calls_trace_without_running():
    with FakeTensorMode():
        q = torch.empty(1, 512, 4, 128, dtype=torch.bfloat16, device="cuda")
        kv = torch.empty(1, 512, 2, 128, dtype=torch.bfloat16, device="cuda")
        torch.ops.flashprefill.prefill_dense(q, kv, kv, torch.empty_like(q), 128, 2, 4, 0.18, 2, 0)
        qv = torch.empty(700, 4, 128, dtype=torch.bfloat16, device="cuda")
        kvv = torch.empty(700, 2, 128, dtype=torch.bfloat16, device="cuda")
        cu = torch.empty(3, dtype=torch.int32, device="cuda")
        torch.ops.flashprefill.prefill_varlen(qv, kvv, kvv, torch.empty_like(qv), cu, 500, 0.18)


@pytest.mark.gpu
def test_ops_match_python_entry_points():
    from tests import gpu_util as gu
    q, k, v, cu = gu.make_packed([3000, 700], 4, 2, torch.bfloat16, seed0=3)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    cud = torch.tensor(cu, dtype=torch.int32, device="cuda")
    o1, o2 = torch.empty_like(q), torch.empty_like(q)
    fp.flash_prefill_varlen_func(q, k, v, o1, cud, 3000, 0.18, 128, 2, 4, 2)
    torch.ops.flashprefill.prefill_varlen(q, k, v, o2, cud, 3000, 0.18, 128, 2, 4, 2)
    qd, kd, vd = q[None, :3000], k[None, :3000], v[None, :3000]
    d1, d2 = torch.empty_like(qd), torch.empty_like(qd)
    fp.flash_prefill(qd, kd, vd, d1, 128, 2, 4, 0.18, 2, 0)
    torch.ops.flashprefill.prefill_dense(qd, kd, vd, d2, 128, 2, 4, 0.18, 2, 0)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(d1, d2)
