"""The in-tree PyTorch extension (nsa_hopper_b200._C) with the reference op signature."""
import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import indices
from tests.helpers import compare, make_qkv

pytestmark = pytest.mark.gpu


def test_forward_lse_op():
    from nsa_hopper_b200 import ops

    q, k, v = make_qkv(1, 16, 2, 640, 128, 128, seed=21)
    sel = indices.rule0(1, 2, 640, 16, 64, seed=21)
    o, lse = ops.forward_lse(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(sel).cuda(), 64, 1)
    torch.cuda.synchronize()
    assert o.dtype == torch.bfloat16 and lse.dtype == torch.float32
    compare(o, lse, *oracle.forward(q, k, v, sel, 64, 1))


def test_forward_op_reference_signature():
    from nsa_hopper_b200 import ops

    q, k, v = make_qkv(1, 8, 2, 512, 64, 64, seed=22)
    sel = indices.perm_qblock(1, 2, 512, 4, 16, 64, seed=22)
    o = ops.forward(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(sel).cuda(), 64, 16)
    torch.cuda.synchronize()
    assert o.dtype == torch.float32
    r, _ = oracle.forward(q, k, v, sel, 64, 16)
    assert np.abs(o.cpu().numpy() - r).max() <= 1e-2


def test_op_rejects_bad_dtype():
    from nsa_hopper_b200 import ops

    q = torch.randn(1, 4, 64, 64, device="cuda")
    sel = torch.zeros(1, 2, 4, 1, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError):
        ops.forward(q, q[:, :2], q[:, :2], sel, 64, 16)
