"""Failure detection on the GPU without a GPU fault: a launch whose first wait can only run
out of time must return through the bounded-wait path, report NSA_DEVERR_TIMEOUT in the
device error word, and leave the context usable for the next launch."""
import pytest
import torch

import oracle
from nsa_hopper_b200 import capi, indices
from tests.helpers import compare, make_qkv

pytestmark = pytest.mark.gpu


def _desc(q, k, v, sel, o, lse, err, **kw):
    B, Hq, T, D = q.shape
    return capi.make_desc(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), sel=sel.data_ptr(), o=o.data_ptr(),
                          lse=lse.data_ptr(), err=err.data_ptr(), batch=B, heads_q=Hq, heads_kv=k.shape[1],
                          seq_len=T, d_qk=D, d_v=v.shape[3], n_qblocks=sel.shape[2], n_sel=sel.shape[3],
                          block_size=64, q_block=1, o_dtype=capi.DTYPE_BF16, **kw)


def test_stalled_wait_reports_timeout_and_context_survives():
    B, Hq, Hkv, T, D, n = 1, 16, 1, 1024, 64, 8
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, seed=12)
    sel_np = indices.rule0(B, Hkv, T, n, 64, seed=12)
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    sel = torch.from_numpy(sel_np).cuda()
    o = torch.zeros(B, Hq, T, D, dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros(B, Hq, T, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    capi.run(_desc(dq, dk, dv, sel, o, lse, err, timeout_ms=50, debug_flags=capi.NSA_DEBUG_STALL), stream)
    torch.cuda.synchronize()  # must not raise: the kernel ended on its own
    assert int(err.item()) & capi.NSA_DEVERR_TIMEOUT
    # the same context keeps working
    err.zero_()
    capi.run(_desc(dq, dk, dv, sel, o, lse, err), stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    o_ref, lse_ref = oracle.forward(q, k, v, sel_np, 64, 1)
    compare(o, lse, o_ref, lse_ref)
