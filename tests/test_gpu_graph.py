"""CUDA graph capture of the forward (nsa_sel_run through the C ABI).

A captured launch keeps its dynamic work-counter slot (and the reset queued before it) for every
replay, so captured launches take slots that eager launches never use.  The test wraps the eager
slots twice (more than 4096 eager launches), then replays the graph on one stream while eager
launches run on another, and checks both results (a shared slot would make the two launches skip
each other's work units)."""
import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import capi, indices
from tests.helpers import compare, make_qkv

pytestmark = pytest.mark.gpu


def _desc(q, k, v, sel, o, lse):
    B, Hq, T, D = q.shape
    return capi.make_desc(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), sel=sel.data_ptr(), o=o.data_ptr(),
                          lse=lse.data_ptr(), batch=B, heads_q=Hq, heads_kv=k.shape[1], seq_len=T, d_qk=D, d_v=D,
                          n_qblocks=T, n_sel=sel.shape[3], block_size=64, q_block=1, o_dtype=capi.DTYPE_BF16)


def test_graph_replay_beside_eager_launches_on_another_stream():
    B, Hq, Hkv, T, D, n = 1, 16, 1, 2048, 64, 8  # 2048 units > 148 CTAs: the dynamic counter is used
    inputs = []
    for seed in (31, 32):
        q, k, v = make_qkv(B, Hq, Hkv, T, D, D, seed=seed)
        sel = indices.rule0(B, Hkv, T, n, 64, seed=seed)
        inputs.append((q, k, v, sel))
    dev = [(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(s).cuda()) for q, k, v, s in inputs]
    o_g = torch.empty(B, Hq, T, D, device="cuda", dtype=torch.bfloat16)
    l_g = torch.empty(B, Hq, T, device="cuda", dtype=torch.float32)
    o_e, l_e = torch.empty_like(o_g), torch.empty_like(l_g)
    d_g = _desc(*dev[0], o_g, l_g)
    d_e = _desc(*dev[1], o_e, l_e)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    capi.run(d_g, s1.cuda_stream)  # eager warm-up: module, attributes and counter base are resolved
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        capi.run(d_g, torch.cuda.current_stream().cuda_stream)
    # wrap the eager slots twice; the last launch reuses a slot that two earlier launches used
    for i in range(4200):
        if i == 4199:
            o_e.fill_(float("nan"))
        capi.run(d_e, s2.cuda_stream)
    torch.cuda.synchronize()
    ref_g = oracle.forward(*inputs[0][:3], inputs[0][3], 64, 1)
    ref_e = oracle.forward(*inputs[1][:3], inputs[1][3], 64, 1)
    compare(o_e, l_e, *ref_e)
    for _ in range(3):  # replays on s1 next to eager launches on s2
        o_g.fill_(float("nan"))
        o_e.fill_(float("nan"))
        torch.cuda.synchronize()
        with torch.cuda.stream(s1):
            g.replay()
        for _ in range(4):
            capi.run(d_e, s2.cuda_stream)
        torch.cuda.synchronize()
        compare(o_g, l_g, *ref_g)
        compare(o_e, l_e, *ref_e)


def test_static_unit_schedule_flag_gives_identical_results():
    """NSA_DEBUG_STATIC_UNITS (fixed strides instead of the counter) changes only the schedule."""
    q, k, v, sel = [t.cuda() if hasattr(t, "cuda") else torch.from_numpy(t).cuda()
                    for t in (*make_qkv(1, 16, 1, 2048, 64, 64, seed=33), indices.rule0(1, 1, 2048, 8, 64, seed=33))]
    o1 = torch.empty(1, 16, 2048, 64, device="cuda", dtype=torch.bfloat16)
    l1 = torch.empty(1, 16, 2048, device="cuda", dtype=torch.float32)
    o2, l2 = torch.empty_like(o1), torch.empty_like(l1)
    capi.run(_desc(q, k, v, sel, o1, l1), torch.cuda.current_stream().cuda_stream)
    d2 = _desc(q, k, v, sel, o2, l2)
    d2.debug_flags = capi.NSA_DEBUG_STATIC_UNITS
    capi.run(d2, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16)) and torch.equal(l1, l2)
