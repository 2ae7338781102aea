"""nsa_sel_run_host: host inputs in, host outputs back, with the copies pipelined against the
kernel over (b, kvh) rows x token slices.  Its outputs must equal the device-buffer launch bit for
bit, leave host rows outside the shard untouched, and handle BQ > 1, ragged T and varlen."""
import ctypes

import numpy as np
import pytest
import torch

from nsa_hopper_b200 import capi, workload

pytestmark = pytest.mark.gpu


def _case(B, Hq, Hkv, T, D, n, BQ, o_f32, seed, varlen=False):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, Hq, T, D, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, device=dev, generator=g).to(torch.bfloat16)
    NQB = (T + BQ - 1) // BQ
    rng = np.random.default_rng(seed)
    sel = torch.from_numpy(rng.integers(-1, max(1, T // 64), size=(B, Hkv, NQB, n), dtype=np.int32)).to(dev)
    cu = None
    if varlen:
        cu = torch.tensor([0, T // 3, T // 3 + 5, T], dtype=torch.int32, device=dev)
    return q, k, v, sel, cu


def _desc(q, k, v, sel, cu, o, lse, BQ, o_f32, **kw):
    B, Hq, T, D = q.shape
    d = capi.make_desc(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), sel=sel.data_ptr(), o=o.data_ptr(),
                       lse=lse.data_ptr() if lse is not None else None, batch=B, heads_q=Hq, heads_kv=k.shape[1],
                       seq_len=T, d_qk=D, d_v=v.shape[3], n_qblocks=sel.shape[2], n_sel=sel.shape[3], block_size=64,
                       q_block=BQ, o_dtype=capi.DTYPE_F32 if o_f32 else capi.DTYPE_BF16, **kw)
    if cu is not None:
        d.cu_seqlens = cu.data_ptr()
        d.n_seqs = cu.numel() - 1
    return d


@pytest.mark.parametrize("B,Hq,Hkv,T,D,n,BQ,o_f32,slices,varlen", [
    (1, 64, 4, 8192, 128, 16, 1, False, 0, False),
    (2, 16, 2, 3000, 64, 8, 4, True, 3, False),
    (1, 32, 8, 5000, 128, 16, 1, False, 5, True),
    (1, 8, 1, 777, 64, 4, 2, True, 0, False),
    (1, 64, 4, 2048, 128, 16, 8, False, 3, False),  # 128-row tiles: the row-owner kernel
])
def test_host_path_equals_device_launch(B, Hq, Hkv, T, D, n, BQ, o_f32, slices, varlen):
    q, k, v, sel, cu = _case(B, Hq, Hkv, T, D, n, BQ, o_f32, T + n, varlen)
    odt = torch.float32 if o_f32 else torch.bfloat16
    o_ref = torch.empty(B, Hq, T, D, device="cuda", dtype=odt)
    l_ref = torch.empty(B, Hq, T, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    capi.run(_desc(q, k, v, sel, cu, o_ref, l_ref, BQ, o_f32), s)
    # host copies of the inputs; device buffers start as garbage
    hq, hk, hv, hs = (x.cpu().pin_memory() for x in (q, k, v, sel))
    ho = torch.full(o_ref.shape, 7.0, dtype=odt).pin_memory()
    hl = torch.full(l_ref.shape, 7.0).pin_memory()
    dq, dk, dv, ds = (torch.full_like(x, 3) for x in (q, k, v, sel))
    do, dl = torch.empty_like(o_ref), torch.empty_like(l_ref)
    io = capi.make_host_io(q=hq.data_ptr(), k=hk.data_ptr(), v=hv.data_ptr(), sel=hs.data_ptr(), o=ho.data_ptr(),
                           lse=hl.data_ptr(), token_slices=slices)
    capi.run_host(_desc(dq, dk, dv, ds, cu, do, dl, BQ, o_f32), io, s)
    torch.cuda.synchronize()
    assert torch.equal(ho, o_ref.cpu()) and torch.equal(hl, l_ref.cpu())


def test_host_path_shard_leaves_other_rows_untouched():
    B, Hq, Hkv, T, D, n, BQ = 1, 32, 4, 4096, 128, 16, 1
    q, k, v, sel, cu = _case(B, Hq, Hkv, T, D, n, BQ, False, 11)
    o_ref = torch.empty(B, Hq, T, D, device="cuda", dtype=torch.bfloat16)
    l_ref = torch.empty(B, Hq, T, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    capi.run(_desc(q, k, v, sel, cu, o_ref, l_ref, BQ, False), s)
    hq, hk, hv, hs = (x.cpu().pin_memory() for x in (q, k, v, sel))
    ho = torch.full(o_ref.shape, 7.0, dtype=torch.bfloat16).pin_memory()
    hl = torch.full(l_ref.shape, 7.0).pin_memory()
    do, dl = torch.empty_like(o_ref), torch.empty_like(l_ref)
    dq, dk, dv, ds = (torch.empty_like(x) for x in (q, k, v, sel))
    io = capi.make_host_io(q=hq.data_ptr(), k=hk.data_ptr(), v=hv.data_ptr(), sel=hs.data_ptr(), o=ho.data_ptr(),
                           lse=hl.data_ptr())
    capi.run_host(_desc(dq, dk, dv, ds, cu, do, dl, BQ, False, bkv_begin=1, bkv_end=3, qb_begin=1000, qb_end=3001),
                  io, s)
    torch.cuda.synchronize()
    G = Hq // Hkv
    inside = torch.zeros(B, Hq, T, dtype=torch.bool)
    inside[:, G:3 * G, 1000:3001] = True
    assert torch.equal(ho[inside], o_ref.cpu()[inside]) and torch.equal(hl[inside], l_ref.cpu()[inside])
    assert (ho[~inside] == 7.0).all() and (hl[~inside] == 7.0).all()
