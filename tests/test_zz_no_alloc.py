"""The allocation-free selection entry point (nsa_sel_select_noalloc), for callers that cannot
allocate device memory themselves.  It must give the same rows as the workspace form on two
calls in a row (the static scratch keeps the previous call's contents), allocate nothing across
calls, accept a block-key table of exactly the static scratch's size and refuse one block more
before any launch.  Kept last in collection so the memory check sees a warmed-up process."""
import ctypes

import numpy as np
import pytest
import torch

from nsa_hopper_b200 import capi

STATIC_BYTES = 16 << 20


def test_static_scratch_size_and_oversize_refusal():
    lib = capi.load()
    assert lib.nsa_sel_select_static_scratch_bytes() == STATIC_BYTES
    assert capi.select_workspace_bytes(1, 16, 65536, 256, 64) == STATIC_BYTES  # exactly the limit
    # one more selection block (T = 65536 + 64: 1025 blocks) is 16 KB over: refused before any launch
    assert capi.select_workspace_bytes(1, 16, 65536 + 64, 256, 64) == STATIC_BYTES + 16 * 256 * 4
    for B, Hq, Hkv, T, d in [(1, 16, 16, 65536 + 64, 256), (1, 64, 64, 65536, 256)]:
        rc = lib.nsa_sel_select_noalloc(ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256), B, Hq, Hkv,
                                        T, d, 64, 16, 32, 16, None)
        assert rc == capi.NSA_ERR_UNSUPPORTED
        assert "static scratch" in capi.last_error()


def _select_both(B, Hq, Hkv, T, D, n, lp, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, Hq, T, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    kk = min(n, (T + lp - 1) // lp)
    ws = torch.empty(capi.select_workspace_bytes(B, Hkv, T, D, lp) // 4, device="cuda", dtype=torch.float32)
    ref = torch.empty(B, Hkv, T, kk, device="cuda", dtype=torch.int32)
    stream = torch.cuda.current_stream().cuda_stream
    capi.select(q.data_ptr(), k.data_ptr(), ws.data_ptr(), ref.data_ptr(), B, Hq, Hkv, T, D, lp, n, stream=stream)
    del ws
    return q, k, ref, stream


@pytest.mark.gpu
def test_noalloc_matches_workspace_form_and_allocates_nothing():
    B, Hq, Hkv, T, D, n, lp = 1, 64, 4, 8192, 128, 16, 64
    q, k, ref, stream = _select_both(B, Hq, Hkv, T, D, n, lp, seed=11)
    got = torch.full_like(ref, -7)
    for _ in range(2):  # two calls in a row, each checked (selection rows are exact integers)
        got.fill_(-7)
        capi.select_noalloc(q.data_ptr(), k.data_ptr(), got.data_ptr(), B, Hq, Hkv, T, D, lp, n, stream=stream)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(20):
        capi.select_noalloc(q.data_ptr(), k.data_ptr(), got.data_ptr(), B, Hq, Hkv, T, D, lp, n, stream=stream)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.equal(got, ref)
    assert np.all(got.cpu().numpy()[..., 0] >= 0)


@pytest.mark.gpu
def test_noalloc_at_exactly_the_scratch_limit():
    """A block-key table of exactly 16 MB (16 KV heads x 1024 blocks x 256 dims x 4 B) is accepted
    and matches the workspace form, after a smaller call left other contents in the scratch."""
    B, Hq, Hkv, T, D, n, lp = 1, 16, 16, 65536, 256, 16, 64
    assert capi.select_workspace_bytes(B, Hkv, T, D, lp) == STATIC_BYTES
    q, k, ref, stream = _select_both(B, Hq, Hkv, T, D, n, lp, seed=12)
    got = torch.full_like(ref, -7)
    for _ in range(2):
        got.fill_(-7)
        capi.select_noalloc(q.data_ptr(), k.data_ptr(), got.data_ptr(), B, Hq, Hkv, T, D, lp, n, stream=stream)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
