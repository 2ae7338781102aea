"""The allocation-free selection entry point (nsa_sel_select_noalloc): same result as the
workspace form, no device allocation across calls, and oversize requests refused before any
launch.  Kept last in collection so the memory check sees a warmed-up process."""
import ctypes

import numpy as np
import pytest
import torch

from nsa_hopper_b200 import capi

STATIC_BYTES = 16 << 20


def test_static_scratch_size_and_oversize_refusal():
    lib = capi.load()
    assert lib.nsa_sel_select_static_scratch_bytes() == STATIC_BYTES
    # 64 KV heads x 1024 blocks x 256 dims x 4 B = 64 MB > 16 MB: refused before touching a device
    rc = lib.nsa_sel_select_noalloc(ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256), 1, 64, 64,
                                    65536, 256, 64, 16, 32, 16, None)
    assert rc == capi.NSA_ERR_UNSUPPORTED
    assert "static scratch" in capi.last_error()


@pytest.mark.gpu
def test_noalloc_matches_workspace_form_and_allocates_nothing():
    B, Hq, Hkv, T, D, n, lp = 1, 64, 4, 8192, 128, 16, 64
    g = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn(B, Hq, T, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    kk = min(n, (T + lp - 1) // lp)
    ws = torch.empty(capi.select_workspace_bytes(B, Hkv, T, D, lp) // 4, device="cuda", dtype=torch.float32)
    ref = torch.empty(B, Hkv, T, kk, device="cuda", dtype=torch.int32)
    got = torch.full_like(ref, -7)
    stream = torch.cuda.current_stream().cuda_stream
    capi.select(q.data_ptr(), k.data_ptr(), ws.data_ptr(), ref.data_ptr(), B, Hq, Hkv, T, D, lp, n, stream=stream)
    capi.select_noalloc(q.data_ptr(), k.data_ptr(), got.data_ptr(), B, Hq, Hkv, T, D, lp, n, stream=stream)  # warm-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(20):
        capi.select_noalloc(q.data_ptr(), k.data_ptr(), got.data_ptr(), B, Hq, Hkv, T, D, lp, n, stream=stream)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.equal(got, ref)
    assert np.all(got.cpu().numpy()[..., 0] >= 0)
