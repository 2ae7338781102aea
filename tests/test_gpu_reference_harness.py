"""Drop-in check: build the op exactly as the reference's test harness does and run its check.

reference test_v2.py:4-6 JIT-loads `nsa_v2.cu` with `-arch=sm_90a` flags and calls
`mod.forward(Q,K,V,sel,LP,BQ,cyc)`, comparing with `ref_selected` by scaled error < 3e-2 and
printing the load fraction from `cyc` (test_v2.py:21-26).  Here the same call builds
nsa_hopper_b200/csrc/nsa_sel_reference_op.cu and the oracle stands in for `ref_selected`.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import indices

pytestmark = pytest.mark.gpu

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "nsa_hopper_b200", "csrc",
                   "nsa_sel_reference_op.cu")


@pytest.fixture(scope="module")
def mod():
    from torch.utils.cpp_extension import load

    return load("nsa_v2", [SRC], extra_cuda_cflags=["-arch=sm_90a", "-O3", "--use_fast_math", "--expt-relaxed-constexpr"],
                extra_include_paths=["/workspace/nsa/cutlass/include"], verbose=False)


@pytest.mark.parametrize("B,Hq,Hkv,S,D,KSEL,BQ", [(1, 8, 2, 512, 64, 4, 16), (1, 16, 2, 1024, 128, 8, 8),
                                                  (1, 4, 4, 512, 64, 4, 64), (1, 16, 1, 1024, 64, 6, 4),
                                                  (1, 8, 2, 2048, 128, 16, 16)])
def test_reference_harness_flow(mod, B, Hq, Hkv, S, D, KSEL, BQ):
    torch.manual_seed(7)
    NQB = (S + BQ - 1) // BQ
    Q = torch.randn(B, Hq, S, D, device="cuda", dtype=torch.bfloat16)
    K = torch.randn(B, Hkv, S, D, device="cuda", dtype=torch.bfloat16)
    V = torch.randn(B, Hkv, S, D, device="cuda", dtype=torch.bfloat16)
    sel = torch.from_numpy(indices.perm_qblock(B, Hkv, S, KSEL, BQ, 64, seed=7)).cuda()
    cyc = torch.zeros(NQB * B * Hkv * 2, dtype=torch.int64, device="cuda")
    o = mod.forward(Q, K, V, sel, 64, BQ, cyc)
    assert o.dtype == torch.float32 and o.shape == (B, Hq, S, D)
    r, _ = oracle.forward(Q.cpu(), K.cpu(), V.cpu(), sel.cpu(), 64, BQ)
    e = np.abs(o.double().cpu().numpy() - r).max() / np.abs(r).max()
    assert e < 3e-2  # the harness's PASS bar
    w, mm = cyc[0::2].float().mean().item(), cyc[1::2].float().mean().item()
    assert w + mm > 0 and 0.0 <= w / (w + mm) <= 1.0

