"""The block-selection kernel (nsa_sel_select through ops.select_blocks) against the reference's
own selection (nsa_full_* fixtures: reference select_blocks in fp64, nsa_reference.py:27-44)
and against the PyTorch restatement of the same scores."""
import numpy as np
import pytest
import torch

from nsa_hopper_b200 import indices, nsa, ops
from tests import golden_cases

pytestmark = pytest.mark.gpu


def _visible(row_sel, t, lp):
    return sorted(int(x) for x in row_sel if 0 <= x and x * lp <= t)


@pytest.mark.parametrize("name", golden_cases.full_case_names())
def test_selection_matches_reference(name):
    c = golden_cases.load(name)
    q, k = c["q"].cuda(), c["k"].cuda()
    sel = ops.select_blocks(q, k, c["n_sel"], c["LP"]).cpu().numpy()
    n_blk = (c["T"] + c["LP"] - 1) // c["LP"]
    assert sel.shape == (c["B"], c["Hkv"], c["T"], min(c["n_sel"], n_blk))
    r, blk = c["blk_rows"], c["blk"]
    scale = np.abs(blk[np.isfinite(blk)]).max()
    kk = sel.shape[-1]
    checked = 0
    for (b, h, t), row in zip(r, blk):
        got = sel[b, h, t]
        nvis = int(np.isfinite(row).sum())
        # exactly min(k, visible) entries, best first, then -1 padding
        assert (got[:min(kk, nvis)] >= 0).all() and (got[min(kk, nvis):] == -1).all()
        scores = row[got[got >= 0]]
        assert (np.diff(scores) <= 1e-6 * scale).all()            # sorted by score, highest first
        s_sorted = np.sort(row[np.isfinite(row)])[::-1]
        if len(s_sorted) > kk and s_sorted[kk - 1] - s_sorted[kk] < 1e-4 * scale:
            continue                                               # near-tie at the boundary
        assert _visible(got, t, c["LP"]) == _visible(c["sel"][b, h, t], t, c["LP"]), (b, h, t)
        checked += 1
    assert checked > len(r) // 2


@pytest.mark.parametrize("B,Hq,Hkv,T,D,n,lp", [(1, 16, 1, 4096, 128, 16, 64), (2, 8, 2, 3000, 64, 8, 128),
                                               (1, 64, 4, 8192, 128, 16, 64), (1, 4, 4, 700, 192, 32, 64)])
def test_selection_matches_tensor_op_restatement(B, Hq, Hkv, T, D, n, lp):
    g = torch.Generator(device="cuda").manual_seed(T)
    q = torch.randn(B, Hq, T, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    sel = ops.select_blocks(q, k, n, lp).cpu().numpy()
    Kc, _ = nsa.compress_kv(k, k, 32, 16)
    blk = nsa.block_scores(q, Kc, lp).cpu().numpy()            # fp32 restatement of the scores
    kk = sel.shape[-1]
    rng = np.random.default_rng(0)
    scale = np.abs(blk[np.isfinite(blk)]).max()
    bad = 0
    for _ in range(400):
        b, h, t = rng.integers(0, B), rng.integers(0, Hkv), rng.integers(0, T)
        row = blk[b, h, t]
        s_sorted = np.sort(row[np.isfinite(row)])[::-1]
        if len(s_sorted) > kk and s_sorted[kk - 1] - s_sorted[kk] < 1e-5 * scale:
            continue
        want = sorted(int(x) for x in np.argsort(-row, kind="stable")[:kk] if np.isfinite(row[x]))
        bad += _visible(sel[b, h, t], t, lp) != want
    assert bad == 0


def test_selection_feeds_the_selected_branch():
    """The kernel's output (with -1 padding) is a valid index tensor for the selected branch."""
    B, Hq, Hkv, T, D = 1, 16, 2, 1500, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(B, Hq, T, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    sel = ops.select_blocks(q, k, 8, 64)
    o, lse = ops.forward_lse(q, k, v, sel, 64, 1)
    torch.cuda.synchronize()
    assert torch.isfinite(lse).all() and torch.isfinite(o.float()).all()
