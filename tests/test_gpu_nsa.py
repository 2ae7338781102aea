"""The full NSA forward on the GPU (nsa_hopper_b200.nsa, selected branch on the B200 kernel)
against the reference's own fp64 ``nsa_forward`` fixtures, with the reference's metric and bar:
max|err| / max|out| <= 3e-2 for bf16 (validate.py:10, 22-24)."""
import numpy as np
import pytest
import torch

from nsa_hopper_b200 import nsa
from tests import golden_cases

pytestmark = pytest.mark.gpu
CASES = golden_cases.full_case_names()
BF16_FLOOR = 3e-2  # validate.py:10


def _scaled_err(o, c):
    got = golden_cases.rows_of(o.double().cpu().numpy(), c["rows"])
    return np.abs(got - c["o_rows"]).max() / float(c["out_absmax"])


@pytest.mark.parametrize("name", CASES)
def test_validate_fn_with_reference_selection(name):
    """validate.check(fn) path: fn(Q, K, V, sel, cfg) with the reference's selection."""
    c = golden_cases.load(name)
    dev = torch.device("cuda")
    q, k, v = c["q"].to(dev), c["k"].to(dev), c["v"].to(dev)
    cfg = dict(n_sel=c["n_sel"], l_prime=c["LP"], window=c["window"])
    o = nsa.validate_fn(q, k, v, torch.from_numpy(c["sel"]).to(dev), cfg)
    torch.cuda.synchronize()
    assert o.dtype == torch.float32 and o.shape == q.shape
    err = _scaled_err(o, c)
    assert err <= BF16_FLOOR / 3, err  # well inside the reference's own bf16 floor
    cs = golden_cases.checksums(o.double().cpu().numpy())
    assert (np.abs(cs - c["checksums"]) <= 2e-3 * (np.abs(c["checksums"]) + o.numel() ** 0.5)).all()


@pytest.mark.parametrize("name", CASES)
def test_nsa_forward_own_selection(name):
    """nsa_forward selecting its own blocks on the GPU: the selection agrees with the
    reference's away from near-ties, and the output meets the bf16 bar."""
    c = golden_cases.load(name)
    dev = torch.device("cuda")
    q, k, v = c["q"].to(dev), c["k"].to(dev), c["v"].to(dev)
    o, sel = nsa.nsa_forward(q, k, v, n_sel=c["n_sel"], l_prime=c["LP"], window=c["window"])
    torch.cuda.synchronize()
    sel = sel.cpu().numpy()
    assert sel.shape == c["sel"].shape
    r, blk = c["blk_rows"], c["blk"]
    kk = sel.shape[-1]
    scale = np.abs(blk[np.isfinite(blk)]).max()
    agree = 0
    for (b, h, t), row in zip(r, blk):
        s_sorted = np.sort(row[np.isfinite(row)])[::-1]
        if len(s_sorted) > kk and s_sorted[kk - 1] - s_sorted[kk] < 1e-4 * scale:
            continue
        ref_set = sorted(x for x in c["sel"][b, h, t] if x >= 0 and np.isfinite(row[x]))
        got_set = sorted(x for x in sel[b, h, t] if x >= 0 and np.isfinite(row[x]))
        assert all(x == -1 or np.isfinite(row[x]) for x in sel[b, h, t])  # only visible blocks or -1
        assert ref_set == got_set, (b, h, t)
        agree += 1
    assert agree > len(r) // 2
    # output rows whose (b, kvh, t) selection equals the reference's meet the bf16 bar
    G = c["Hq"] // c["Hkv"]
    rows = c["rows"]
    def vis(row_sel, t):  # the visible part of a selection row (the reference pads with future blocks)
        return sorted(x for x in row_sel if 0 <= x and x * c["LP"] <= t)

    same = np.array([vis(sel[b, hq // G, t], t) == vis(c["sel"][b, hq // G, t], t) for b, hq, t in rows])
    assert same.mean() > 0.5
    got = golden_cases.rows_of(o.double().cpu().numpy(), rows)
    err = np.abs(got[same] - c["o_rows"][same]).max() / float(c["out_absmax"])
    assert err <= BF16_FLOOR / 3, err
