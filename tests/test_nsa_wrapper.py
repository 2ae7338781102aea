"""The full-NSA wrapper's host-side branches (nsa_hopper_b200.nsa) on CPU, against fixtures made
by the reference's own ``nsa_forward`` in fp64 (tests/golden/make_golden.py, nsa_full_*).

The wrapper's compressed branch, sliding-window branch, block scoring and gate run here on
CPU tensors; the selected branch -- a B200 kernel in the product -- is supplied by the oracle
in this test only, so the combination checks every other piece of the wrapper exactly."""
import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import nsa
from tests import golden_cases

CASES = golden_cases.full_case_names()


@pytest.mark.parametrize("name", CASES)
def test_wrapper_branches_reproduce_reference(name):
    c = golden_cases.load(name)
    q, k, v = c["q"], c["k"], c["v"]
    sel = torch.from_numpy(c["sel"])
    Kc, Vc = nsa.compress_kv(k, v, 32, 16)
    o_cmp = nsa.compressed_branch(q, Kc, Vc, chunk=256).double().numpy()
    o_win = nsa.window_branch(q, k, v, c["window"], chunk=256).double().numpy()
    o_sel, _ = oracle.forward(q, k, v, sel, c["LP"], 1)
    g = nsa.gate_weights(None, "cpu").double().numpy()
    o = g[0] * o_cmp + g[1] * o_sel + g[2] * o_win
    got = golden_cases.rows_of(o, c["rows"])
    # fp32 branches against the fp64 reference: the reference's own fp32 floor is 2e-6 scaled
    # (validate.py:10); the CPU fp32 matmuls here stay within a few of those
    err = np.abs(got - c["o_rows"]).max() / float(c["out_absmax"])
    assert err < 2e-5, err


@pytest.mark.parametrize("name", CASES)
def test_block_scores_and_selection_match_reference(name):
    c = golden_cases.load(name)
    q, k = c["q"], c["k"]
    Kc, _ = nsa.compress_kv(k, c["v"], 32, 16)
    blk = nsa.block_scores(q, Kc, c["LP"]).double().numpy()
    r = c["blk_rows"]
    got = blk[r[:, 0], r[:, 1], r[:, 2]]
    ref = c["blk"]
    fin = np.isfinite(ref)
    assert (np.isfinite(got) == fin).all()                       # identical causal block mask
    scale = np.abs(ref[fin]).max()
    assert np.abs(got[fin] - ref[fin]).max() <= 1e-5 * scale
    # the selection: the same set of blocks wherever the reference's ranking has no near-tie
    sel = nsa.select_blocks(q, Kc, c["n_sel"], c["LP"]).numpy()
    ref_sel = c["sel"]
    kk = ref_sel.shape[-1]
    for (b, h, t), row in zip(r, ref):
        s_sorted = np.sort(row[np.isfinite(row)])[::-1]
        if len(s_sorted) > kk and s_sorted[kk - 1] - s_sorted[kk] < 1e-4 * scale:
            continue  # near-tie at the selection boundary
        fin_sel = [x for x in ref_sel[b, h, t] if np.isfinite(row[x])]
        got_sel = [x for x in sel[b, h, t] if np.isfinite(row[x])]
        assert sorted(fin_sel) == sorted(got_sel), (b, h, t)


def test_compress_kv_matches_reference_definition():
    g = torch.Generator().manual_seed(3)
    K = torch.randn(2, 3, 100, 16, generator=g)
    V = torch.randn(2, 3, 100, 8, generator=g)
    Kc, Vc = nsa.compress_kv(K, V, 32, 16)
    n = (100 - 32) // 16 + 1
    idx = torch.arange(32).view(1, -1) + torch.arange(n).view(-1, 1) * 16
    torch.testing.assert_close(Kc, K[:, :, idx, :].mean(3))
    torch.testing.assert_close(Vc, V[:, :, idx, :].mean(3))
    assert nsa.compress_kv(K[:, :, :20], V[:, :, :20], 32, 16)[0].shape == (2, 3, 0, 16)


def test_gate_weights():
    torch.testing.assert_close(nsa.gate_weights(None, "cpu"), torch.full((3,), 1 / 3))
    w = torch.tensor([0.5, -1.0, 2.0])
    gs = torch.sigmoid(w)
    torch.testing.assert_close(nsa.gate_weights(w, "cpu"), gs / gs.sum())


def test_nsa_forward_refuses_cpu_tensors():
    q = torch.zeros(1, 2, 64, 64)
    with pytest.raises(RuntimeError):
        nsa.nsa_forward(q, q[:, :1], q[:, :1])
