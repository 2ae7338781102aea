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


def _linspace_f32_device_rule(T, n):
    """The selection kernel's float32 linspace (nsa_select_kernel.cuh: linspace_f32): step rounded
    to float32, each value formed in double from the nearer end, then rounded."""
    f32 = np.float32
    if n == 1:
        return np.zeros(1, f32)
    step = f32(f32(T - 1) / f32(n - 1))
    i = np.arange(n)
    lo = (np.float64(step) * i).astype(f32)
    hi = (np.float64(T - 1) - np.float64(step) * (n - 1 - i)).astype(f32)
    return np.where(i < n // 2, lo, hi)


def _floor_div_f32_device_rule(a, b):
    f32 = np.float32
    out = []
    for x in a:
        x, bb = f32(x), f32(b)
        mod = f32(np.fmod(x, bb))
        div = f32(f32(x - mod) / bb)
        if mod != 0 and ((bb < 0) != (mod < 0)):
            div = f32(div - f32(1))
        if div != 0:
            fl = f32(np.floor(div))
            if f32(div - fl) > f32(0.5):
                fl = f32(fl + f32(1))
            out.append(fl)
        else:
            out.append(f32(np.copysign(f32(0), f32(x / bb))))
    return np.array(out, dtype=f32)


@pytest.mark.parametrize("T", [33, 100, 500, 512, 768, 1000, 1024, 2048, 4097, 8192, 12345, 65536, 131072])
def test_selection_kernel_block_mapping_matches_reference(T):
    """The compressed-key -> selection-block map the selection kernel derives on the device is the
    reference's (src // l_prime) on torch.linspace (nsa_reference.py:35-36), bit for bit."""
    n = (T - 32) // 16 + 1
    ref = torch.linspace(0, T - 1, n).numpy()
    mine = _linspace_f32_device_rule(T, n)
    assert (ref.view(np.int32) == mine.view(np.int32)).all()
    for lp in (64, 128, 256):
        want = (torch.from_numpy(ref) // lp).numpy()
        assert (_floor_div_f32_device_rule(mine, lp) == want).all()


def _compressed_limit_device_rule(t, T, n):
    """nsa_linspace.cuh: compressed_limit (the last compressed key visible to query t)."""
    if n <= 1:
        return n - 1
    pos = _linspace_f32_device_rule(T, n)
    est = int(np.floor(t * (n - 1) / (T - 1)))
    best = -1
    for i in range(max(0, est - 2), min(n - 1, est + 3) + 1):
        if pos[i] <= np.float32(t):
            best = i
    return best


@pytest.mark.parametrize("T", [40, 500, 1024, 2048, 4097, 65536])
def test_compressed_key_map_matches_reference_mask(T):
    """The kernel's compressed key map (key i visible to t iff linspace(i) <= t) is the reference's
    cmask = cpos <= arange(S) (nsa_reference.py:62-63) for every (sampled) token."""
    n = (T - 32) // 16 + 1
    cpos = torch.linspace(0, T - 1, n)
    assert (np.diff(cpos.numpy()) >= 0).all()
    ts = range(T) if T <= 4097 else np.random.default_rng(0).integers(0, T, 3000)
    for t in ts:
        want = int((cpos <= torch.tensor(float(t))).sum().item()) - 1
        assert _compressed_limit_device_rule(int(t), T, n) == want, t


@pytest.mark.parametrize("T,window,bq", [(1000, 512, 1), (1000, 512, 4), (777, 100, 8), (130, 1000, 2), (64, 64, 16)])
def test_window_selection_rows_cover_exactly_the_window(T, window, bq):
    """Each query block's row lists exactly the 64-key blocks that meet [t0 - window + 1, t1]
    (t0, t1 the block's first and last tokens), in descending order, -1 padded."""
    sel = nsa.window_selection(1, 1, T, window, 64, "cpu", bq)[0, 0].numpy()
    assert sel.shape == ((T + bq - 1) // bq, (window + bq - 2) // 64 + 2)
    for qb in range(sel.shape[0]):
        t0, t1 = qb * bq, min(T, qb * bq + bq) - 1
        want = list(range(t1 // 64, max(0, t0 - window + 1) // 64 - 1, -1))
        row = [int(x) for x in sel[qb]]
        assert row[:len(want)] == want and all(x == -1 for x in row[len(want):])


def test_branch_q_block_fills_the_query_tile():
    assert [nsa.branch_q_block(g) for g in (1, 4, 8, 16, 32, 64, 128)] == [128, 32, 16, 8, 4, 2, 1]
    assert [nsa.branch_q_block(g) for g in (3, 12, 24, 48)] == [16, 4, 2, 1]
