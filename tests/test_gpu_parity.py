"""Parity of the sm_100a kernel (called through the C ABI) with the CPU oracle.

Every case feeds the same seeded bf16 inputs to both sides.  Bars: indices and masking are
exact (the mask-probe tests count contributing keys); O within 2e-2 max-abs and LSE within 1e-3
relative of the fp64 oracle (tests/helpers.py).
"""
import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import indices
from tests.helpers import compare, make_qkv, run_capi

pytestmark = pytest.mark.gpu


def _check_rule(B, Hq, Hkv, T, dqk, dv, n, rule, seed=0, l_prime=64):
    q, k, v = make_qkv(B, Hq, Hkv, T, dqk, dv, seed)
    sel = indices.generate(rule, B=B, Hkv=Hkv, T=T, n=n, block=l_prime, seed=seed)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), l_prime=l_prime)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel, l_prime, 1)
    return compare(o, lse, o_ref, lse_ref)


def test_config0_full():
    """B=1 T=1024 Hq=16 Hkv=1 D=64 n=8, rule 0 (whole tensor)."""
    _check_rule(1, 16, 1, 1024, 64, 64, 8, "rule0")


def test_config1_shape_small_T():
    """BASELINE config 1 heads/dims (Hq=64 Hkv=4 D=128 n=16) at T=2048."""
    _check_rule(1, 64, 4, 2048, 128, 128, 16, "rule0", seed=1)


def test_config2_reuse_rule():
    _check_rule(2, 64, 4, 1536, 128, 128, 16, "rule0_reuse", seed=2)


def test_config3_dk192():
    """d_qk=192, d_v=128, rule 3 (block 0 + the two most recent blocks)."""
    _check_rule(1, 32, 2, 2048, 192, 128, 16, "rule3", seed=3)


def test_config4_varlen_small_group():
    """G=4 packed varlen batch with cu_seqlens; lengths not multiples of 64."""
    lens = [300, 1000, 77, 2048, 64, 129]
    Hq, Hkv, D, n = 32, 8, 128, 16
    T = sum(lens)
    q, k, v = make_qkv(1, Hq, Hkv, T, D, D, seed=4)
    sel = indices.varlen_rule0(lens, Hkv, n, 64, seed=4)
    cu = indices.cu_seqlens_of(lens)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), cu_seqlens=torch.from_numpy(cu))
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel, 64, 1, cu_seqlens=cu)
    compare(o, lse, o_ref, lse_ref)


@pytest.mark.parametrize("B,Hq,Hkv,S,D,KSEL,BQ", [
    (1, 8, 2, 512, 64, 4, 16), (1, 16, 2, 1024, 128, 8, 8), (1, 4, 4, 512, 64, 4, 64),
    (1, 16, 1, 1024, 64, 6, 4), (1, 8, 2, 2048, 128, 16, 16),      # test_v1.py / test_v2.py shapes
    (1, 8, 2, 512, 64, 8, 16), (1, 16, 1, 768, 64, 6, 16),         # test_v0.py shapes (G=16, BQ=16)
])
def test_reference_harness_shapes_fp32(B, Hq, Hkv, S, D, KSEL, BQ):
    """Per-query-block selection with fp32 O, the reference op's own mode (test_v*.py)."""
    q, k, v = make_qkv(B, Hq, Hkv, S, D, D, seed=7)
    sel = indices.perm_qblock(B, Hkv, S, KSEL, BQ, 64, seed=7)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), BQ=BQ, out_f32=True)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel, 64, BQ)
    r = compare(o, lse, o_ref, lse_ref, o_atol=1e-2)
    assert r["o_scaled"] < 3e-2  # the reference tests' PASS bar (test_v2.py:25)


@pytest.mark.parametrize("l_prime", [128, 256])
def test_large_blocks(l_prime):
    B, Hq, Hkv, S, D, KSEL, BQ = 1, 8, 2, 1024, 128, 4, 8
    q, k, v = make_qkv(B, Hq, Hkv, S, D, D, seed=11)
    sel = indices.perm_qblock(B, Hkv, S, KSEL, BQ, l_prime, seed=11, heads_share=False)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), BQ=BQ, l_prime=l_prime)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel, l_prime, BQ)
    compare(o, lse, o_ref, lse_ref)


def test_edge_selection_rows():
    """-1 padding, duplicates, id == n_blk, id > n_blk, future blocks, all-padding rows,
    T not a multiple of 64 and G = 1."""
    B, Hq, Hkv, T, D, n = 1, 2, 2, 500, 64, 6
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, seed=5)
    rng = np.random.default_rng(5)
    nblk = (T + 63) // 64
    sel = rng.integers(-3, nblk + 3, size=(B, Hkv, T, n)).astype(np.int32)
    sel[:, :, ::7, :] = -1                 # rows with nothing selected
    sel[:, :, 3::11, 1] = sel[:, :, 3::11, 0]  # duplicates
    sel[:, 0, 5::13, :] = nblk             # the reference's scratch id
    o, lse = run_capi(q, k, v, torch.from_numpy(sel))
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel, 64, 1)
    compare(o, lse, o_ref, lse_ref)
    # rows without a visible key: O exactly 0, LSE -inf
    counts = oracle.count_keys(sel, T, 64, 1).reshape(B, Hkv, T)
    empty = np.repeat(counts == 0, Hq // Hkv, axis=1)
    assert empty.any()
    assert (o.float().cpu().numpy()[empty] == 0).all()


def test_mask_probe_counts_exact():
    """Q = 0 makes every visible key weigh exactly 1: exp(LSE) must equal the oracle's key
    count and O the mean of one-hot V rows, so the set of contributing keys is pinned."""
    B, Hq, Hkv, T, D, n = 1, 16, 2, 1100, 128, 16
    _, k, _ = make_qkv(B, Hq, Hkv, T, D, D, seed=6)
    q = torch.zeros(B, Hq, T, D, dtype=torch.bfloat16)
    v = torch.zeros(B, Hkv, T, D, dtype=torch.bfloat16)
    pos = torch.arange(T)
    v[:, :, pos, pos % D] = 1.0  # key p contributes to column p % D
    sel = indices.rule0(B, Hkv, T, n, 64, seed=6)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), out_f32=True)
    torch.cuda.synchronize()
    counts = oracle.count_keys(sel, T, 64, 1).reshape(B, Hkv, T)
    cnt = np.repeat(counts, Hq // Hkv, axis=1).astype(np.float64)
    got = np.exp(lse.cpu().numpy().astype(np.float64))
    assert np.array_equal(np.rint(got), cnt), "visible-key counts differ"
    # column histogram: O[..., d] * count = number of visible keys p with p % D == d
    o_np = o.cpu().numpy().astype(np.float64) * cnt[..., None]
    ref = oracle.forward(q, k, v, sel, 64, 1)[0] * cnt[..., None]
    assert np.array_equal(np.rint(o_np), np.rint(ref)), "contributing key sets differ"


def test_shards_compose():
    """Disjoint shards over (b*Hkv+kvh) and query blocks reproduce the full launch bit for bit."""
    B, Hq, Hkv, T, D, n = 2, 16, 2, 768, 128, 16
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, seed=8)
    sel = torch.from_numpy(indices.rule0(B, Hkv, T, n, 64, seed=8))
    o_full, l_full = run_capi(q, k, v, sel)
    o_sh = torch.full_like(o_full, float("nan"))
    l_sh = torch.full_like(l_full, float("nan"))
    for bkv in [(0, 1), (1, 4)]:
        for qb in [(0, 300), (300, 768)]:
            run_capi(q, k, v, sel, shard=(bkv[0], bkv[1], qb[0], qb[1]), o=o_sh, lse=l_sh)
    torch.cuda.synchronize()
    assert torch.equal(o_full.view(torch.int16), o_sh.view(torch.int16))
    assert torch.equal(l_full, l_sh)


def test_grid_size_does_not_change_results():
    B, Hq, Hkv, T, D, n = 1, 16, 1, 1024, 64, 8
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, seed=9)
    sel = torch.from_numpy(indices.rule0(B, Hkv, T, n, 64, seed=9))
    o1, l1 = run_capi(q, k, v, sel)
    o2, l2 = run_capi(q, k, v, sel, max_ctas=7)
    torch.cuda.synchronize()
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16)) and torch.equal(l1, l2)


def test_cycle_counters_and_error_word():
    B, Hq, Hkv, S, D, KSEL, BQ = 1, 8, 2, 512, 64, 4, 16
    q, k, v = make_qkv(B, Hq, Hkv, S, D, D, seed=10)
    sel = indices.perm_qblock(B, Hkv, S, KSEL, BQ, 64, seed=10)
    NQB = sel.shape[2]
    cyc = torch.zeros(NQB * B * Hkv * 2, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    run_capi(q, k, v, torch.from_numpy(sel), BQ=BQ, out_f32=True, cyc=cyc, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    c = cyc.cpu().numpy()
    assert (c[1::2] > 0).all()  # every query block did some work
