"""The row-owner kernel (nsa_ro_kernel.cuh: query rows on the MMA's M, P in tensor memory)
against the oracle, on the shapes that route to it: tiles of 128 query rows, or 64 (G divides the
tile's rows and BQ is a multiple of rows / G; 64-row tiles run on M = 64 MMAs, covered further by
tests/test_gpu_ro_m64.py)."""
import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import capi, indices, nsa, ops
from tests.helpers import compare, make_qkv, run_capi

pytestmark = pytest.mark.gpu


def _routes_to_row_owner(Hq, Hkv, BQ):
    G = Hq // Hkv
    return any(rows % G == 0 and BQ % (rows // G) == 0 for rows in (128, 64))


@pytest.mark.parametrize("B,Hq,Hkv,S,D,KSEL,BQ,lp,f32", [
    (1, 16, 1, 1000, 64, 6, 8, 64, True),       # G = 16, 8 tokens per tile, T not a multiple of 64
    (2, 64, 4, 1024, 128, 16, 8, 64, False),    # the north-star head layout, bf16 O
    (1, 32, 4, 1111, 128, 8, 16, 128, True),    # G = 8, l' = 128
    (1, 128, 1, 300, 64, 4, 1, 64, False),      # G = 128: one token per tile
    (1, 64, 2, 777, 64, 5, 4, 256, True),       # G = 32, l' = 256
    (1, 1, 1, 700, 128, 4, 128, 64, False),     # G = 1: 128 tokens share a row
    (1, 16, 1, 768, 64, 6, 16, 64, True),       # BQ = 16: two tiles per query block
    (1, 32, 2, 1000, 128, 16, 4, 64, True),     # 64-row tiles (BQ * G = 64, the reference's mode)
    (1, 8, 2, 2048, 128, 16, 16, 64, False),    # 64-row tiles, G = 4
    (1, 4, 4, 512, 64, 4, 64, 128, True),       # 64-row tiles, G = 1
])
def test_row_owner_matches_oracle(B, Hq, Hkv, S, D, KSEL, BQ, lp, f32):
    assert _routes_to_row_owner(Hq, Hkv, BQ)
    q, k, v = make_qkv(B, Hq, Hkv, S, D, D, seed=S + KSEL)
    sel = indices.perm_qblock(B, Hkv, S, KSEL, BQ, lp, seed=S, heads_share=False)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), BQ=BQ, l_prime=lp, out_f32=f32)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel, lp, BQ)
    compare(o, lse, o_ref, lse_ref)


def test_row_owner_plan():
    d = capi.make_desc(q=256, k=256, v=256, sel=256, o=256, batch=1, heads_q=64, heads_kv=4, seq_len=4096, d_qk=128,
                       d_v=128, n_qblocks=512, n_sel=16, block_size=64, q_block=8, o_dtype=capi.DTYPE_BF16)
    p = capi.plan(d)
    assert p["n_cols"] == 128 and p["q_per_unit"] == 8 and p["tmem_cols"] == 512


def test_row_owner_edge_selection_rows():
    """-1 padding, duplicates, the scratch id, ids past the end and future blocks, per query block."""
    B, Hq, Hkv, T, D, n, BQ = 1, 16, 2, 900, 64, 6, 16
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, seed=15)
    rng = np.random.default_rng(15)
    nblk = (T + 63) // 64
    NQB = (T + BQ - 1) // BQ
    sel = rng.integers(-3, nblk + 3, size=(B, Hkv, NQB, n)).astype(np.int32)
    sel[:, :, ::7, :] = -1
    sel[:, :, 3::11, 1] = sel[:, :, 3::11, 0]
    sel[:, 0, 5::13, :] = nblk
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), BQ=BQ, out_f32=True)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel, 64, BQ)
    compare(o, lse, o_ref, lse_ref)


def test_row_owner_mask_probe_counts_exact():
    """Q = 0: exp(LSE) is the exact number of visible keys of every row (tile rows, causal edge,
    ragged end)."""
    B, Hq, Hkv, T, D, n, BQ = 1, 16, 2, 1100, 128, 16, 8
    _, k, _ = make_qkv(B, Hq, Hkv, T, D, D, seed=16)
    q = torch.zeros(B, Hq, T, D, dtype=torch.bfloat16)
    v = torch.zeros(B, Hkv, T, D, dtype=torch.bfloat16)
    sel = indices.perm_qblock(B, Hkv, T, n, BQ, 64, seed=16, heads_share=False)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), BQ=BQ, out_f32=True)
    torch.cuda.synchronize()
    counts = oracle.count_keys(sel, T, 64, BQ).reshape(B, Hkv, T)
    cnt = np.repeat(counts, Hq // Hkv, axis=1).astype(np.float64)
    got = np.exp(lse.cpu().numpy().astype(np.float64))
    assert np.array_equal(np.rint(got), cnt)


@pytest.mark.parametrize("T,window,D", [(1500, 128, 64), (2048, 512, 128), (777, 100, 128)])
def test_row_owner_window_branch(T, window, D):
    B, Hq, Hkv = 1, 32, 2
    g = torch.Generator(device="cuda").manual_seed(T)
    q = torch.randn(B, Hq, T, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    bq = 128 // (Hq // Hkv)
    sel = nsa.window_selection(B, Hkv, T, window, 64, q.device, bq)
    o, lse = ops.forward_ext(q, k, v, sel, 64, bq, window=window)
    ref = nsa.window_branch(q, k, v, window)
    torch.cuda.synchronize()
    assert (o - ref).abs().max().item() <= 2e-2


@pytest.mark.parametrize("T,D", [(1500, 64), (4096, 128), (40, 64)])
def test_row_owner_compressed_branch_accumulates(T, D):
    """Compressed key map on the row-owner kernel, written with a weight and then added into an
    existing O (TMA reduce-add from the swizzled staging boxes)."""
    B, Hq, Hkv = 1, 16, 1
    g = torch.Generator(device="cuda").manual_seed(3 * T)
    q = torch.randn(B, Hq, T, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    Kc, Vc = nsa.compress_kv(k, v, 32, 16)
    if Kc.shape[2] == 0:
        pytest.skip("no compressed keys")
    Kc, Vc = Kc.to(torch.bfloat16).contiguous(), Vc.to(torch.bfloat16).contiguous()
    bq = 128 // (Hq // Hkv)
    sel = nsa.compressed_selection(B, Hkv, T, Kc.shape[2], q.device, bq)
    ref = nsa.compressed_branch(q, Kc.float(), Vc.float())
    w = torch.tensor([0.25], device="cuda")
    base = torch.randn(B, Hq, T, D, device="cuda", generator=g)
    o, _ = ops.forward_ext(q, Kc, Vc, sel, 64, bq, key_map=1, out=base.clone(), weight=w, accumulate=True)
    torch.cuda.synchronize()
    assert (o - (base + 0.25 * ref)).abs().max().item() <= 1e-2


def test_row_owner_varlen():
    """G = 64 with per-token rows of a packed varlen batch: 64-row tiles of one token each, block
    ids relative to each sequence start, lengths not multiples of 64."""
    lens = [300, 77, 1000, 64, 129]
    Hq, Hkv, D, n = 64, 1, 64, 8
    T = sum(lens)
    assert _routes_to_row_owner(Hq, Hkv, 1)
    q, k, v = make_qkv(1, Hq, Hkv, T, D, D, seed=21)
    sel = indices.varlen_rule0(lens, Hkv, n, 64, seed=21)
    cu = indices.cu_seqlens_of(lens)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), cu_seqlens=torch.from_numpy(cu))
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel, 64, 1, cu_seqlens=cu)
    compare(o, lse, o_ref, lse_ref)


def test_row_owner_shards_compose():
    """Disjoint (b*Hkv+kvh, query-block) shards reproduce the full row-owner launch bit for bit."""
    B, Hq, Hkv, T, D, n, BQ = 2, 32, 2, 1024, 128, 16, 8
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, seed=22)
    sel = torch.from_numpy(indices.perm_qblock(B, Hkv, T, n, BQ, 64, seed=22, heads_share=False))
    o_full, l_full = run_capi(q, k, v, sel, BQ=BQ)
    o_sh = torch.full_like(o_full, float("nan"))
    l_sh = torch.full_like(l_full, float("nan"))
    for bkv in [(0, 1), (1, 4)]:
        for qb in [(0, 50), (50, 128)]:
            run_capi(q, k, v, sel, BQ=BQ, shard=(bkv[0], bkv[1], qb[0], qb[1]), o=o_sh, lse=l_sh)
    torch.cuda.synchronize()
    assert torch.equal(o_full.view(torch.int16), o_sh.view(torch.int16))
    assert torch.equal(l_full, l_sh)


@pytest.mark.parametrize("Hq,Hkv,BQ,S,D", [(32, 2, 4, 1024, 128),   # 64-row tiles: the reference's BQ * G = 64
                                           (128, 1, 1, 512, 64),    # G = 128: one token per 128-row tile
                                           (16, 1, 8, 768, 64)])    # 128-row tiles
def test_row_owner_fills_cycle_counters(Hq, Hkv, BQ, S, D):
    """A non-empty cyc (the reference op's counters, nsa_v2.cu:69-71) no longer changes the kernel:
    the row-owner kernel runs, fills every query block's counters and matches the oracle."""
    B, KSEL, lp = 1, 6, 64
    d = capi.make_desc(q=256, k=256, v=256, sel=256, o=256, cyc=256, batch=B, heads_q=Hq, heads_kv=Hkv, seq_len=S,
                       d_qk=D, d_v=D, n_qblocks=(S + BQ - 1) // BQ, n_sel=KSEL, block_size=lp, q_block=BQ,
                       o_dtype=capi.DTYPE_F32)
    assert capi.plan(d)["n_cols"] == 128  # row-owner tiles
    q, k, v = make_qkv(B, Hq, Hkv, S, D, D, seed=S + Hq)
    sel = indices.perm_qblock(B, Hkv, S, KSEL, BQ, lp, seed=S)
    NQB = sel.shape[2]
    cyc = torch.zeros(NQB * B * Hkv * 2, dtype=torch.int64, device="cuda")
    o = ops.forward(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(sel).cuda(), lp, BQ, cyc)
    torch.cuda.synchronize()
    r, _ = oracle.forward(q, k, v, sel, lp, BQ)
    assert np.abs(o.cpu().numpy() - r).max() <= 1e-2
    c = cyc.cpu().numpy()
    assert (c[1::2] > 0).all() and (c >= 0).all()
