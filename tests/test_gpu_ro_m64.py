"""64-row tiles of the row-owner kernel (G * tokens per tile = 64, the reference's BQ * G = 64
mode) computed by M = 64 MMAs: rows in TMEM lanes 0-15 of each 32-lane quarter, 16-lane access
shapes in the softmax.  Checked against the oracle, against the 128-row padded form of the same
tiles (NSA_DEBUG_RO_PAD128), on the exact mask probe, with a high dynamic range that makes the
lazy O rescale fire on some rows of a warp and not on others, and on the window / compressed
branches with 64-row tiles."""
import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import capi, indices, nsa, ops
from tests.helpers import compare, make_qkv, run_capi

pytestmark = pytest.mark.gpu


def _is_64_row_tile(Hq, Hkv, BQ, D, f32):
    d = capi.make_desc(q=256, k=256, v=256, sel=256, o=256, batch=1, heads_q=Hq, heads_kv=Hkv, seq_len=4096,
                       d_qk=D, d_v=D, n_qblocks=(4096 + BQ - 1) // BQ, n_sel=4, block_size=64, q_block=BQ,
                       o_dtype=capi.DTYPE_F32 if f32 else capi.DTYPE_BF16)
    p = capi.plan(d)
    return p["n_cols"] == 128 and p["q_per_unit"] * (Hq // Hkv) == 64


SHAPES = [
    # B, Hq, Hkv, S, D, KSEL, BQ, lp, f32
    (1, 32, 2, 1000, 128, 16, 4, 64, True),     # G = 16, BQ = 4: the reference sweep's head layout
    (2, 64, 2, 777, 64, 6, 2, 64, False),       # G = 32, bf16 O, ragged T
    (1, 64, 1, 640, 128, 8, 1, 64, True),       # G = 64, one token per tile
    (1, 16, 2, 1111, 64, 5, 8, 128, True),      # G = 8, l' = 128
    (1, 8, 2, 2048, 128, 16, 16, 64, False),    # G = 4
    (1, 4, 4, 512, 64, 4, 64, 128, True),       # G = 1, 64 tokens per tile
    (1, 64, 2, 1500, 128, 8, 2, 256, True),     # G = 32, l' = 256
]


@pytest.mark.parametrize("B,Hq,Hkv,S,D,KSEL,BQ,lp,f32", SHAPES)
def test_m64_matches_oracle_and_padded_form(B, Hq, Hkv, S, D, KSEL, BQ, lp, f32):
    assert _is_64_row_tile(Hq, Hkv, BQ, D, f32)
    q, k, v = make_qkv(B, Hq, Hkv, S, D, D, seed=S + 7 * KSEL)
    sel = torch.from_numpy(indices.perm_qblock(B, Hkv, S, KSEL, BQ, lp, seed=S + 1, heads_share=False))
    o, lse = run_capi(q, k, v, sel, BQ=BQ, l_prime=lp, out_f32=f32)
    o_pad, lse_pad = run_capi(q, k, v, sel, BQ=BQ, l_prime=lp, out_f32=f32, debug_flags=capi.NSA_DEBUG_RO_PAD128)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel.numpy(), lp, BQ)
    compare(o, lse, o_ref, lse_ref)
    compare(o_pad, lse_pad, o_ref, lse_ref)
    # the two forms differ only in the order the row sums are accumulated
    fin = torch.isfinite(lse_pad)
    assert torch.equal(fin, torch.isfinite(lse))
    assert (lse[fin] - lse_pad[fin]).abs().max().item() <= 1e-5 * max(1.0, lse_pad[fin].abs().max().item())
    tol = 1e-5 if f32 else 8e-3
    assert (o.float() - o_pad.float()).abs().max().item() <= tol


def test_m64_mask_probe_counts_exact():
    """Q = 0: exp(LSE) is the exact number of visible keys of every row of the 64-row tiles
    (causal edge of the diagonal block, ragged end, -1 padding)."""
    B, Hq, Hkv, T, D, n, BQ = 1, 32, 2, 1100, 128, 16, 4
    _, k, _ = make_qkv(B, Hq, Hkv, T, D, D, seed=31)
    q = torch.zeros(B, Hq, T, D, dtype=torch.bfloat16)
    v = torch.zeros(B, Hkv, T, D, dtype=torch.bfloat16)
    sel = indices.perm_qblock(B, Hkv, T, n, BQ, 64, seed=31, heads_share=False)
    sel[:, :, ::9, 3:] = -1
    assert _is_64_row_tile(Hq, Hkv, BQ, D, True)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), BQ=BQ, out_f32=True)
    torch.cuda.synchronize()
    counts = oracle.count_keys(sel, T, 64, BQ).reshape(B, Hkv, T)
    cnt = np.repeat(counts, Hq // Hkv, axis=1).astype(np.float64)
    got = np.exp(lse.cpu().numpy().astype(np.float64))
    assert np.array_equal(np.rint(got), cnt)
    assert torch.count_nonzero(o).item() == 0


@pytest.mark.parametrize("amp", [6.0, 12.0])
def test_m64_rescale_some_rows_of_a_warp(amp):
    """Queries scaled by `amp`: scores spread over tens of units of log2, so the running max of
    some rows of a warp grows by more than 2^8 between chunks while others' does not; the
    warp-uniform rescale with a per-row factor must match the oracle."""
    B, Hq, Hkv, T, D, n, BQ = 1, 32, 2, 1024, 64, 16, 4
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, seed=int(amp))
    q = (q.float() * amp).to(torch.bfloat16)
    sel = indices.perm_qblock(B, Hkv, T, n, BQ, 64, seed=5, heads_share=False)
    o, lse = run_capi(q, k, v, torch.from_numpy(sel), BQ=BQ, out_f32=True)
    torch.cuda.synchronize()
    o_ref, lse_ref = oracle.forward(q, k, v, sel, 64, BQ)
    compare(o, lse, o_ref, lse_ref)


@pytest.mark.parametrize("T,window,D", [(1500, 128, 64), (2048, 512, 128)])
def test_m64_window_branch(T, window, D):
    """The window branch with 64-row tiles (q_block = 64 / G) on the M = 64 form."""
    B, Hq, Hkv = 1, 32, 2
    g = torch.Generator(device="cuda").manual_seed(T + 1)
    q = torch.randn(B, Hq, T, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    bq = 64 // (Hq // Hkv)
    sel = nsa.window_selection(B, Hkv, T, window, 64, q.device, bq)
    o, _ = ops.forward_ext(q, k, v, sel, 64, bq, window=window)
    ref = nsa.window_branch(q, k, v, window)
    torch.cuda.synchronize()
    assert (o - ref).abs().max().item() <= 2e-2


def test_m64_compressed_branch_accumulates():
    """The compressed key map with 64-row tiles, weighted and added into an existing O."""
    B, Hq, Hkv, T, D = 1, 16, 1, 1500, 64
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn(B, Hq, T, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, device="cuda", generator=g).to(torch.bfloat16)
    Kc, Vc = nsa.compress_kv(k, v, 32, 16)
    Kc, Vc = Kc.to(torch.bfloat16).contiguous(), Vc.to(torch.bfloat16).contiguous()
    bq = 64 // (Hq // Hkv)
    sel = nsa.compressed_selection(B, Hkv, T, Kc.shape[2], q.device, bq)
    ref = nsa.compressed_branch(q, Kc.float(), Vc.float())
    w = torch.tensor([0.5], device="cuda")
    base = torch.randn(B, Hq, T, D, device="cuda", generator=g)
    o, _ = ops.forward_ext(q, Kc, Vc, sel, 64, bq, key_map=1, out=base.clone(), weight=w, accumulate=True)
    torch.cuda.synchronize()
    assert (o - (base + 0.5 * ref)).abs().max().item() <= 1e-2
