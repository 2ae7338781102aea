"""The CPU oracle against the reference's golden fixtures and against its own invariants.

No GPU needed: this pins the checker that every GPU parity test relies on.
"""
import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import indices
from tests import golden_cases
from tests.helpers import make_qkv


@pytest.mark.parametrize("name", golden_cases.case_names())
def test_oracle_matches_reference_fixture(name):
    c = golden_cases.load(name)
    o, lse = oracle.forward(c["q"], c["k"], c["v"], c["sel"], c["LP"], c["BQ"])
    # fp64 restatement vs the reference's fp64: rounding-level agreement on every element
    np.testing.assert_allclose(golden_cases.rows_of(o, c["rows"]), c["o_rows"], rtol=0, atol=1e-10)
    np.testing.assert_allclose(golden_cases.checksums(o), c["checksums"], rtol=1e-10, atol=1e-8)
    fin = np.isfinite(c["lse"])
    assert (np.isfinite(lse) == fin).all()
    np.testing.assert_allclose(lse[fin], c["lse"][fin], rtol=0, atol=1e-10)


@pytest.mark.parametrize("name", ["token_cfg0", "qblock_g8_d128", "token_bigrow"])
def test_oracle_fp32_mode_close_to_reference(name):
    c = golden_cases.load(name)
    o, lse = oracle.forward(c["q"], c["k"], c["v"], c["sel"], c["LP"], c["BQ"], f32=True)
    np.testing.assert_allclose(golden_cases.rows_of(o, c["rows"]), c["o_rows"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(lse, c["lse"], rtol=1e-5, atol=1e-5)


def _small(seed=0, B=1, Hq=4, Hkv=2, T=300, D=64):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    return q, k, v


def test_padding_duplicates_and_scratch_id_select_nothing_new():
    q, k, v = _small()
    T = q.shape[2]
    nblk = (T + 63) // 64
    base = indices.rule0(1, 2, T, 4, 64, seed=3)
    o0, l0 = oracle.forward(q, k, v, base, 64, 1)
    extra = np.concatenate([base, np.full(base.shape[:-1] + (3,), -1, np.int32)], -1)
    extra[..., 4] = base[..., 0]          # duplicate of an entry already present
    extra[..., 5] = nblk                  # the reference's discarded scratch column
    extra[..., 6] = -7                    # any negative value is padding
    o1, l1 = oracle.forward(q, k, v, extra, 64, 1)
    np.testing.assert_array_equal(o0, o1)
    np.testing.assert_array_equal(l0, l1)


def test_out_of_range_block_raises_in_strict_mode_like_the_reference():
    q, k, v = _small()
    sel = indices.rule0(1, 2, q.shape[2], 4, 64, seed=1)
    sel[0, 0, 10, 3] = 1000
    with pytest.raises(IndexError):
        oracle.forward(q, k, v, sel, 64, 1, strict=True)
    o, _ = oracle.forward(q, k, v, sel, 64, 1)  # non-strict: the entry selects nothing
    assert np.isfinite(o).all()


def test_empty_rows_give_zero_and_minus_inf():
    q, k, v = _small()
    sel = np.full((1, 2, q.shape[2], 3), -1, np.int32)
    sel[:, :, ::2, 0] = 0
    o, lse = oracle.forward(q, k, v, sel, 64, 1)
    assert (o[:, :, 1::2] == 0).all() and np.isneginf(lse[:, :, 1::2]).all()
    assert np.isfinite(lse[:, :, ::2]).all()


def test_mask_probe_q_zero_counts_keys():
    q, k, v = _small(T=257)
    q = torch.zeros_like(q)
    sel = indices.rule0(1, 2, 257, 5, 64, seed=4)
    _, lse = oracle.forward(q, k, v, sel, 64, 1)
    cnt = oracle.count_keys(sel, 257, 64, 1).reshape(1, 2, 257).repeat(2, axis=1)
    np.testing.assert_allclose(np.exp(lse), cnt, rtol=1e-12)


def test_varlen_equals_separate_sequences():
    lens = [100, 257, 64]
    Hq, Hkv, D = 4, 2, 64
    T = sum(lens)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, Hq, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(1, Hkv, T, D, generator=g).to(torch.bfloat16)
    v = torch.randn(1, Hkv, T, D, generator=g).to(torch.bfloat16)
    sel = indices.varlen_rule0(lens, Hkv, 6, 64, seed=5)
    cu = indices.cu_seqlens_of(lens)
    o, lse = oracle.forward(q, k, v, sel, 64, 1, cu_seqlens=cu)
    for s in range(len(lens)):
        a, b = cu[s], cu[s + 1]
        o_s, l_s = oracle.forward(q[:, :, a:b], k[:, :, a:b], v[:, :, a:b], sel[:, :, a:b], 64, 1)
        np.testing.assert_array_equal(o[:, :, a:b], o_s)
        np.testing.assert_array_equal(lse[:, :, a:b], l_s)


def test_row_ranges_compose():
    q, k, v = _small(B=2)
    sel = indices.rule0(2, 2, q.shape[2], 4, 64, seed=6)
    o, l = oracle.forward(q, k, v, sel, 64, 1)
    o2 = np.full_like(o, np.nan)
    l2 = np.full_like(l, np.nan)
    for bkv in [(0, 1), (1, 4)]:
        for tr in [(0, 123), (123, q.shape[2])]:
            oracle.forward(q, k, v, sel, 64, 1, bkv_range=bkv, t_range=tr, out=o2, lse_out=l2)
    np.testing.assert_array_equal(o, o2)
    np.testing.assert_array_equal(l, l2)


def test_window_form_equals_full_rows():
    """oracle.forward_window (Q/O/LSE holding only the computed token rows) gives exactly the
    rows of the full-array form."""
    q, k, v = make_qkv(2, 8, 2, 700, 64, 32, seed=3)
    sel = indices.rule0(2, 2, 700, 8, 64, seed=3)
    o, l = oracle.forward(q, k, v, sel, 64, 1, f32=True)
    ow, lw = oracle.forward_window(q[:, :, 300:450].contiguous(), k, v, sel, 64, 1, (300, 450))
    assert np.array_equal(ow, o[:, :, 300:450]) and np.array_equal(lw, l[:, :, 300:450])
    ow, lw = oracle.forward_window(q[:, :, 650:].contiguous(), k, v, sel, 64, 1, (650, 700), bkv_range=(3, 4),
                                   f32=False)
    o64, l64 = oracle.forward(q, k, v, sel, 64, 1)
    assert np.array_equal(ow[1, 4:], o64[1, 4:, 650:]) and np.isnan(ow[0]).all()
