"""Index generators, algorithmic work accounting and the multi-GPU shard planner (CPU only)."""
import numpy as np
import pytest

import oracle
from nsa_hopper_b200 import indices, shard, workload


def _check_rule0_rows(sel, T, n, block=64, fixed_back=1):
    t = np.arange(T)
    cur = t // block
    for r in sel.reshape(-1, T, n):
        assert (r[:, 0] == 0).all()
        valid = r >= 0
        assert (valid.sum(-1) == np.minimum(n, cur + 1)).all()
        assert (np.where(valid, r, 0).max(-1) <= cur).all()
        for row in r[:: max(1, T // 97)]:
            v = row[row >= 0]
            assert len(set(v.tolist())) == len(v)
        for d in range(fixed_back):
            ok = cur - d > 0
            assert np.array([cur[i] - d in r[i] for i in np.nonzero(ok)[0]]).all()


def test_rule0_properties():
    T, n = 3000, 16
    _check_rule0_rows(indices.rule0(2, 3, T, n, seed=1), T, n)


def test_rule3_properties():
    T, n = 3000, 16
    _check_rule0_rows(indices.rule3(1, 2, T, n, seed=2), T, n, fixed_back=2)


def test_rule0_is_deterministic():
    assert np.array_equal(indices.rule0(1, 2, 700, 8, seed=3), indices.rule0(1, 2, 700, 8, seed=3))
    assert not np.array_equal(indices.rule0(1, 2, 700, 8, seed=3), indices.rule0(1, 2, 700, 8, seed=4))


def test_reuse_rule_copies_previous_rows():
    sel = indices.rule0_reuse(1, 2, 4000, 16, seed=5)
    same = (sel[..., 1:, :] == sel[..., :-1, :]).all(-1)
    # past t = 1024 rows are random, so repeats are the injected 30% copies
    frac = same[..., 1024:].mean()
    assert 0.27 < frac < 0.33


def test_perm_qblock_matches_reference_rule():
    sel = indices.perm_qblock(1, 2, 512, 4, 16, 64, seed=0)
    for qb in range(sel.shape[2]):
        avail = max(1, (qb * 16) // 64 + 1)
        k = min(4, avail)
        row = sel[0, 0, qb]
        assert (row[k:] == -1).all() and sorted(row[:k].tolist()) == sorted(set(row[:k].tolist()))
        assert row[:k].max() < avail


def test_varlen_lengths_in_range():
    lens = indices.varlen_lengths(16, 256, 16384, seed=0)
    assert len(lens) == 16 and lens.min() >= 256 and lens.max() <= 16384


def test_visible_keys_matches_oracle_counts():
    rng = np.random.default_rng(0)
    T = 700
    sel = rng.integers(-2, 14, size=(2, 2, T, 7)).astype(np.int32)
    np.testing.assert_array_equal(workload.visible_keys(sel, T, 64), oracle.count_keys(sel, T, 64, 1))
    lens = [100, 400, 200]
    cu = indices.cu_seqlens_of(lens)
    s2 = indices.varlen_rule0(lens, 2, 9, 64, seed=1)
    np.testing.assert_array_equal(workload.visible_keys(s2, 700, 64, cu), oracle.count_keys(s2, 700, 64, 1, cu_seqlens=cu))


def test_north_star_work_matches_survey_figures():
    w = workload.CONFIGS["ns"]
    sel = workload.make_indices(w, seed=0)
    work = workload.algorithmic_work(w, sel)
    assert abs(work["flops"] / 1e12 - 2.115) < 0.01      # F = 2.115 TFLOP
    assert abs(work["bytes"] / 1e9 - 138.6) < 0.5        # gathered K/V + Q + O + LSE + idx = 138.6 GB


@pytest.mark.parametrize("B,Hkv,T,world", [(1, 4, 65536, 1), (1, 4, 65536, 2), (1, 4, 65536, 4), (1, 4, 65536, 8),
                                           (4, 4, 32768, 8), (1, 4, 1000, 3), (2, 8, 777, 5)])
def test_shard_plan_covers_every_row_once(B, Hkv, T, world):
    plans = shard.plan(B, Hkv, T, world)
    assert len(plans) == world
    cover = np.zeros((B * Hkv, T), np.int32)
    for rects in plans:
        for b0, b1, q0, q1 in rects:
            cover[b0:b1, q0:q1] += 1
    assert (cover == 1).all()
    if world <= 8 and (B * Hkv) % world == 0 or world % (B * Hkv) == 0:
        assert all(len(r) == 1 for r in plans)
    cost = shard.token_cost(T)
    loads = [sum(cost[q0:q1].sum() * (b1 - b0) for b0, b1, q0, q1 in r) for r in plans]
    assert max(loads) <= 1.02 * (sum(loads) / world) + cost.max()


def _cover_ok(B, Hkv, T, plans):
    cover = np.zeros((B * Hkv, T), np.int32)
    for rects in plans:
        assert rects, "a rank received no rows"
        for b0, b1, q0, q1 in rects:
            assert 0 <= b0 < b1 <= B * Hkv and 0 <= q0 < q1 <= T, (b0, b1, q0, q1)
            cover[b0:b1, q0:q1] += 1
    return (cover == 1).all()


def test_balanced_cuts_skewed_costs_stay_in_range():
    """Skewed costs must not push cuts past the end (non-empty, increasing ranges)."""
    cuts = shard._balanced_cuts(np.array([1.0, 1.0, 1.0, 100.0]), 4)
    assert cuts == [0, 1, 2, 3, 4]
    assert _cover_ok(1, 1, 3, shard.plan(1, 1, 3, 3))
    with pytest.raises(ValueError):
        shard.plan(1, 1, 3, 4)


try:
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=200, deadline=None)
    @given(B=st.integers(1, 4), Hkv=st.integers(1, 8), T=st.integers(1, 300), world=st.integers(1, 40),
           top_n=st.integers(1, 16), block=st.sampled_from([1, 7, 64]))
    def test_shard_plan_property_every_row_once(B, Hkv, T, world, top_n, block):
        """Property: whenever a plan exists, its rectangles are in range, non-empty, and cover every
        (batch*KV-head, token) row exactly once."""
        if world > B * Hkv * T:
            with pytest.raises(ValueError):
                shard.plan(B, Hkv, T, world, top_n=top_n, block=block)
            return
        plans = shard.plan(B, Hkv, T, world, top_n=top_n, block=block)
        assert len(plans) == world
        assert _cover_ok(B, Hkv, T, plans)
except ImportError:  # pragma: no cover - hypothesis is optional
    pass
