"""Seeded selection-index generators for the benchmark and test workloads.

Block ids are in units of the selection block (64 keys in every BASELINE config); rows are
padded with -1 (the reference's padding value, ref_only.py:9-12, test_v2.py:17-20).  All
generators use numpy's PCG64 so the same seed gives the same indices on every host.

Rules (per (batch, KV head, query token t), cur = t // block):
  rule0        block 0 and block cur, the rest drawn uniformly without replacement from the
               blocks in between; min(n, cur + 1) entries (1, NS, 4).
  rule0_reuse  rule0, except that each token with probability ``reuse_p`` copies the row of
               token t-1 (reuse_p = 0.3).
  rule3        block 0, cur-1 and cur plus random blocks in between.
  perm_qblock  the reference tests' rule (test_v0.py:36-40, test_v2.py:17-20): per query block
               qb, a random permutation prefix of the causally visible blocks.
"""
from __future__ import annotations

from typing import Optional, Sequence

import numpy as np


def _floyd_sample(rng: np.random.Generator, m: np.ndarray, k: int) -> np.ndarray:
    """Uniform k-subsets of range(m[r]) for every row r with m[r] >= k (Floyd's algorithm,
    vectorised over rows).  Returns int64 [rows, k] in draw order."""
    rows = m.shape[0]
    out = np.empty((rows, k), dtype=np.int64)
    for i in range(k):
        j = m - k + i  # candidate range [0, j]
        t = np.floor(rng.random(rows) * (j + 1)).astype(np.int64)
        t = np.minimum(t, j)
        if i:
            dup = (out[:, :i] == t[:, None]).any(axis=1)
            t = np.where(dup, j, t)
        out[:, i] = t
    return out


def _fixed_plus_random(rng: np.random.Generator, T: int, n: int, block: int, n_fixed_back: int) -> np.ndarray:
    """Rows for one (batch, head): block 0, the `n_fixed_back` blocks ending at cur, then
    uniform picks from the blocks strictly between; int32 [T, n]."""
    t = np.arange(T, dtype=np.int64)
    cur = t // block
    out = np.full((T, n), -1, dtype=np.int32)
    # fixed blocks: 0, cur - n_fixed_back + 1 .. cur (deduplicated, kept in that order)
    fixed = [np.zeros(T, dtype=np.int64)] + [cur - d for d in range(n_fixed_back - 1, -1, -1)]
    col = np.zeros(T, dtype=np.int64)
    taken = []
    for f in fixed:
        ok = f >= 0
        for prev in taken:
            ok &= f != prev
        ok &= col < n
        out[np.arange(T)[ok], col[ok]] = f[ok]
        col += ok
        taken.append(np.where(ok, f, -1))
    # random part from blocks 1 .. cur - n_fixed_back (inclusive)
    lo = 1
    hi = cur - n_fixed_back  # inclusive upper bound of the random range
    m = np.maximum(hi - lo + 1, 0)
    want = np.minimum(n - col, m)
    # rows that take every candidate
    all_rows = np.nonzero((want == m) & (m > 0))[0]
    for r in all_rows:
        c = int(col[r])
        vals = np.arange(lo, hi[r] + 1)
        out[r, c:c + len(vals)] = vals
    # rows that sample
    samp = np.nonzero(want < m)[0]
    if samp.size:
        kk = int(want[samp].max())
        assert (want[samp] == kk).all()  # = n - #fixed once cur is large enough
        picks = _floyd_sample(rng, m[samp], kk) + lo
        cs = col[samp]
        for i in range(kk):
            out[samp, cs + i] = picks[:, i]
    return out


def rule0(B: int, Hkv: int, T: int, n: int, block: int = 64, seed: int = 0) -> np.ndarray:
    """int32 [B, Hkv, T, n]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return np.stack([np.stack([_fixed_plus_random(rng, T, n, block, 1) for _ in range(Hkv)]) for _ in range(B)])


def rule3(B: int, Hkv: int, T: int, n: int, block: int = 64, seed: int = 0) -> np.ndarray:
    """Block 0 plus the two most recent blocks, the rest random; int32 [B, Hkv, T, n]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return np.stack([np.stack([_fixed_plus_random(rng, T, n, block, 2) for _ in range(Hkv)]) for _ in range(B)])


def rule0_reuse(B: int, Hkv: int, T: int, n: int, block: int = 64, seed: int = 0, reuse_p: float = 0.3) -> np.ndarray:
    """rule0 where each token copies token t-1's row with probability reuse_p."""
    sel = rule0(B, Hkv, T, n, block, seed)
    rng = np.random.Generator(np.random.PCG64(seed + 0x5EED))
    reuse = rng.random((B, Hkv, T)) < reuse_p
    reuse[..., 0] = False
    # source token: the last non-reusing token at or before t
    t = np.arange(T)
    src = np.where(reuse, -1, t[None, None, :])
    src = np.maximum.accumulate(src, axis=-1)
    return np.take_along_axis(sel, src[..., None].astype(np.int64), axis=2).astype(np.int32)


def varlen_rule0(seq_lens: Sequence[int], Hkv: int, n: int, block: int = 64, seed: int = 0) -> np.ndarray:
    """rule0 relative to each sequence start, packed: int32 [1, Hkv, sum(seq_lens), n]."""
    rng_seeds = np.random.Generator(np.random.PCG64(seed)).integers(0, 2**31 - 1, size=len(seq_lens))
    parts = [rule0(1, Hkv, int(L), n, block, int(s))[0] for L, s in zip(seq_lens, rng_seeds)]
    return np.concatenate(parts, axis=1)[None]


def varlen_lengths(n_seqs: int = 16, lo: int = 256, hi: int = 16384, seed: int = 0) -> np.ndarray:
    """Sequence lengths drawn log-uniformly from [lo, hi]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return np.exp(rng.uniform(np.log(lo), np.log(hi), size=n_seqs)).astype(np.int64)


def perm_qblock(B: int, Hkv: int, S: int, KSEL: int, BQ: int, LP: int, seed: int = 7,
                heads_share: bool = True) -> np.ndarray:
    """The reference tests' per-query-block rule: sel[:, :, qb, :k] = randperm(avail)[:k] with
    avail = max(1, (qb*BQ)//LP + 1), k = min(KSEL, avail), -1 padded (test_v2.py:17-20).  The
    reference writes the same row for every (b, kvh) (``sel[:,:,qb,:k] = ...``); set
    ``heads_share=False`` for independent rows."""
    rng = np.random.Generator(np.random.PCG64(seed))
    NQB = (S + BQ - 1) // BQ
    sel = np.full((B, Hkv, NQB, KSEL), -1, dtype=np.int32)
    reps = 1 if heads_share else B * Hkv
    for r in range(reps):
        for qb in range(NQB):
            avail = max(1, (qb * BQ) // LP + 1)
            k = min(KSEL, avail)
            row = rng.permutation(avail)[:k]
            if heads_share:
                sel[:, :, qb, :k] = row
            else:
                sel[r // Hkv, r % Hkv, qb, :k] = row
    return sel


def cu_seqlens_of(seq_lens: Sequence[int]) -> np.ndarray:
    return np.concatenate([[0], np.cumsum(np.asarray(seq_lens, dtype=np.int64))]).astype(np.int32)


def generate(rule: str, *, B: int, Hkv: int, T: int, n: int, block: int = 64, seed: int = 0,
             seq_lens: Optional[Sequence[int]] = None) -> np.ndarray:
    if rule == "rule0":
        return rule0(B, Hkv, T, n, block, seed)
    if rule == "rule0_reuse":
        return rule0_reuse(B, Hkv, T, n, block, seed)
    if rule == "rule3":
        return rule3(B, Hkv, T, n, block, seed)
    if rule == "varlen_rule0":
        assert seq_lens is not None and B == 1
        return varlen_rule0(seq_lens, Hkv, n, block, seed)
    raise ValueError(rule)
