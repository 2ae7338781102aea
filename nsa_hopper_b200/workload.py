"""BASELINE workloads and their algorithmic work (the numerators of the roofline).

Configurations follow the reference's BASELINE list (configs 0-4 and the north-star shape).
Algorithmic work per (b, kvh, t) row, with G = Hq/Hkv:
  FLOPs  = G * 2 * (d_qk + d_v) * visible_keys(t)                 (QK^T + PV, valid keys only)
  bytes  = gathered K/V: n_blocks(t) * block * (d_qk + d_v) * 2    (every selected block that has a
           visible key, counted once per token with no cross-token reuse)
         + Q (G*d_qk*2) + O bf16 (G*d_v*2) + LSE (G*4) + indices (KSEL*4 per query block)
"""
from __future__ import annotations

import dataclasses
from typing import Dict, Optional

import numpy as np

from . import indices


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    B: int
    T: int
    Hq: int
    Hkv: int
    d_qk: int
    d_v: int
    block: int
    n: int
    rule: str
    BQ: int = 1
    n_seqs: int = 0  # > 0: varlen batch packed into T tokens (B == 1)

    @property
    def G(self) -> int:
        return self.Hq // self.Hkv


CONFIGS: Dict[str, Workload] = {
    "cfg0": Workload("cfg0", 1, 1024, 16, 1, 64, 64, 64, 8, "rule0"),
    "cfg1": Workload("cfg1", 1, 8192, 64, 4, 128, 128, 64, 16, "rule0"),
    "cfg2": Workload("cfg2", 4, 32768, 64, 4, 128, 128, 64, 16, "rule0_reuse"),
    "cfg3": Workload("cfg3", 1, 65536, 64, 4, 192, 128, 64, 16, "rule3"),
    "cfg4": Workload("cfg4", 1, 0, 32, 8, 128, 128, 64, 16, "varlen_rule0", n_seqs=16),
    "ns": Workload("ns", 1, 65536, 64, 4, 128, 128, 64, 16, "rule0"),
}


def varlen_setup(w: Workload, seed: int = 0):
    lens = indices.varlen_lengths(w.n_seqs, 256, 16384, seed)
    return lens, indices.cu_seqlens_of(lens)


def make_indices(w: Workload, seed: int = 0, B: Optional[int] = None) -> np.ndarray:
    B = w.B if B is None else B
    if w.rule == "varlen_rule0":
        lens, _ = varlen_setup(w, seed)
        return indices.varlen_rule0(lens, w.Hkv, w.n, w.block, seed)
    return indices.generate(w.rule, B=B, Hkv=w.Hkv, T=w.T, n=w.n, block=w.block, seed=seed)


def _distinct_visible(sel: np.ndarray, T: int, block: int, cu_seqlens: Optional[np.ndarray]):
    """Per (b*Hkv+kvh, t, entry): is the entry the first occurrence of a block that holds a
    visible key, and how many keys of it are visible.  Per-token selection (BQ == 1)."""
    B, Hkv, NQB, KSEL = sel.shape
    assert NQB == T
    s = sel.reshape(B * Hkv, T, KSEL).astype(np.int64)
    t = np.arange(T, dtype=np.int64)
    if cu_seqlens is None:
        seq0 = np.zeros(T, dtype=np.int64)
        end = np.full(T, T, dtype=np.int64)
    else:
        cu = np.asarray(cu_seqlens, dtype=np.int64)
        sid = np.searchsorted(cu, t, side="right") - 1
        seq0, end = cu[sid], cu[sid + 1]
    nblk = (end - seq0 + block - 1) // block
    start = seq0[None, :, None] + s * block
    valid = (s >= 0) & (s < nblk[None, :, None]) & (start <= t[None, :, None]) & (start < end[None, :, None])
    key = np.where(valid, s, -1)
    order = np.argsort(key, axis=-1, kind="stable")
    srt = np.take_along_axis(key, order, -1)
    first_sorted = (srt >= 0) & np.concatenate([np.ones_like(srt[..., :1], dtype=bool), srt[..., 1:] != srt[..., :-1]], -1)
    first = np.zeros_like(first_sorted)
    np.put_along_axis(first, order, first_sorted, -1)
    last_key = np.minimum(t[None, :, None], end[None, :, None] - 1)
    nvis = np.clip(last_key - start + 1, 0, block)
    return first, np.where(first, nvis, 0)


def gathered_blocks(sel: np.ndarray, T: int, block: int, cu_seqlens: Optional[np.ndarray] = None) -> np.ndarray:
    """Distinct selected blocks holding at least one visible key, per (b*Hkv+kvh, t): int32 [B*Hkv, T]."""
    first, _ = _distinct_visible(sel, T, block, cu_seqlens)
    return first.sum(-1).astype(np.int32)


def visible_keys(sel: np.ndarray, T: int, block: int, cu_seqlens: Optional[np.ndarray] = None) -> np.ndarray:
    """Keys each query token attends to, per (b*Hkv+kvh, t): int32 [B*Hkv, T]."""
    _, nvis = _distinct_visible(sel, T, block, cu_seqlens)
    return nvis.sum(-1).astype(np.int32)


def algorithmic_work(w: Workload, sel: np.ndarray, T: Optional[int] = None,
                     cu_seqlens: Optional[np.ndarray] = None) -> Dict[str, float]:
    """FLOPs and bytes of one full forward over `sel` ([B,Hkv,T,KSEL], per-token selection)."""
    T = w.T if T is None else T
    B = sel.shape[0]
    G = w.G
    first, nvis = _distinct_visible(sel, T, w.block, cu_seqlens)
    keys = nvis.astype(np.float64).sum()
    flops = G * 2.0 * (w.d_qk + w.d_v) * keys
    nblk = first.astype(np.float64).sum()
    kv_bytes = nblk * w.block * (w.d_qk + w.d_v) * 2.0
    rows = B * w.Hkv * T
    q_bytes = rows * G * w.d_qk * 2.0
    o_bytes = rows * G * w.d_v * 2.0
    lse_bytes = rows * G * 4.0
    idx_bytes = sel.size * 4.0
    return {
        "flops": flops,
        "kv_bytes": kv_bytes,
        "bytes": kv_bytes + q_bytes + o_bytes + lse_bytes + idx_bytes,
        "q_bytes": q_bytes,
        "o_bytes": o_bytes,
        "tokens": float(B * T),
        "visible_keys": keys,
        "gathered_blocks": nblk,
    }


def rect_work(w: Workload, sel: np.ndarray, rects, T: Optional[int] = None,
              cu_seqlens: Optional[np.ndarray] = None) -> Dict[str, float]:
    """algorithmic_work restricted to the (bkv_begin, bkv_end, t_begin, t_end) rectangles of a
    shard: the FLOPs, gathered K/V bytes and all bytes of the rows the rectangles cover."""
    T = w.T if T is None else T
    G = w.G
    first, nvis = _distinct_visible(sel, T, w.block, cu_seqlens)
    keys_row = nvis.sum(-1).astype(np.float64)   # [B*Hkv, T]
    blk_row = first.sum(-1).astype(np.float64)
    out = {"flops": 0.0, "kv_bytes": 0.0, "bytes": 0.0, "tokens": 0.0, "rows": 0.0}
    for b0, b1, t0, t1 in rects:
        keys = keys_row[b0:b1, t0:t1].sum()
        nblk = blk_row[b0:b1, t0:t1].sum()
        rows = (b1 - b0) * (t1 - t0)
        kv = nblk * w.block * (w.d_qk + w.d_v) * 2.0
        out["flops"] += G * 2.0 * (w.d_qk + w.d_v) * keys
        out["kv_bytes"] += kv
        out["bytes"] += kv + rows * G * (w.d_qk * 2.0 + w.d_v * 2.0 + 4.0) + rows * w.n * 4.0
        out["rows"] += rows
    return out
