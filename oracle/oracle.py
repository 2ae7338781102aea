"""TEST INFRASTRUCTURE ONLY: ctypes wrapper around the C oracle (oracle/nsa_sel_oracle.c).

The oracle is the CPU restatement of the reference's selected-branch forward
(ref_only.py:2-20, nsa_reference.py:18-25) and is used exclusively as the checker by
tests/, by ``__graft_entry__.smoke()`` and by ``bench.py``'s CPU-baseline / reference arm.
Nothing in the ``nsa_hopper_b200`` package imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

ERR_ARG, ERR_INDEX, ERR_NOMEM = -1, -2, -3


def build() -> str:
    """Compile the oracle with its Makefile (idempotent); returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    p = ctypes.c_void_p
    i = ctypes.c_int
    common = [p, p, p, p, p, i, i, i, i, i, i, i, i, i, i, i, ctypes.c_double, i, i, i, i, i, p, p, i]
    lib.nsa_oracle_forward.argtypes = common
    lib.nsa_oracle_forward.restype = i
    lib.nsa_oracle_forward_f32.argtypes = common
    lib.nsa_oracle_forward_f32.restype = i
    lib.nsa_oracle_forward_window.argtypes = common
    lib.nsa_oracle_forward_window.restype = i
    lib.nsa_oracle_forward_window_f32.argtypes = common
    lib.nsa_oracle_forward_window_f32.restype = i
    lib.nsa_oracle_count_keys.argtypes = [p, p, i, i, i, i, i, i, i, i, p, i]
    lib.nsa_oracle_count_keys.restype = i
    _lib = lib
    return lib


def _bits(x) -> np.ndarray:
    """bf16 data as a contiguous uint16 numpy array (accepts torch bf16 tensors or uint16)."""
    if hasattr(x, "detach"):  # torch tensor
        import torch

        x = x.detach().to("cpu").contiguous()
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        return x.view(torch.int16).numpy().view(np.uint16)
    a = np.ascontiguousarray(x)
    if a.dtype != np.uint16:
        raise TypeError("expected bf16 bit patterns as uint16")
    return a


def _i32(x) -> np.ndarray:
    if hasattr(x, "detach"):
        x = x.detach().to("cpu").contiguous().numpy()
    return np.ascontiguousarray(x, dtype=np.int32)


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def default_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def forward(q, k, v, sel, l_prime: int, BQ: int, *, cu_seqlens=None, scale: float = 0.0, f32: bool = False,
            bkv_range: Optional[Tuple[int, int]] = None, t_range: Optional[Tuple[int, int]] = None,
            strict: bool = False, threads: Optional[int] = None, out=None, lse_out=None):
    """Selected-branch forward on the CPU.

    q [B,Hq,T,dqk], k [B,Hkv,T,dqk], v [B,Hkv,T,dv] as bf16 (torch) or uint16 bit patterns;
    sel int32 [B,Hkv,NQB,KSEL].  Returns (O [B,Hq,T,dv], LSE [B,Hq,T]) as float64 (float32 with
    ``f32``).  Only rows inside ``bkv_range`` x ``t_range`` are computed (others stay NaN unless
    ``out``/``lse_out`` are supplied).  ``strict`` mirrors the reference raising on a block id
    greater than the block count.
    """
    lib = _load()
    qb, kb, vb = _bits(q), _bits(k), _bits(v)
    s = _i32(sel)
    B, Hq, T, dqk = qb.shape
    Hkv, dv = kb.shape[1], vb.shape[3]
    NQB, KSEL = s.shape[2], s.shape[3]
    dt = np.float32 if f32 else np.float64
    o = out if out is not None else np.full((B, Hq, T, dv), np.nan, dtype=dt)
    lse = lse_out if lse_out is not None else np.full((B, Hq, T), np.nan, dtype=dt)
    cu = None if cu_seqlens is None else _i32(cu_seqlens)
    n_seqs = 0 if cu is None else len(cu) - 1
    b0, b1 = bkv_range if bkv_range is not None else (0, B * Hkv)
    t0, t1 = t_range if t_range is not None else (0, T)
    fn = lib.nsa_oracle_forward_f32 if f32 else lib.nsa_oracle_forward
    rc = fn(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(s), _ptr(cu), n_seqs, B, Hq, Hkv, T, dqk, dv, NQB, KSEL, l_prime, BQ,
            float(scale), b0, b1, t0, t1, 1 if strict else 0, _ptr(o), _ptr(lse),
            threads if threads else default_threads())
    if rc == ERR_INDEX:
        raise IndexError("selection holds a block id greater than the block count")
    if rc != 0:
        raise ValueError(f"oracle rejected the arguments (code {rc})")
    return o, lse


def forward_window(q_win, k, v, sel, l_prime: int, BQ: int, t_range: Tuple[int, int], *, cu_seqlens=None,
                   scale: float = 0.0, f32: bool = True, bkv_range: Optional[Tuple[int, int]] = None,
                   threads: Optional[int] = None):
    """``forward`` on the token rows ``t_range`` = [t0, t1) only, with ``q_win`` holding just those
    rows: q_win [B,Hq,t1-t0,dqk]; k, v and sel whole (T = k.shape[2]).  Returns (O [B,Hq,t1-t0,dv],
    LSE [B,Hq,t1-t0]) for the rows of ``bkv_range`` (others NaN); float32 by default."""
    lib = _load()
    qb, kb, vb = _bits(q_win), _bits(k), _bits(v)
    s = _i32(sel)
    B, Hq, nt, dqk = qb.shape
    Hkv, T, dv = kb.shape[1], kb.shape[2], vb.shape[3]
    t0, t1 = t_range
    if t1 - t0 != nt or not (0 <= t0 < t1 <= T):
        raise ValueError(f"q_win holds {nt} rows, t_range {t_range} for T={T}")
    NQB, KSEL = s.shape[2], s.shape[3]
    dt = np.float32 if f32 else np.float64
    o = np.full((B, Hq, nt, dv), np.nan, dtype=dt)
    lse = np.full((B, Hq, nt), np.nan, dtype=dt)
    cu = None if cu_seqlens is None else _i32(cu_seqlens)
    n_seqs = 0 if cu is None else len(cu) - 1
    b0, b1 = bkv_range if bkv_range is not None else (0, B * Hkv)
    fn = lib.nsa_oracle_forward_window_f32 if f32 else lib.nsa_oracle_forward_window
    rc = fn(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(s), _ptr(cu), n_seqs, B, Hq, Hkv, T, dqk, dv, NQB, KSEL, l_prime, BQ,
            float(scale), b0, b1, t0, t1, 0, _ptr(o), _ptr(lse), threads if threads else default_threads())
    if rc != 0:
        raise ValueError(f"oracle rejected the arguments (code {rc})")
    return o, lse


def count_keys(sel, T: int, l_prime: int, BQ: int, *, cu_seqlens=None, threads: Optional[int] = None) -> np.ndarray:
    """Visible keys per (b*Hkv+kvh, t) row: int32 [B*Hkv, T]."""
    lib = _load()
    s = _i32(sel)
    B, Hkv, NQB, KSEL = s.shape
    cu = None if cu_seqlens is None else _i32(cu_seqlens)
    n_seqs = 0 if cu is None else len(cu) - 1
    counts = np.zeros((B * Hkv, T), dtype=np.int32)
    rc = lib.nsa_oracle_count_keys(_ptr(s), _ptr(cu), n_seqs, B, Hkv, T, NQB, KSEL, l_prime, BQ, _ptr(counts),
                                   threads if threads else default_threads())
    if rc != 0:
        raise ValueError(f"oracle rejected the arguments (code {rc})")
    return counts
