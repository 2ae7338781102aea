"""TEST INFRASTRUCTURE ONLY: numpy fp64 restatement of the gradients of the selected-branch
attention, the checker of the backward kernel (never the product; nothing in ``nsa_hopper_b200``
imports it).

The reference has no backward pass (its README (2).md:85).  What is differentiated here is its
own selected-branch forward, ``ref_only.ref_selected`` (ref_only.py:2-20), for per-token
selection (BQ = 1): the key mask is built the same way (entries scattered into a per-token
keep mask over ``n_blk`` blocks plus a scratch column that absorbs -1 and ``n_blk``, expanded to
``l_prime`` keys each, intersected with the causal mask), the scores are
``q.k / sqrt(d)`` and the softmax of a row without a visible key is 0 (``nan_to_num``).  The
gradient of that function, for an upstream gradient dO, is
    P = softmax(S), O = P V, D = rowsum(dO * O), dS = P * (dO V^T - D),
    dQ = scale dS K,  dK = scale dS^T Q,  dV = P^T dO,
summed over the G query heads that share a KV head for dK and dV.  ``tests/golden/bwd_*.npz``
hold autograd results of the reference's own function (``tests/golden/make_golden.py``), which
pin this restatement (``tests/test_oracle_backward.py``).
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np


def _f64(x) -> np.ndarray:
    if hasattr(x, "detach"):  # a torch tensor (bf16 included; the conversion to fp64 is exact)
        return x.detach().cpu().double().numpy()
    return np.asarray(x, dtype=np.float64)


def key_mask(sel_rows: np.ndarray, T: int, l_prime: int) -> np.ndarray:
    """bool [T, T]: key p is visible to token t (ref_only.py:9-16 with BQ = 1)."""
    n_blk = (T + l_prime - 1) // l_prime
    sel_rows = np.asarray(sel_rows, dtype=np.int64)
    keep = np.zeros((T, n_blk + 1), dtype=bool)
    idx = np.where((sel_rows >= 0) & (sel_rows <= n_blk), sel_rows, n_blk)
    keep[np.arange(T)[:, None], idx] = True
    tok = np.repeat(keep[:, :n_blk], l_prime, axis=1)[:, :T]
    return tok & np.tril(np.ones((T, T), dtype=bool))


def backward(q, k, v, sel, l_prime: int, d_o, scale: Optional[float] = None
             ) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """dQ [B,Hq,T,d], dK, dV [B,Hkv,T,d] (fp64) of the selected branch for upstream gradient d_o."""
    q, k, v, d_o = _f64(q), _f64(k), _f64(v), _f64(d_o)
    sel = np.asarray(sel)
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    s = (1.0 / np.sqrt(D)) if scale is None else float(scale)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for b in range(B):
        for kvh in range(Hkv):
            mask = key_mask(sel[b, kvh], T, l_prime)
            kb, vb = k[b, kvh], v[b, kvh]
            for g in range(G):
                h = kvh * G + g
                S = np.where(mask, (q[b, h] @ kb.T) * s, -np.inf)
                m = S.max(axis=-1, keepdims=True)
                m = np.where(np.isfinite(m), m, 0.0)
                E = np.exp(S - m)
                lsum = E.sum(axis=-1, keepdims=True)
                P = np.divide(E, lsum, out=np.zeros_like(E), where=lsum > 0)
                O = P @ vb
                dP = d_o[b, h] @ vb.T
                dS = P * (dP - (d_o[b, h] * O).sum(axis=-1, keepdims=True))
                dq[b, h] = s * (dS @ kb)
                dk[b, kvh] += s * (dS.T @ q[b, h])
                dv[b, kvh] += P.T @ d_o[b, h]
    return dq, dk, dv



def dq_rows(q, k, v, sel, l_prime: int, d_o, b: int, h: int, t0: int, t1: int,
            scale: Optional[float] = None) -> np.ndarray:
    """dQ[b, h, t0:t1] alone (fp64): a query row's gradient needs only its own row of the
    attention, so large problems can be checked on a token window."""
    G = q.shape[1] // k.shape[1]
    kvh = h // G
    T = k.shape[2]
    qh, doh = _f64(q[b, h, t0:t1]), _f64(d_o[b, h, t0:t1])
    kb, vb = _f64(k[b, kvh, :t1]), _f64(v[b, kvh, :t1])
    s = (1.0 / np.sqrt(qh.shape[-1])) if scale is None else float(scale)
    mask = key_mask(np.asarray(sel)[b, kvh], T, l_prime)[t0:t1, :t1]
    S = np.where(mask, (qh @ kb.T) * s, -np.inf)
    m = S.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    E = np.exp(S - m)
    lsum = E.sum(axis=-1, keepdims=True)
    P = np.divide(E, lsum, out=np.zeros_like(E), where=lsum > 0)
    O = P @ vb
    dS = P * (doh @ vb.T - (doh * O).sum(axis=-1, keepdims=True))
    return s * (dS @ kb)
