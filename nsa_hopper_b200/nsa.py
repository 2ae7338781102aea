"""Full NSA forward around the B200 selected-branch kernel.

This is the caller the reference's ``validate.check(fn)`` drives (validate.py:12-28): the three
NSA branches and the learned gate of ``nsa_forward`` (nsa_reference.py:46-89).  On the GPU all
three attention branches run on the sm_100a kernel: the selected branch with the selection
kernel's (or the given) index rows, the sliding-window branch with per-token rows covering the
window and the kernel's window bound, the compressed branch over the mean-pooled keys with the
kernel's compressed key map.  The tensor-op functions below (``compressed_branch``,
``window_branch``, ``block_scores``, ``select_blocks``) restate the same branches for CPU tests
and cross-checks.  Semantics follow the reference line for line where it matters for results:

* compression: overlapping mean pooling of ``cmp_block`` keys every ``cmp_stride``
  (nsa_reference.py:5-16);
* compressed-branch mask: compressed key i is visible to query t iff
  ``linspace(0, S-1, n_cmp)[i] <= t`` in float32 (nsa_reference.py:62-64);
* block scores: group-summed queries against the compressed keys, summed into the selection
  block of each compressed key's linspace position, future blocks masked, top-n
  (nsa_reference.py:27-44, 70-71) -- on the GPU by the selection kernel (``ops.select_blocks``);
  ``block_scores``/``select_blocks`` below restate it with tensor ops (used on CPU and as a
  cross-check);
* sliding window: key s visible to query t iff ``0 <= t - s < window`` (nsa_reference.py:80-82);
* gate: 1/3 each, or ``sigmoid(gate_w)`` normalised (nsa_reference.py:84-89);
* fully masked rows give 0 (nsa_reference.py:24).

The dense branches are evaluated in query chunks so that memory stays O(chunk x keys).
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch


def compress_kv(K: torch.Tensor, V: torch.Tensor, block: int = 32, stride: int = 16
                ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Mean-pooled compressed keys and values [B, H, n_cmp, D] (fp32), n_cmp = (S-block)//stride+1."""
    B, H, S, D = K.shape
    n = max(0, (S - block) // stride + 1)
    if n == 0:
        return (K.new_zeros((B, H, 0, D), dtype=torch.float32), V.new_zeros((B, H, 0, V.shape[3]), dtype=torch.float32))
    Kc = K.float().unfold(2, block, stride)[:, :, :n].mean(-1)
    Vc = V.float().unfold(2, block, stride)[:, :, :n].mean(-1)
    return Kc, Vc


def compressed_positions(S: int, n_cmp: int, device) -> torch.Tensor:
    """``torch.linspace(0, S-1, n_cmp)`` in float32, computed on the CPU (as the reference's
    masks are) and moved to ``device``."""
    return torch.linspace(0, S - 1, n_cmp, dtype=torch.float32).to(device)


def _masked_attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor, scale: float) -> torch.Tensor:
    """softmax(q k^T * scale, masked) v with fully masked rows -> 0.  q [.., M, D], k/v [.., N, D]."""
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return torch.matmul(p, v)


def compressed_branch(Q: torch.Tensor, Kc: torch.Tensor, Vc: torch.Tensor, chunk: int = 1024) -> torch.Tensor:
    """Attention of every query over the compressed keys it may see (fp32 [B, Hq, S, d_v])."""
    B, Hq, S, D = Q.shape
    Hkv, n_cmp = Kc.shape[1], Kc.shape[2]
    G = Hq // Hkv
    out = torch.zeros(B, Hq, S, Vc.shape[3], dtype=torch.float32, device=Q.device)
    if n_cmp == 0:
        return out
    cpos = compressed_positions(S, n_cmp, Q.device)
    scale = 1.0 / (D ** 0.5)
    q5 = Q.float().view(B, Hkv, G, S, D)
    k5, v5 = Kc.unsqueeze(2), Vc.unsqueeze(2)
    for t0 in range(0, S, chunk):
        t1 = min(S, t0 + chunk)
        t = torch.arange(t0, t1, device=Q.device, dtype=torch.float32)
        mask = (cpos.view(1, -1) <= t.view(-1, 1)).view(1, 1, 1, t1 - t0, n_cmp)
        o = _masked_attend(q5[:, :, :, t0:t1], k5, v5, mask, scale)
        out[:, :, t0:t1] = o.reshape(B, Hq, t1 - t0, -1)
    return out


def window_branch(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, window: int, chunk: int = 1024) -> torch.Tensor:
    """Causal sliding-window attention, key s visible to query t iff 0 <= t - s < window."""
    B, Hq, S, D = Q.shape
    Hkv = K.shape[1]
    G = Hq // Hkv
    scale = 1.0 / (D ** 0.5)
    out = torch.zeros(B, Hq, S, V.shape[3], dtype=torch.float32, device=Q.device)
    q5 = Q.float().view(B, Hkv, G, S, D)
    k5, v5 = K.float().unsqueeze(2), V.float().unsqueeze(2)
    for t0 in range(0, S, chunk):
        t1 = min(S, t0 + chunk)
        s0 = max(0, t0 - window + 1)
        t = torch.arange(t0, t1, device=Q.device).view(-1, 1)
        s = torch.arange(s0, t1, device=Q.device).view(1, -1)
        d = t - s
        mask = ((d >= 0) & (d < window)).view(1, 1, 1, t1 - t0, t1 - s0)
        o = _masked_attend(q5[:, :, :, t0:t1], k5[:, :, :, s0:t1], v5[:, :, :, s0:t1], mask, scale)
        out[:, :, t0:t1] = o.reshape(B, Hq, t1 - t0, -1)
    return out


def block_scores(Q: torch.Tensor, Kc: torch.Tensor, l_prime: int, t_range: Optional[Tuple[int, int]] = None
                 ) -> torch.Tensor:
    """Selection-block importance [B, Hkv, T, n_blk] (fp32; future blocks -inf) for queries
    t in ``t_range``: group-summed queries against compressed keys, summed per block."""
    B, Hq, S, D = Q.shape
    Hkv, n_cmp = Kc.shape[1], Kc.shape[2]
    G = Hq // Hkv
    t0, t1 = t_range if t_range is not None else (0, S)
    n_blk = (S + l_prime - 1) // l_prime
    qg = Q.float().view(B, Hkv, G, S, D)[:, :, :, t0:t1].sum(2)          # [B, Hkv, T, D]
    sc = torch.matmul(qg, Kc.transpose(-1, -2)) / (D ** 0.5)            # [B, Hkv, T, n_cmp]
    src = compressed_positions(S, n_cmp, Q.device)
    tgt = torch.div(src, l_prime, rounding_mode="floor").long().clamp(max=n_blk - 1)
    blk = torch.zeros(B, Hkv, t1 - t0, n_blk, dtype=torch.float32, device=Q.device)
    blk.index_add_(3, tgt, sc)
    qpos = torch.arange(t0, t1, device=Q.device).view(-1, 1)
    bpos = torch.arange(n_blk, device=Q.device).view(1, -1) * l_prime
    return blk.masked_fill((bpos > qpos).view(1, 1, t1 - t0, n_blk), float("-inf"))


def select_blocks(Q: torch.Tensor, Kc: torch.Tensor, n_sel: int, l_prime: int, chunk: int = 2048) -> torch.Tensor:
    """Top-n selection blocks per (batch, KV head, token): int32 [B, Hkv, S, min(n_sel, n_blk)]."""
    B, Hq, S, D = Q.shape
    n_blk = (S + l_prime - 1) // l_prime
    k = min(n_sel, n_blk)
    out = torch.empty(B, Kc.shape[1], S, k, dtype=torch.int32, device=Q.device)
    for t0 in range(0, S, chunk):
        t1 = min(S, t0 + chunk)
        out[:, :, t0:t1] = block_scores(Q, Kc, l_prime, (t0, t1)).topk(k, dim=-1).indices.to(torch.int32)
    return out


def branch_q_block(G: int) -> int:
    """Query tokens per selection row for the window and compressed branches: every token of a
    query block shares its row (the union of the tokens' blocks; the kernel masks each token
    exactly).  BQ = 128 / G fills a 128-row query tile of the row-owner kernel (G heads x BQ
    tokens on the MMA's M); a G that does not divide 128 gets the largest power of two with
    G * BQ <= 64 for the swap-AB kernel.  Measured at B=1, T=65536, Hq=64, Hkv=4, d=128 on a
    B200 (window 512, 32/16 compression): window 14.4 ms (BQ=1) / 7.1 (BQ=4) / 3.7 (BQ=8,
    row owner); compressed 27.9 / 17.7 / 7.4 ms."""
    if G <= 128 and 128 % G == 0:
        return 128 // G
    bq = 1
    while G * bq * 2 <= 64:
        bq *= 2
    return bq


def window_selection(B: int, Hkv: int, T: int, window: int, l_prime: int, device, q_block: int = 1) -> torch.Tensor:
    """Selection rows covering keys [t - window + 1, t] for every token t of each query block of
    q_block tokens: blocks t1//l' down to max(0, t0 - window + 1)//l' for the block's first and
    last tokens t0, t1 (-1 padding), int32 [B, Hkv, ceil(T/q_block), (window + q_block - 2)//l' + 2]."""
    nqb = (T + q_block - 1) // q_block
    nw = (window + q_block - 2) // l_prime + 2
    t0 = torch.arange(nqb, device=device, dtype=torch.int32) * q_block
    t1 = torch.clamp(t0 + q_block - 1, max=T - 1)
    lo = torch.clamp(t0 - window + 1, min=0) // l_prime
    sel = (t1 // l_prime).view(-1, 1) - torch.arange(nw, device=device, dtype=torch.int32).view(1, -1)
    sel = torch.where(sel >= lo.view(-1, 1), sel, torch.full_like(sel, -1))
    return sel.view(1, 1, nqb, nw).expand(B, Hkv, nqb, nw).contiguous()


def compressed_selection(B: int, Hkv: int, T: int, n_cmp: int, device, q_block: int = 1) -> torch.Tensor:
    """Every 64-key block of the compressed keys, for every query block: int32
    [B, Hkv, ceil(T/q_block), ceil(n_cmp/64)] (the kernel drops the blocks past a unit's last
    visible key, and its compressed key map hides the keys past each token's position)."""
    nb = (n_cmp + 63) // 64
    nqb = (T + q_block - 1) // q_block
    return torch.arange(nb, device=device, dtype=torch.int32).view(1, 1, 1, nb).expand(B, Hkv, nqb, nb).contiguous()


def window_branch_kernel(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, window: int,
                         q_block: Optional[int] = None) -> torch.Tensor:
    """The sliding-window branch on the B200 kernel (bf16 inputs, fp32 O)."""
    from . import ops

    B, Hq, T, _ = Q.shape
    bq = q_block or branch_q_block(Hq // K.shape[1])
    sel = window_selection(B, K.shape[1], T, window, 64, Q.device, bq)
    o, _ = ops.forward_ext(Q, K, V, sel, 64, bq, window=window, key_map=0)
    return o


def compressed_branch_kernel(Q: torch.Tensor, Kc: torch.Tensor, Vc: torch.Tensor,
                             q_block: Optional[int] = None) -> torch.Tensor:
    """The compressed branch on the B200 kernel: compressed keys/values (bf16) with the
    compressed key map (key i visible to t iff float32 linspace(0, T-1, n_cmp)[i] <= t)."""
    from . import ops

    B, Hq, T, _ = Q.shape
    n_cmp = Kc.shape[2]
    if n_cmp == 0:
        return torch.zeros(B, Hq, T, Vc.shape[3], dtype=torch.float32, device=Q.device)
    bq = q_block or branch_q_block(Hq // Kc.shape[1])
    sel = compressed_selection(B, Kc.shape[1], T, n_cmp, Q.device, bq)
    o, _ = ops.forward_ext(Q, Kc.to(torch.bfloat16).contiguous(), Vc.to(torch.bfloat16).contiguous(), sel, 64, bq,
                           window=0, key_map=1)
    return o


def gate_weights(gate_w: Optional[torch.Tensor], device) -> torch.Tensor:
    if gate_w is None:
        return torch.full((3,), 1.0 / 3.0, dtype=torch.float32, device=device)
    g = torch.sigmoid(gate_w.to(device=device, dtype=torch.float32))
    return g / g.sum()


def nsa_forward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, *, n_sel: int = 16, l_prime: int = 64,
                window: int = 512, cmp_block: int = 32, cmp_stride: int = 16, gate_w: Optional[torch.Tensor] = None,
                sel_override: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """NSA forward with the reference's signature (nsa_reference.py:46-89): returns (O fp32
    [B, Hq, S, D], sel int32 [B, Hkv, S, k]).  Q/K/V are CUDA tensors; the selected branch runs
    in bf16 on the tensor cores (inputs are rounded to bf16 for it)."""
    from . import ops  # the CUDA extension; raises if it is not built

    if not Q.is_cuda:
        raise RuntimeError("nsa_forward needs CUDA tensors (the selected branch is a B200 kernel)")
    Qb, Kb, Vb = (x.to(torch.bfloat16).contiguous() for x in (Q, K, V))
    B, Hq, T, _ = Qb.shape
    Hkv = Kb.shape[1]
    Kc, Vc = compress_kv(Kb, Vb, cmp_block, cmp_stride)
    if sel_override is not None:
        sel = sel_override.to(device=Q.device, dtype=torch.int32).contiguous()
    else:  # the B200 selection kernel (scores in fp32, top-k per token)
        sel = ops.select_blocks(Qb, Kb, n_sel, l_prime, cmp_block, cmp_stride)
    # The gate is fused into the three attention launches: each writes (first) or TMA-adds (the
    # others) its gate-weighted result into one fp32 O; the weights stay on the device.
    g = gate_weights(gate_w, Q.device)
    O = torch.empty(B, Hq, T, Vb.shape[3], dtype=torch.float32, device=Q.device)
    ops.forward_ext(Qb, Kb, Vb, sel, l_prime, 1, out=O, weight=g[1:2], with_lse=False)
    n_cmp = Kc.shape[2]
    if n_cmp > 0:
        bq = branch_q_block(Hq // Hkv)
        csel = compressed_selection(B, Hkv, T, n_cmp, Q.device, bq)
        ops.forward_ext(Qb, Kc.to(torch.bfloat16).contiguous(), Vc.to(torch.bfloat16).contiguous(), csel, 64, bq,
                        key_map=1, out=O, weight=g[0:1], accumulate=True, with_lse=False)
    bq = branch_q_block(Hq // Hkv)
    wsel = window_selection(B, Hkv, T, window, 64, Q.device, bq)
    ops.forward_ext(Qb, Kb, Vb, wsel, 64, bq, window=window, out=O, weight=g[2:3], accumulate=True, with_lse=False)
    return O, sel


def validate_fn(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, sel: torch.Tensor, cfg: Dict) -> torch.Tensor:
    """The ``fn(Q, K, V, sel, cfg)`` that ``validate.check(fn, dtype)`` calls (validate.py:21)."""
    o, _ = nsa_forward(Q, K, V, n_sel=cfg["n_sel"], l_prime=cfg["l_prime"], window=cfg["window"], sel_override=sel)
    return o
