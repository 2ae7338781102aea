"""Shared test helpers: seeded inputs, a C-ABI call on torch buffers, the oracle check."""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import numpy as np
import torch

import oracle
from nsa_hopper_b200 import capi

# Tolerances stated by the north star: bf16 O max-abs error <= 2e-2, LSE <= 1e-3 relative,
# both against an fp32 (here: fp64) reference on the same bf16 inputs.
O_ATOL = 2e-2
LSE_RTOL = 1e-3


def make_qkv(B: int, Hq: int, Hkv: int, T: int, d_qk: int, d_v: int, seed: int = 0):
    """N(0,1) fp32 drawn on the CPU with a seeded generator, rounded to bf16."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, T, d_qk, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, d_qk, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, d_v, generator=g).to(torch.bfloat16)
    return q, k, v


def run_capi(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sel: torch.Tensor, *, l_prime: int = 64,
             BQ: int = 1, cu_seqlens: Optional[torch.Tensor] = None, out_f32: bool = False,
             with_lse: bool = True, cyc: Optional[torch.Tensor] = None, err: Optional[torch.Tensor] = None,
             scale: float = 0.0, timeout_ms: int = 0, shard: Optional[Tuple[int, int, int, int]] = None,
             o: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None, max_ctas: int = 0,
             debug_flags: int = 0):
    """Launch through nsa_sel_run on the current stream; returns (O, LSE) device tensors."""
    dev = torch.device("cuda")
    q, k, v = q.to(dev).contiguous(), k.to(dev).contiguous(), v.to(dev).contiguous()
    sel = sel.to(dev, torch.int32).contiguous()
    B, Hq, T, dqk = q.shape
    Hkv, dv = k.shape[1], v.shape[3]
    if o is None:
        o = torch.full((B, Hq, T, dv), float("nan"), device=dev, dtype=torch.float32 if out_f32 else torch.bfloat16)
    if lse is None and with_lse:
        lse = torch.full((B, Hq, T), float("nan"), device=dev, dtype=torch.float32)
    cu = None if cu_seqlens is None else cu_seqlens.to(dev, torch.int32).contiguous()
    d = capi.make_desc(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), sel=sel.data_ptr(),
        cu_seqlens=cu.data_ptr() if cu is not None else None, n_seqs=(cu.numel() - 1) if cu is not None else 0,
        o=o.data_ptr(), lse=lse.data_ptr() if lse is not None else None,
        cyc=cyc.data_ptr() if cyc is not None else None, err=err.data_ptr() if err is not None else None,
        batch=B, heads_q=Hq, heads_kv=Hkv, seq_len=T, d_qk=dqk, d_v=dv, n_qblocks=sel.shape[2], n_sel=sel.shape[3],
        block_size=l_prime, q_block=BQ, o_dtype=capi.DTYPE_F32 if out_f32 else capi.DTYPE_BF16, scale=scale,
        timeout_ms=timeout_ms, max_ctas=max_ctas, debug_flags=debug_flags)
    if shard is not None:
        d.bkv_begin, d.bkv_end, d.qb_begin, d.qb_end = shard
    capi.run(d, torch.cuda.current_stream().cuda_stream)
    return o, lse


def compare(o_dev: torch.Tensor, lse_dev: Optional[torch.Tensor], o_ref: np.ndarray, lse_ref: np.ndarray,
            o_atol: float = O_ATOL, lse_rtol: float = LSE_RTOL) -> dict:
    o = o_dev.float().cpu().numpy().astype(np.float64)
    assert np.isfinite(o).all(), f"non-finite O at {np.argwhere(~np.isfinite(o))[:5].tolist()}"
    err = np.abs(o - o_ref)
    idx = np.unravel_index(int(np.argmax(err)), err.shape)
    res = {"o_max_abs": float(err.max()), "o_argmax": tuple(int(i) for i in idx),
           "o_scaled": float(err.max() / max(np.abs(o_ref).max(), 1e-30))}
    assert res["o_max_abs"] <= o_atol, f"O mismatch {res}; got {o[idx]} want {o_ref[idx]}"
    if lse_dev is not None:
        lse = lse_dev.cpu().numpy().astype(np.float64)
        inf_ref = np.isneginf(lse_ref)
        assert (np.isneginf(lse) == inf_ref).all(), \
            f"-inf LSE pattern differs at {np.argwhere(np.isneginf(lse) != inf_ref)[:5].tolist()}"
        fin = ~inf_ref
        rel = np.abs(lse[fin] - lse_ref[fin]) / np.maximum(np.abs(lse_ref[fin]), 1.0)
        res["lse_max_rel"] = float(rel.max()) if rel.size else 0.0
        assert res["lse_max_rel"] <= lse_rtol, f"LSE mismatch {res}"
    return res


def run_backward_capi(q, k, v, sel, d_o, o, lse, *, l_prime: int = 64, scale: float = 0.0, grads=None,
                      timeout_ms: int = 0):
    """nsa_sel_backward on torch buffers through the C ABI; returns (dQ, dK, dV, err) device
    tensors.  ``grads`` = (dq, dk, dv) fp32 buffers to accumulate into (zeros if None)."""
    dev = torch.device("cuda")
    q, k, v, d_o = (x.to(dev).contiguous() for x in (q, k, v, d_o))
    sel = sel.to(dev, torch.int32).contiguous() if torch.is_tensor(sel) else torch.from_numpy(
        np.ascontiguousarray(sel, dtype=np.int32)).to(dev)
    B, Hq, T, d = q.shape
    Hkv = k.shape[1]
    if grads is None:
        grads = (torch.zeros(B, Hq, T, d, device=dev), torch.zeros(B, Hkv, T, d, device=dev),
                 torch.zeros(B, Hkv, T, d, device=dev))
    dq, dk, dv = grads
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    desc = capi.make_bwd_desc(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), sel=sel.data_ptr(), o=o.data_ptr(), lse=lse.data_ptr(),
        d_o=d_o.data_ptr(), dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(), err=err.data_ptr(), batch=B,
        heads_q=Hq, heads_kv=Hkv, seq_len=T, d=d, n_sel=sel.shape[-1], block_size=l_prime,
        o_dtype=capi.DTYPE_BF16 if o.dtype == torch.bfloat16 else capi.DTYPE_F32, scale=scale,
        timeout_ms=timeout_ms)
    ws = torch.empty(capi.backward_workspace_bytes(desc), dtype=torch.uint8, device=dev)
    desc.workspace = ws.data_ptr()
    capi.backward(desc, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return dq, dk, dv, err


def scaled_err(x: np.ndarray, ref: np.ndarray) -> float:
    """max |x - ref| / max |ref| (the reference validate.py's metric, validate.py:12-28)."""
    return float(np.abs(np.asarray(x, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))
