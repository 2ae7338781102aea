"""PyTorch-facing ops: the reference's ``forward`` signature plus the BASELINE ``forward_lse``.

These call the in-tree extension ``nsa_hopper_b200._C`` (nsa_sel_torch.cpp), which calls the C
ABI of ``libnsa_sel.so``.  There is no CPU or eager fallback: if the extension or the library
is missing, or the device is not a B200, the call raises.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

try:
    from . import _C  # type: ignore[attr-defined]
except ImportError as e:  # pragma: no cover - exercised only when the build is missing
    raise ImportError("nsa_hopper_b200._C is not built: run `python -m nsa_hopper_b200.build`") from e


def forward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, sel: torch.Tensor, l_prime: int, BQ: int,
            cyc: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Drop-in for the reference op ``mod.forward(Q,K,V,sel,l_prime,BQ,cyc)`` (nsa_v2.cu:147):
    returns fp32 O [B,Hq,S,D].  ``cyc`` may be an int64 CUDA tensor of NQB*B*Hkv*2 entries
    (accumulated into) or empty/None."""
    if cyc is None:
        cyc = torch.empty(0, dtype=torch.int64, device=Q.device)
    return _C.forward(Q, K, V, sel, int(l_prime), int(BQ), cyc)


def forward_lse(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, sel: torch.Tensor, l_prime: int = 64,
                BQ: int = 1, cu_seqlens: Optional[torch.Tensor] = None, scale: float = 0.0,
                out_f32: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Selected-branch forward returning (O bf16 [B,Hq,T,d_v], LSE fp32 [B,Hq,T])."""
    o, lse = _C.forward_lse(Q, K, V, sel, int(l_prime), int(BQ), cu_seqlens, float(scale), bool(out_f32))
    return o, lse


def forward_ext(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, sel: torch.Tensor, l_prime: int = 64, BQ: int = 1,
                window: int = 0, key_map: int = 0, scale: float = 0.0, out: Optional[torch.Tensor] = None,
                weight: Optional[torch.Tensor] = None, accumulate: bool = False,
                with_lse: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """Forward with extended key visibility (fp32 O, fp32 LSE): ``window`` > 0 limits query t to
    keys p with t - p < window; ``key_map`` = 1 treats K/V as compressed keys (kv_len rows) visible
    to t iff float32 linspace(0, T-1, kv_len)[i] <= t (the compressed branch of NSA).

    Fused output combination: the result is multiplied by ``weight[0]`` (an fp32 CUDA tensor, read
    on the device) and written to ``out``, or added into it when ``accumulate`` (TMA reduce-add),
    so the NSA gate g_c*O_cmp + g_s*O_sel + g_w*O_win is three launches into one buffer.
    ``with_lse=False`` skips the LSE (an empty tensor is returned in its place)."""
    o, lse = _C.forward_ext(Q, K, V, sel, int(l_prime), int(BQ), int(window), int(key_map), float(scale), out, weight,
                            bool(accumulate), bool(with_lse))
    return o, lse


def select_blocks(Q: torch.Tensor, K: torch.Tensor, n_sel: int, l_prime: int = 64, cmp_block: int = 32,
                  cmp_stride: int = 16) -> torch.Tensor:
    """Block selection on the GPU (nsa_sel_select): int32 [B, Hkv, T, min(n_sel, ceil(T/l_prime))],
    best block first, -1 where fewer blocks are visible (reference nsa_reference.py:27-44)."""
    return _C.select_blocks(Q, K, int(n_sel), int(l_prime), int(cmp_block), int(cmp_stride))


def backward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, sel: torch.Tensor, O: torch.Tensor,
             LSE: torch.Tensor, dO: torch.Tensor, l_prime: int = 64, scale: float = 0.0
             ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients (fp32 dQ, dK, dV) of the selected-branch forward for the upstream gradient dO,
    given that forward's O (bf16 or fp32) and LSE.  Per-token selection (sel [B,Hkv,T,KSEL]),
    d = 128, G = Hq/Hkv in {8, 16} (nsa_sel_backward; the reference has no backward pass).  The
    workspace comes from torch's caching allocator; the library allocates nothing."""
    from . import capi

    for name, t in (("Q", Q), ("K", K), ("V", V), ("dO", dO)):
        if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
    if O.dtype not in (torch.bfloat16, torch.float32) or not O.is_contiguous():
        raise ValueError("O must be a contiguous bf16 or fp32 tensor")
    if LSE.dtype != torch.float32 or not LSE.is_contiguous():
        raise ValueError("LSE must be a contiguous fp32 tensor")
    sel = sel.to(torch.int32).contiguous()
    B, Hq, T, d = Q.shape
    Hkv = K.shape[1]
    dq = torch.zeros(B, Hq, T, d, device=Q.device, dtype=torch.float32)
    dk = torch.zeros(B, Hkv, T, d, device=Q.device, dtype=torch.float32)
    dv = torch.zeros_like(dk)
    desc = capi.make_bwd_desc(
        q=Q.data_ptr(), k=K.data_ptr(), v=V.data_ptr(), sel=sel.data_ptr(), o=O.data_ptr(), lse=LSE.data_ptr(),
        d_o=dO.data_ptr(), dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(), batch=B, heads_q=Hq,
        heads_kv=Hkv, seq_len=T, d=d, n_sel=sel.shape[-1], block_size=int(l_prime),
        o_dtype=capi.DTYPE_BF16 if O.dtype == torch.bfloat16 else capi.DTYPE_F32, scale=float(scale))
    ws = torch.empty(capi.backward_workspace_bytes(desc), device=Q.device, dtype=torch.uint8)
    desc.workspace = ws.data_ptr()
    capi.backward(desc, torch.cuda.current_stream(Q.device).cuda_stream)
    return dq, dk, dv


class SelectedAttention(torch.autograd.Function):
    """Selected-branch attention with its backward: ``O = SelectedAttention.apply(Q, K, V, sel)``
    (per-token selection, l_prime = 64) returns bf16 O and supports ``O.backward(dO)``; Q, K, V
    receive bf16 gradients computed by nsa_sel_backward."""

    @staticmethod
    def forward(ctx, Q, K, V, sel, l_prime: int = 64):
        O, LSE = forward_lse(Q, K, V, sel, l_prime, 1)
        ctx.save_for_backward(Q, K, V, sel, O, LSE)
        ctx.l_prime = l_prime
        return O

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, sel, O, LSE = ctx.saved_tensors
        dq, dk, dv = backward(Q, K, V, sel, O, LSE, dO.contiguous().to(torch.bfloat16), ctx.l_prime)
        return dq.to(Q.dtype), dk.to(K.dtype), dv.to(V.dtype), None, None


def library_version() -> int:
    return int(_C.library_version())
