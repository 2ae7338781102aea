"""The kernel's extended key visibility (sliding window; compressed keys with the float32
linspace key map) against the tensor-op restatements of the reference's window and compressed
branches (nsa_reference.py:59-64, 79-82), which tests/test_nsa_wrapper.py pins to the reference."""
import numpy as np
import pytest
import torch

from nsa_hopper_b200 import nsa, ops

pytestmark = pytest.mark.gpu


def _qkv(B, Hq, Hkv, T, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda h: torch.randn(B, h, T, D, device="cuda", generator=g).to(torch.bfloat16)
    return mk(Hq), mk(Hkv), mk(Hkv)


def _lse_masked(q, k, mask, scale):
    G = q.shape[1] // k.shape[1]
    s = torch.matmul(q.float(), k.float().repeat_interleave(G, 1).transpose(-1, -2)) * scale
    s = s.masked_fill(~mask, float("-inf"))
    return torch.logsumexp(s, -1)


@pytest.mark.parametrize("bq", [1, 0])
@pytest.mark.parametrize("B,Hq,Hkv,T,D,window", [(1, 16, 2, 1500, 64, 128), (1, 8, 2, 777, 128, 100),
                                                 (2, 4, 4, 512, 64, 512), (1, 64, 4, 2048, 128, 512),
                                                 (1, 16, 1, 300, 64, 1000)])
def test_window_branch_on_kernel(B, Hq, Hkv, T, D, window, bq):
    """bq = 0: the wrapper's shared query blocks (64 / G tokens per selection row)."""
    q, k, v = _qkv(B, Hq, Hkv, T, D, T + window)
    bq = bq or nsa.branch_q_block(Hq // Hkv)
    sel = nsa.window_selection(B, Hkv, T, window, 64, q.device, bq)
    o, lse = ops.forward_ext(q, k, v, sel, 64, bq, window=window, key_map=0)
    ref = nsa.window_branch(q, k, v, window)
    torch.cuda.synchronize()
    assert (o - ref).abs().max().item() <= 2e-2
    t = torch.arange(T, device="cuda")
    d = t.view(-1, 1) - t.view(1, -1)
    mask = ((d >= 0) & (d < window)).view(1, 1, T, T)
    want = _lse_masked(q, k, mask, D ** -0.5)
    assert ((lse - want).abs() / want.abs().clamp(min=1)).max().item() <= 1e-3


@pytest.mark.parametrize("bq", [1, 0])
@pytest.mark.parametrize("B,Hq,Hkv,T,D", [(1, 8, 2, 512, 64), (1, 16, 1, 1500, 64), (2, 8, 2, 1024, 128),
                                          (1, 64, 4, 4096, 128), (1, 4, 4, 40, 64), (1, 64, 4, 1111, 64)])
def test_compressed_branch_on_kernel(B, Hq, Hkv, T, D, bq):
    """bq = 0: the wrapper's shared query blocks (64 / G tokens per selection row)."""
    q, k, v = _qkv(B, Hq, Hkv, T, D, 3 * T)
    Kc, Vc = nsa.compress_kv(k, v, 32, 16)
    Kc, Vc = Kc.to(torch.bfloat16), Vc.to(torch.bfloat16)  # the kernel's operands
    bq = bq or nsa.branch_q_block(Hq // Hkv)
    o = nsa.compressed_branch_kernel(q, Kc, Vc, q_block=bq)
    ref = nsa.compressed_branch(q, Kc.float(), Vc.float())
    torch.cuda.synchronize()
    assert (o - ref).abs().max().item() <= 2e-2
    if Kc.shape[2] > 0:
        sel = nsa.compressed_selection(B, Hkv, T, Kc.shape[2], q.device, bq)
        _, lse = ops.forward_ext(q, Kc, Vc, sel, 64, bq, window=0, key_map=1)
        cpos = nsa.compressed_positions(T, Kc.shape[2], q.device)
        mask = (cpos.view(1, -1) <= torch.arange(T, device="cuda", dtype=torch.float32).view(-1, 1))
        want = _lse_masked(q, Kc, mask.view(1, 1, T, -1), D ** -0.5)
        assert ((lse - want).abs() / want.abs().clamp(min=1)).max().item() <= 1e-3


def test_window_covering_everything_equals_causal_attention():
    B, Hq, Hkv, T, D = 1, 8, 2, 700, 64
    q, k, v = _qkv(B, Hq, Hkv, T, D, 9)
    nb = (T + 63) // 64
    all_blocks = torch.arange(nb, device="cuda", dtype=torch.int32).view(1, 1, 1, nb).expand(B, Hkv, T, nb).contiguous()
    o_w, l_w = ops.forward_ext(q, k, v, all_blocks, 64, 1, window=T, key_map=0)
    o_c, l_c = ops.forward_ext(q, k, v, all_blocks, 64, 1, window=0, key_map=0)
    torch.cuda.synchronize()
    assert torch.equal(o_w, o_c) and torch.equal(l_w, l_c)


def test_weighted_output_and_accumulate():
    """out= / weight= / accumulate=: O = w * result, or O += w * result through a TMA reduce-add."""
    B, Hq, Hkv, T, D = 1, 16, 2, 900, 128
    q, k, v = _qkv(B, Hq, Hkv, T, D, 77)
    sel = nsa.window_selection(B, Hkv, T, 256, 64, q.device, 4)
    plain, lse = ops.forward_ext(q, k, v, sel, 64, 4, window=256)
    w = torch.tensor([0.0, 0.37], device="cuda")[1:]  # a weight that is not at the tensor's start
    o, l2 = ops.forward_ext(q, k, v, sel, 64, 4, window=256, out=torch.full_like(plain, 5.0), weight=w, with_lse=False)
    base = torch.randn(plain.shape, device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    acc, _ = ops.forward_ext(q, k, v, sel, 64, 4, window=256, out=base.clone(), weight=w, accumulate=True)
    torch.cuda.synchronize()
    assert l2.numel() == 0
    tol = 1e-6 * plain.abs().max().item()
    assert (o - 0.37 * plain).abs().max().item() <= tol
    assert (acc - (base + 0.37 * plain)).abs().max().item() <= tol + 1e-6 * base.abs().max().item()
    with pytest.raises(RuntimeError):  # accumulate needs an output to add into
        ops.forward_ext(q, k, v, sel, 64, 4, window=256, accumulate=True)


@pytest.mark.parametrize("T", [40, 1000])
def test_nsa_forward_fused_gate_equals_branch_sum(T):
    """nsa_forward's fused gate (three launches into one fp32 O) equals the gate applied to the
    three branch outputs computed separately."""
    B, Hq, Hkv, D = 1, 32, 2, 64
    q, k, v = _qkv(B, Hq, Hkv, T, D, 5 + T)
    gate_w = torch.tensor([0.3, -1.0, 0.8])
    o, sel = nsa.nsa_forward(q, k, v, n_sel=4, l_prime=64, window=128, gate_w=gate_w)
    g = nsa.gate_weights(gate_w, q.device)
    Kc, Vc = nsa.compress_kv(k, v, 32, 16)
    o_cmp = nsa.compressed_branch_kernel(q, Kc, Vc)
    o_sel = ops.forward(q, k, v, sel, 64, 1)
    o_win = nsa.window_branch_kernel(q, k, v, 128)
    want = g[0] * o_cmp + g[1] * o_sel + g[2] * o_win
    torch.cuda.synchronize()
    assert (o - want).abs().max().item() <= 1e-5 * max(1.0, want.abs().max().item())


def test_row_owner_rescale_of_one_row_in_a_warp():
    """A lazy O rescale that only some rows of a warp need (the row-owner kernel's tensor-memory
    pass runs warp-wide).  G = 1 with 128-token tiles and window 128: row t = 128 of its tile sees
    only key 128 in its first chunk; that key gets a very low score for it, so the row's running
    max jumps by far more than 2^8 at the next chunk while its neighbours' do not."""
    B, H, T, D, window = 1, 1, 512, 64, 128
    g = torch.Generator(device="cuda").manual_seed(77)
    q = torch.randn(B, H, T, D, device="cuda", generator=g)
    k = torch.randn(B, H, T, D, device="cuda", generator=g)
    v = torch.randn(B, H, T, D, device="cuda", generator=g)
    k[:, :, 128] = -8.0 * q[:, :, 128]
    q, k, v = (x.to(torch.bfloat16) for x in (q, k, v))
    bq = nsa.branch_q_block(1)
    assert bq == 128
    sel = nsa.window_selection(B, H, T, window, 64, q.device, bq)
    o, _ = ops.forward_ext(q, k, v, sel, 64, bq, window=window, key_map=0)
    ref = nsa.window_branch(q, k, v, window)
    torch.cuda.synchronize()
    assert (o - ref).abs().max().item() <= 2e-2
