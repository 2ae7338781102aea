"""Backward of the selected branch (nsa_sel_backward, through the C ABI) against the reference's
own gradients (autograd of ref_only.ref_selected: tests/golden/bwd_*.npz) and the CPU
restatement oracle/backward.py.

Tolerance: every gradient tensor within 2e-2 scaled error (max |err| / max |ref|, the metric of the
reference's validate.py, whose bf16 floor is 3e-2): the kernel rounds P and dS to bf16 for the
tensor-core products, as the forward rounds P."""
import numpy as np
import pytest
import torch

from nsa_hopper_b200 import capi, indices, ops
from oracle import backward as obwd
from tests import golden_cases
from tests.helpers import make_qkv, run_backward_capi, run_capi, scaled_err

pytestmark = pytest.mark.gpu
GRAD_TOL = 2e-2


def _forward(q, k, v, sel, lp):
    return run_capi(q, k, v, torch.as_tensor(np.asarray(sel)), l_prime=lp)


@pytest.mark.parametrize("name", golden_cases.bwd_case_names())
def test_backward_matches_reference_autograd(name):
    c = golden_cases.load_bwd(name)
    o, lse = _forward(c["q"], c["k"], c["v"], c["sel"], c["LP"])
    dq, dk, dv, err = run_backward_capi(c["q"], c["k"], c["v"], c["sel"], c["d_o"], o, lse, l_prime=c["LP"])
    assert int(err.item()) == 0
    ref = obwd.backward(c["q"], c["k"], c["v"], c["sel"], c["LP"], c["d_o"])
    for key, x, r in (("dq", dq, ref[0]), ("dk", dk, ref[1]), ("dv", dv, ref[2])):
        x = x.cpu().numpy()
        assert np.isfinite(x).all()
        # the reference's own fp64 gradients on the sampled rows
        e_rows = np.abs(golden_cases.rows_of(x, c[key + "_rows"]) - c[key + "_vals"]).max() / float(c[key + "_absmax"])
        assert e_rows <= GRAD_TOL, (key, e_rows)
        # every element against the restatement (pinned to those gradients on the CPU)
        assert scaled_err(x, r) <= GRAD_TOL, (key, scaled_err(x, r))


def test_backward_larger_group16_against_oracle():
    B, Hq, Hkv, T, D, n = 1, 32, 2, 2048, 128, 16
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, 41)
    g = torch.Generator().manual_seed(42)
    d_o = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
    sel = indices.rule0(B, Hkv, T, n, 64, seed=41)
    o, lse = _forward(q, k, v, sel, 64)
    dq, dk, dv, err = run_backward_capi(q, k, v, sel, d_o, o, lse)
    assert int(err.item()) == 0
    ref = obwd.backward(q, k, v, sel, 64, d_o)
    for x, r in zip((dq, dk, dv), ref):
        assert scaled_err(x.cpu().numpy(), r) <= GRAD_TOL


def test_backward_sum_identities_and_dq_window_at_a_larger_size():
    """Size-independent checks at T = 16K, Hq 64 / Hkv 4: summed over keys, dV equals the sum of
    dO over the query rows (each row's P sums to 1) and dK is zero (each row's dS sums to 0); dQ
    of a 128-token window against the restatement."""
    B, Hq, Hkv, T, D, n = 1, 64, 4, 16384, 128, 16
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, 43)
    g = torch.Generator().manual_seed(44)
    d_o = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
    sel = indices.rule0(B, Hkv, T, n, 64, seed=43)
    o, lse = _forward(q, k, v, sel, 64)
    dq, dk, dv, err = run_backward_capi(q, k, v, sel, d_o, o, lse)
    assert int(err.item()) == 0
    G = Hq // Hkv
    sum_do = d_o.double().view(B, Hkv, G, T, D).sum((2, 3))
    sum_dv = dv.double().cpu().sum(2)
    scale_dv = d_o.double().abs().view(B, Hkv, G, T, D).sum((2, 3))
    assert ((sum_dv - sum_do).abs() <= 5e-3 * scale_dv + 1e-2).all()
    sum_dk = dk.double().cpu().sum(2)
    assert (sum_dk.abs() <= 5e-3 * dk.double().cpu().abs().sum(2) + 1e-2).all()
    for h, t0 in ((0, 1000), (37, T - 128)):
        r = obwd.dq_rows(q, k, v, sel, 64, d_o, 0, h, t0, t0 + 128)
        assert scaled_err(dq[0, h, t0:t0 + 128].cpu().numpy(), r) <= GRAD_TOL


def test_backward_group8_lp128_across_token_windows():
    """G = 8 (one 8-head octet per token box, 8192-token windows) with l' = 128 blocks on a
    sequence of three windows, the last one partial: the exact sum identities on everything and
    dQ windows in each token window against the restatement."""
    B, Hq, Hkv, T, D, n, lp = 1, 32, 4, 2 * 8192 + 100, 128, 8, 128
    q, k, v = make_qkv(B, Hq, Hkv, T, D, D, 45)
    g = torch.Generator().manual_seed(46)
    d_o = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
    sel = indices.rule0(B, Hkv, T, n, lp, seed=45)
    o, lse = _forward(q, k, v, sel, lp)
    dq, dk, dv, err = run_backward_capi(q, k, v, sel, d_o, o, lse, l_prime=lp)
    assert int(err.item()) == 0
    G = Hq // Hkv
    sum_do = d_o.double().view(B, Hkv, G, T, D).sum((2, 3))
    scale_dv = d_o.double().abs().view(B, Hkv, G, T, D).sum((2, 3))
    assert ((dv.double().cpu().sum(2) - sum_do).abs() <= 5e-3 * scale_dv + 1e-2).all()
    assert (dk.double().cpu().sum(2).abs() <= 5e-3 * dk.double().cpu().abs().sum(2) + 1e-2).all()
    for h, t0 in ((3, 4000), (17, 8192 + 77), (30, T - 64)):
        r = obwd.dq_rows(q, k, v, sel, lp, d_o, 0, h, t0, t0 + 64)
        assert scaled_err(dq[0, h, t0:t0 + 64].cpu().numpy(), r) <= GRAD_TOL


def test_backward_accumulates_into_given_buffers():
    """A second call adds its gradients to the first call's.  The kernel sums with reductions in
    an order that changes from run to run (the inverse index is filled by atomic counters), so
    the second call's own gradients differ from the first's in the last bits: the bound is 1e-4
    of each tensor's largest magnitude (fp32 sums of a few hundred terms differ by far less)."""
    c = golden_cases.load_bwd("bwd_rule0_g16")
    o, lse = _forward(c["q"], c["k"], c["v"], c["sel"], c["LP"])
    g1 = run_backward_capi(c["q"], c["k"], c["v"], c["sel"], c["d_o"], o, lse)[:3]
    g2 = run_backward_capi(c["q"], c["k"], c["v"], c["sel"], c["d_o"], o, lse, grads=tuple(x.clone() for x in g1))[:3]
    for a, b in zip(g1, g2):
        torch.testing.assert_close(b, 2 * a, rtol=1e-4, atol=1e-4 * float(a.abs().max()))


def test_autograd_function_gives_the_kernel_gradients():
    c = golden_cases.load_bwd("bwd_rule0_g8_b2")
    dev = torch.device("cuda")
    Q, K, V = (x.to(dev).clone().requires_grad_() for x in (c["q"], c["k"], c["v"]))
    sel = torch.from_numpy(c["sel"]).to(dev)
    O = ops.SelectedAttention.apply(Q, K, V, sel, c["LP"])
    O.backward(c["d_o"].to(dev))
    ref = obwd.backward(c["q"], c["k"], c["v"], c["sel"], c["LP"], c["d_o"])
    for x, r in zip((Q.grad, K.grad, V.grad), ref):
        assert x.dtype == torch.bfloat16
        assert scaled_err(x.float().cpu().numpy(), r) <= GRAD_TOL


def test_backward_rejects_unsupported_group_on_the_device_path():
    q, k, v = make_qkv(1, 16, 4, 256, 128, 128, 3)  # G = 4
    sel = indices.rule0(1, 4, 256, 4, 64, seed=3)
    o, lse = _forward(q, k, v, sel, 64)
    with pytest.raises(capi.NsaSelError, match="group size G=4"):
        run_backward_capi(q, k, v, sel, torch.zeros_like(q), o, lse)
