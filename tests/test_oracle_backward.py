"""The CPU restatement of the backward (oracle/backward.py) against the reference's own
gradients: autograd of ref_only.ref_selected in fp64 (fixtures tests/golden/bwd_*.npz)."""
import numpy as np
import pytest
import torch

from oracle import backward as obwd
from tests import golden_cases


@pytest.mark.parametrize("name", golden_cases.bwd_case_names())
def test_backward_oracle_matches_reference_autograd(name):
    c = golden_cases.load_bwd(name)
    dq, dk, dv = obwd.backward(c["q"], c["k"], c["v"], c["sel"], c["LP"], c["d_o"])
    for key, x in (("dq", dq), ("dk", dk), ("dv", dv)):
        np.testing.assert_allclose(golden_cases.rows_of(x, c[key + "_rows"]), c[key + "_vals"], rtol=0, atol=1e-9)
        np.testing.assert_allclose(golden_cases.checksums(x), c[key + "_checksums"], rtol=1e-9, atol=1e-7)


def test_backward_oracle_matches_autograd_of_its_own_mask():
    """Independent of the fixtures: the restatement equals torch autograd of a dense masked softmax
    attention built from oracle.backward.key_mask (fp64, rows with no visible key give 0)."""
    g = torch.Generator().manual_seed(5)
    B, Hq, Hkv, T, D, LP = 1, 4, 2, 130, 16, 64
    q, k, v = (torch.randn(B, h, T, D, generator=g, dtype=torch.float64) for h in (Hq, Hkv, Hkv))
    d_o = torch.randn(B, Hq, T, D, generator=g, dtype=torch.float64)
    sel = np.full((B, Hkv, T, 3), -1, np.int32)
    sel[..., 0] = np.arange(T) // LP
    sel[0, 1, 5:, 1] = 0
    sel[0, 0, ::3, 2] = 1  # a future block for early tokens: masked
    Q, K, V = (x.clone().requires_grad_() for x in (q, k, v))
    G = Hq // Hkv
    mask = torch.from_numpy(np.stack([obwd.key_mask(sel[0, h], T, LP) for h in range(Hkv)]))
    s = (Q @ K.repeat_interleave(G, 1).transpose(-1, -2)) / D ** 0.5
    s = s.masked_fill(~mask.repeat_interleave(G, 0)[None], float("-inf"))
    O = torch.nan_to_num(torch.softmax(s, -1), nan=0.0) @ V.repeat_interleave(G, 1)
    O.backward(d_o)
    dq, dk, dv = obwd.backward(q, k, v, sel, LP, d_o)
    np.testing.assert_allclose(dq, Q.grad.numpy(), atol=1e-12)
    np.testing.assert_allclose(dk, K.grad.numpy(), atol=1e-12)
    np.testing.assert_allclose(dv, V.grad.numpy(), atol=1e-12)
