"""The reference's frozen test-set protocol (make_testset.py:9-30, validate.py:12-28) on the GPU:
8 shapes x 25 seeded repetitions = 200 cases, repetition 0 with one large-magnitude query row
(x50).  Each case runs the full NSA forward through ``nsa.validate_fn`` (the ``fn`` that
``validate.check(fn, torch.bfloat16)`` calls) and is scored with validate.py's metric,
max|err| / max|out|, against the CPU restatement of the reference's nsa_forward: the compressed
and sliding-window branches and the block scoring of nsa_hopper_b200/nsa.py (pinned to the
reference's own fp64 outputs by the nsa_full_* fixtures, tests/test_nsa_wrapper.py) and the
selected branch of the C oracle, all on the same bf16 inputs and the same selection.  The
reference's bf16 floor is 3e-2 (validate.py:10)."""
import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import nsa

pytestmark = pytest.mark.gpu

GRID = [  # (B, Hq, Hkv, S, D, n_sel, l_prime, window), make_testset.py:9-18
    (1, 8, 2, 512, 64, 4, 64, 128), (1, 8, 2, 512, 64, 16, 64, 128), (2, 16, 2, 1024, 128, 8, 64, 256),
    (1, 4, 4, 512, 64, 4, 64, 128), (1, 16, 1, 768, 64, 8, 128, 256), (1, 8, 2, 500, 64, 4, 64, 128),
    (1, 8, 2, 512, 64, 1, 256, 64), (1, 8, 2, 2048, 128, 16, 64, 512),
]
BF16_FLOOR = 3e-2
CASES = [(i, rep) for i in range(len(GRID)) for rep in range(25)]


def _case(i, rep):
    B, Hq, Hkv, S, D, n_sel, lp, w = GRID[i]
    g = torch.Generator().manual_seed(1337 + 100 * i + rep)
    q = torch.randn(B, Hq, S, D, generator=g)
    k = torch.randn(B, Hkv, S, D, generator=g)
    v = torch.randn(B, Hkv, S, D, generator=g)
    if rep == 0:  # make_testset.py:24-25, the adversarial large-magnitude row
        q[..., 0, :] *= 50.0
    return [x.to(torch.bfloat16) for x in (q, k, v)], dict(n_sel=n_sel, l_prime=lp, window=w)


def _reference(q, k, v, cfg):
    Kc, Vc = nsa.compress_kv(k, v, 32, 16)
    sel = nsa.select_blocks(q, Kc, cfg["n_sel"], cfg["l_prime"])
    o_cmp = nsa.compressed_branch(q, Kc, Vc).double().numpy()
    o_win = nsa.window_branch(q, k, v, cfg["window"]).double().numpy()
    o_sel, _ = oracle.forward(q, k, v, sel, cfg["l_prime"], 1)
    return (o_cmp + o_sel + o_win) / 3.0, sel  # nsa_reference.py:86-88 with the default gate


@pytest.mark.parametrize("i,rep", CASES)
def test_frozen_testset_case(i, rep):
    (q, k, v), cfg = _case(i, rep)
    o_ref, sel = _reference(q, k, v, cfg)
    o = nsa.validate_fn(q.cuda(), k.cuda(), v.cuda(), sel.cuda(), cfg)
    torch.cuda.synchronize()
    err = np.abs(o.double().cpu().numpy() - o_ref).max() / np.abs(o_ref).max()
    assert err <= BF16_FLOOR / 3, (GRID[i], rep, err)
