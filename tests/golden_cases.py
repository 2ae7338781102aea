"""Loader for the golden fixtures in tests/golden (made by tests/golden/make_golden.py)."""
from __future__ import annotations

import glob
import hashlib
import os
from typing import Dict, List

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def case_names() -> List[str]:
    """Selected-branch fixtures (ref_selected / the selected branch of nsa_forward)."""
    return sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))
                  if not os.path.basename(p).startswith(("nsa_full_", "bwd_")))


def bwd_case_names() -> List[str]:
    """Backward fixtures: autograd of ref_selected with a seeded upstream gradient."""
    return sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN_DIR, "bwd_*.npz")))


def full_case_names() -> List[str]:
    """Full NSA forward fixtures (all three branches, the reference's own selection)."""
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(GOLDEN_DIR, "nsa_full_*.npz")))


def load(name: str) -> Dict:
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    c = {k: z[k] for k in z.files}
    for k in ("B", "Hq", "Hkv", "T", "dqk", "dv", "LP", "BQ", "seed", "n_sel", "window"):
        if k in c:
            c[k] = int(c[k])
    c["big_row"] = int(c.get("big_row", 0))
    g = torch.Generator().manual_seed(c["seed"])
    q = torch.randn(c["B"], c["Hq"], c["T"], c["dqk"], generator=g).to(torch.bfloat16)
    k = torch.randn(c["B"], c["Hkv"], c["T"], c["dqk"], generator=g).to(torch.bfloat16)
    v = torch.randn(c["B"], c["Hkv"], c["T"], c["dv"], generator=g).to(torch.bfloat16)
    if c["big_row"]:  # make_testset.py:24-25: one large-magnitude query row
        q = q.clone()
        q[..., 0, :] = (q[..., 0, :].float() * 50.0).to(torch.bfloat16)
    h = hashlib.sha256()
    for t in (q, k, v):
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    if h.hexdigest() != str(c["sha256"]):
        raise RuntimeError(f"{name}: regenerated inputs differ from the fixture's (torch generator changed?)")
    c["q"], c["k"], c["v"] = q, k, v
    return c


def load_bwd(name: str) -> Dict:
    """A backward fixture with its regenerated inputs, including the upstream gradient d_o."""
    c = load(name)
    g = torch.Generator().manual_seed(c["seed"] + 1000)
    d_o = torch.randn(c["B"], c["Hq"], c["T"], c["dqk"], generator=g).to(torch.bfloat16)
    if hashlib.sha256(d_o.contiguous().view(torch.int16).numpy().tobytes()).hexdigest() != str(c["sha256_do"]):
        raise RuntimeError(f"{name}: regenerated dO differs from the fixture's")
    c["d_o"] = d_o
    return c


def checksums(o: np.ndarray) -> np.ndarray:
    w = np.random.Generator(np.random.PCG64(1234)).standard_normal(o.shape)
    return np.array([o.sum(), (o * o).sum(), (o * w).sum()], dtype=np.float64)


def rows_of(o: np.ndarray, rows: np.ndarray) -> np.ndarray:
    return o[rows[:, 0], rows[:, 1], rows[:, 2]]
