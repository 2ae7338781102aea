"""Generate the golden fixtures in this directory from the reference's own PyTorch code.

Run in a container where the reference checkout is available (path given by --reference);
the fixtures it writes are committed, so the tests never need the reference at run time.

For each case the inputs are regenerated from a seed (torch CPU generator, N(0,1) rounded to
bf16) and a SHA-256 of their bf16 bytes is stored so drift of the generator is detected.  The
selection indices are stored verbatim.  Outputs come from:

  * ``ref_only.ref_selected(Q, K, V, sel, l_prime, BQ)`` in fp64 (ref_only.py:2-20) for the
    per-query-block and per-token (BQ = 1) cases;
  * ``nsa_reference.nsa_forward(..., sel_override=sel)`` (nsa_reference.py:46-89): the selected
    branch is recovered exactly from three runs with different gates, since the output is
    g0*o_cmp + g1*o_sel + g2*o_win with g known (nsa_reference.py:84-89).

The reference has no log-sum-exp; ``lse`` is the natural logsumexp of the same masked score
matrix ``ref_selected`` builds (ref_only.py:9-17), computed here in fp64.

Stored per case: the full fp64 LSE, a seeded sample of 256 fp64 output rows and three
full-tensor fp64 checksums of O (sum, sum of squares, a weighted sum), which pin every element.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from nsa_hopper_b200 import indices  # noqa: E402


def qkv(B, Hq, Hkv, T, dqk, dv, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, T, dqk, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, dqk, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, dv, generator=g).to(torch.bfloat16)
    return q, k, v


def digest(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def masked_scores(Q, K, sel, l_prime, BQ):
    """The score matrix ref_selected builds (ref_only.py:9-17), with -inf outside the mask."""
    Q, K = Q.double(), K.double()
    B, Hq, S, D = Q.shape
    Hkv = K.shape[1]
    G = Hq // Hkv
    n_blk = (S + l_prime - 1) // l_prime
    keep = torch.zeros(B, Hkv, sel.shape[2], n_blk + 1, dtype=torch.bool)
    idx = torch.where(sel >= 0, sel, torch.full_like(sel, n_blk)).long()
    keep.scatter_(3, idx, True)
    keep = keep[..., :n_blk]
    tok = keep.repeat_interleave(l_prime, 3)[:, :, :, :S].repeat_interleave(BQ, 2)[:, :, :S, :]
    mask = (tok & torch.tril(torch.ones(S, S, dtype=torch.bool))).repeat_interleave(G, 1)
    s = (Q @ K.repeat_interleave(G, 1).transpose(-1, -2)) / (D ** 0.5)
    return s.masked_fill(~mask, float("-inf"))


def checksums(o: np.ndarray, seed: int) -> np.ndarray:
    w = np.random.Generator(np.random.PCG64(seed)).standard_normal(o.shape)
    return np.array([o.sum(), (o * o).sum(), (o * w).sum()], dtype=np.float64)


def store(path, name, meta, q, k, v, sel, o, lse, full):
    rec = dict(meta)
    rec.update(sha256=digest(q, k, v), sel=sel.astype(np.int32), lse=lse.astype(np.float64),
               checksums=checksums(o, 1234))
    if full:
        rec["o"] = o.astype(np.float32)
    else:
        rng = np.random.Generator(np.random.PCG64(99))
        B, Hq, T, _ = o.shape
        rows = np.stack([rng.integers(0, B, 256), rng.integers(0, Hq, 256), rng.integers(0, T, 256)], 1)
        rec["rows"] = rows.astype(np.int32)
        rec["o_rows"] = o[rows[:, 0], rows[:, 1], rows[:, 2]].astype(np.float64)
    np.savez_compressed(os.path.join(path, name + ".npz"), **{k2: np.asarray(v2) for k2, v2 in rec.items()})
    print("wrote", name, {k2: np.asarray(v2).shape for k2, v2 in rec.items() if k2 not in ("sha256",)})


def nsa_full_cases(out_dir, nsa_forward, compress_kv):
    """Full NSA forward (all three branches, the reference's own block selection) in fp64 on the
    make_testset.py:8-18 grid, one case per shape plus the large-magnitude-row variant
    (make_testset.py:24-25).  Besides O it stores the reference's selection and, for 256 sampled
    (b, kvh, t), the fp64 block scores that selection ranks (nsa_reference.py:31-42, computed
    here with the reference's compress_kv and the same tensor ops), so a selection kernel can be
    checked up to near-ties."""
    grid = [
        # (B, Hq, Hkv, S, D, n_sel, l_prime, window)   make_testset.py:9-18
        (1, 8, 2, 512, 64, 4, 64, 128),
        (1, 8, 2, 512, 64, 16, 64, 128),
        (2, 16, 2, 1024, 128, 8, 64, 256),
        (1, 4, 4, 512, 64, 4, 64, 128),
        (1, 16, 1, 768, 64, 8, 128, 256),
        (1, 8, 2, 500, 64, 4, 64, 128),
        (1, 8, 2, 512, 64, 1, 256, 64),
        (1, 8, 2, 2048, 128, 16, 64, 512),
    ]
    cases = [(f"nsa_full_{i}", *shape, 200 + i, False) for i, shape in enumerate(grid)]
    cases.append(("nsa_full_bigrow", *grid[0], 250, True))
    for name, B, Hq, Hkv, S, D, n_sel, lp, w, seed, big in cases:
        q, k, v = qkv(B, Hq, Hkv, S, D, D, seed)
        if big:
            q = q.clone()
            q[..., 0, :] = (q[..., 0, :].float() * 50.0).to(torch.bfloat16)
        o64, sel = nsa_forward(q, k, v, n_sel=n_sel, l_prime=lp, window=w, dtype=torch.float64)
        # block scores as select_blocks ranks them (fp64)
        G = Hq // Hkv
        Kc, _ = compress_kv(k.double(), v.double(), 32, 16)
        qg = q.double().view(B, Hkv, G, S, D).sum(2)
        sc = (qg @ Kc.transpose(-1, -2)) / (D ** 0.5)
        n_blk = (S + lp - 1) // lp
        src = torch.linspace(0, S - 1, Kc.shape[2])
        tgt = (src // lp).long().clamp(max=n_blk - 1)
        blk = torch.zeros(B, Hkv, S, n_blk, dtype=torch.float64)
        blk.index_add_(3, tgt, sc)
        qpos = torch.arange(S).view(-1, 1)
        bpos = torch.arange(n_blk).view(1, -1) * lp
        blk = blk.masked_fill((bpos > qpos).view(1, 1, S, n_blk), float("-inf"))
        rng = np.random.Generator(np.random.PCG64(77))
        brows = np.stack([rng.integers(0, B, 256), rng.integers(0, Hkv, 256), rng.integers(0, S, 256)], 1)
        o = o64.numpy()
        rec = dict(kind="nsa_forward_full", B=B, Hq=Hq, Hkv=Hkv, T=S, dqk=D, dv=D, LP=lp, BQ=1, n_sel=n_sel,
                   window=w, seed=seed, big_row=int(big), sha256=digest(q, k, v), sel=sel.numpy().astype(np.int32),
                   checksums=checksums(o, 1234), out_absmax=np.abs(o).max(),
                   blk_rows=brows.astype(np.int32), blk=blk.numpy()[brows[:, 0], brows[:, 1], brows[:, 2]])
        rows = np.stack([rng.integers(0, B, 256), rng.integers(0, Hq, 256), rng.integers(0, S, 256)], 1)
        rec["rows"] = rows.astype(np.int32)
        rec["o_rows"] = o[rows[:, 0], rows[:, 1], rows[:, 2]].astype(np.float64)
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), **{k2: np.asarray(v2) for k2, v2 in rec.items()})
        print("wrote", name)


def backward_cases(out_dir, ref_selected):
    """Gradients of the selected branch (the reference has no backward: its README (2).md:85):
    autograd through ``ref_only.ref_selected`` in fp64 (ref_only.py:2-20) with a seeded upstream
    gradient dO, per-token selection (BQ = 1), d = 128, G = 16 and 8.  Stored per case: SHA-256 of
    the bf16 Q, K, V and dO, the selection rows, and for each of dQ, dK, dV three full-tensor fp64
    checksums and 64 seeded fp64 rows."""
    cases = [
        # name, B, Hq, Hkv, T, D, n, l_prime, seed, edit
        ("bwd_rule0_g16", 1, 16, 1, 512, 128, 8, 64, 300, None),
        ("bwd_rule0_g8_b2", 2, 16, 2, 384, 128, 4, 64, 301, None),
        ("bwd_edges_t300", 1, 16, 2, 300, 128, 6, 64, 302, "edges"),
        ("bwd_lp128", 1, 16, 1, 512, 128, 3, 128, 303, None),
        ("bwd_bigrow", 1, 16, 1, 256, 128, 4, 64, 304, "bigrow"),
        ("bwd_lp256", 1, 16, 1, 600, 128, 2, 256, 305, None),
    ]
    for name, B, Hq, Hkv, T, D, n, lp, seed, edit in cases:
        q, k, v = qkv(B, Hq, Hkv, T, D, D, seed)
        if edit == "bigrow":  # make_testset.py:24-25: a large-magnitude query row
            q = q.clone()
            q[..., 0, :] = (q[..., 0, :].float() * 50.0).to(torch.bfloat16)
        sel = indices.rule0(B, Hkv, T, n, lp, seed=seed)
        if edit == "edges":  # repeats, padding in the middle, the scratch id n_blk, future blocks
            n_blk = (T + lp - 1) // lp
            t = np.arange(T)
            sel[..., t % 7 == 3, 1] = sel[..., t % 7 == 3, 0]
            sel[..., t % 5 == 1, n - 1] = -1
            sel[..., t % 11 == 4, 2] = n_blk
            fut = t % 13 == 6
            sel[..., fut, 3] = np.minimum(n_blk - 1, t[fut] // lp + 2)
        g = torch.Generator().manual_seed(seed + 1000)
        do = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
        Q, K, V = (x.double().requires_grad_() for x in (q, k, v))
        O = ref_selected(Q, K, V, torch.from_numpy(sel), lp, 1)
        O.backward(do.double())
        rec = dict(kind="ref_selected_backward", B=B, Hq=Hq, Hkv=Hkv, T=T, dqk=D, dv=D, LP=lp, BQ=1, n_sel=n,
                   seed=seed, big_row=int(edit == "bigrow"), sha256=digest(q, k, v), sha256_do=digest(do),
                   sel=sel.astype(np.int32))
        rng = np.random.Generator(np.random.PCG64(seed))
        for key, grad, H in (("dq", Q.grad, Hq), ("dk", K.grad, Hkv), ("dv", V.grad, Hkv)):
            x = grad.numpy()
            rows = np.stack([rng.integers(0, B, 64), rng.integers(0, H, 64), rng.integers(0, T, 64)], 1)
            rec[key + "_checksums"] = checksums(x, 1234)
            rec[key + "_rows"] = rows.astype(np.int32)
            rec[key + "_vals"] = x[rows[:, 0], rows[:, 1], rows[:, 2]].astype(np.float64)
            rec[key + "_absmax"] = np.abs(x).max()
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), **{k2: np.asarray(v2) for k2, v2 in rec.items()})
        print("wrote", name)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory holding ref_only.py and nsa_reference.py")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", choices=["selected", "nsa_full", "backward"], default=None,
                    help="generate one group of fixtures")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from nsa_reference import compress_kv, nsa_forward  # noqa: E402
    from ref_only import ref_selected  # noqa: E402

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if args.only in (None, "backward"):
        backward_cases(args.out, ref_selected)
    if args.only == "backward":
        return
    if args.only != "selected":
        nsa_full_cases(args.out, nsa_forward, compress_kv)
    if args.only == "nsa_full":
        return
    # ---- per-query-block selection: the reference kernel tests' shapes and rule (test_v2.py:8-20)
    qblock_cases = [
        # name, B, Hq, Hkv, S, D, KSEL, BQ, LP, seed, full
        ("qblock_g4_d64", 1, 8, 2, 512, 64, 4, 16, 64, 7, False),
        ("qblock_g8_d128", 1, 16, 2, 1024, 128, 8, 8, 64, 8, False),
        ("qblock_g1", 1, 4, 4, 512, 64, 4, 64, 64, 9, False),
        ("qblock_g16_bq4", 1, 16, 1, 1024, 64, 6, 4, 64, 10, False),
        ("qblock_lp128", 1, 8, 2, 1024, 128, 4, 8, 128, 11, False),
        ("qblock_lp256_nsel1", 1, 8, 2, 512, 64, 1, 16, 256, 12, False),
    ]
    for name, B, Hq, Hkv, S, D, KSEL, BQ, LP, seed, full in qblock_cases:
        q, k, v = qkv(B, Hq, Hkv, S, D, D, seed)
        sel = indices.perm_qblock(B, Hkv, S, KSEL, BQ, LP, seed=seed, heads_share=False)
        o = ref_selected(q, k, v, torch.from_numpy(sel), LP, BQ).numpy()
        lse = torch.logsumexp(masked_scores(q, k, torch.from_numpy(sel), LP, BQ), -1).numpy()
        store(args.out, name, dict(kind="ref_selected", B=B, Hq=Hq, Hkv=Hkv, T=S, dqk=D, dv=D, LP=LP, BQ=BQ, seed=seed),
              q, k, v, sel, o, lse, full)

    # ---- per-token selection (BASELINE index rules) through ref_selected with BQ = 1
    token_cases = [
        # name, B, Hq, Hkv, T, D, n, rule, seed, big_row, full
        ("token_cfg0", 1, 16, 1, 1024, 64, 8, "rule0", 0, False, False),
        ("token_s500_g1", 1, 2, 2, 500, 64, 6, "rule0", 1, False, False),
        ("token_bigrow", 1, 8, 2, 512, 64, 4, "rule0", 2, True, False),
        ("token_rule3_dk128", 1, 8, 1, 768, 128, 16, "rule3", 3, False, False),
        ("token_reuse", 2, 8, 2, 512, 64, 16, "rule0_reuse", 4, False, False),
    ]
    for name, B, Hq, Hkv, T, D, n, rule, seed, big, full in token_cases:
        q, k, v = qkv(B, Hq, Hkv, T, D, D, seed)
        if big:  # make_testset.py:24-25: a large-magnitude query row
            q = q.clone()
            q[..., 0, :] = (q[..., 0, :].float() * 50.0).to(torch.bfloat16)
        sel = indices.generate(rule, B=B, Hkv=Hkv, T=T, n=n, block=64, seed=seed)
        o = ref_selected(q, k, v, torch.from_numpy(sel), 64, 1).numpy()
        lse = torch.logsumexp(masked_scores(q, k, torch.from_numpy(sel), 64, 1), -1).numpy()
        store(args.out, name, dict(kind="ref_selected", B=B, Hq=Hq, Hkv=Hkv, T=T, dqk=D, dv=D, LP=64, BQ=1, seed=seed,
                                   big_row=int(big)), q, k, v, sel, o, lse, full)

    # ---- d_qk != d_v through ref_selected (scale uses Q's last dim, ref_only.py:17)
    q, k, v = qkv(1, 8, 2, 512, 128, 64, 5)
    sel = indices.rule3(1, 2, 512, 8, 64, seed=5)
    o = ref_selected(q, k, v, torch.from_numpy(sel), 64, 1).numpy()
    lse = torch.logsumexp(masked_scores(q, k, torch.from_numpy(sel), 64, 1), -1).numpy()
    store(args.out, "token_dqk128_dv64", dict(kind="ref_selected", B=1, Hq=8, Hkv=2, T=512, dqk=128, dv=64, LP=64, BQ=1,
                                              seed=5), q, k, v, sel, o, lse, False)

    # ---- the selected branch of nsa_forward itself, per-token selection without padding
    B, Hq, Hkv, T, D, n = 1, 8, 2, 384, 64, 4
    q, k, v = qkv(B, Hq, Hkv, T, D, D, 6)
    sel = indices.rule0(B, Hkv, T, n, 64, seed=6)
    sel = np.where(sel < 0, 0, sel).astype(np.int64)  # nsa_forward cannot take -1 (nsa_reference.py:74)
    gates = [torch.tensor(gw, dtype=torch.float64) for gw in ([0.0, 0.0, 0.0], [2.0, 0.0, -1.0], [-1.0, 1.5, 2.0])]
    outs, gs = [], []
    for gw in gates:
        o_full, _ = nsa_forward(q, k, v, n_sel=n, l_prime=64, window=128, gate_w=gw, dtype=torch.float64,
                                sel_override=torch.from_numpy(sel))
        outs.append(o_full.numpy())
        g = torch.sigmoid(gw)
        gs.append((g / g.sum()).numpy())
    A = np.array(gs)  # outs[i] = sum_j A[i, j] * branch_j
    branches = np.tensordot(np.linalg.inv(A), np.stack(outs), axes=(1, 0))
    o_sel = branches[1]
    lse = torch.logsumexp(masked_scores(q, k, torch.from_numpy(sel), 64, 1), -1).numpy()
    store(args.out, "nsa_forward_selected", dict(kind="nsa_forward", B=B, Hq=Hq, Hkv=Hkv, T=T, dqk=D, dv=D, LP=64, BQ=1,
                                                 seed=6), q, k, v, sel, o_sel, lse, False)


if __name__ == "__main__":
    main()
