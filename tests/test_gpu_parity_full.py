"""Parity at the BASELINE configurations' full sizes (the shapes the bench line is quoted on),
kernel through the C ABI against the CPU oracle on the same inputs.

Inputs are generated on the device (seeded N(0,1) rounded to bf16; the oracle reads host copies
of exactly those values) with the BASELINE index rules of nsa_hopper_b200.workload.  The oracle
runs in fp32 on windows of token rows (oracle.forward_window), so no host copy of a whole Q or O
is needed.  Bars as everywhere: bf16 O max-abs <= 2e-2, LSE <= 1e-3 relative (floor |LSE| >= 1),
exact -inf pattern (rows with no visible key).

Coverage per configuration:
  ns    B=1 T=65536 Hq=64 Hkv=4 D=128 n=16, rule 0: every row of every KV head.
  cfg1  B=1 T=8192: every row.
  cfg2  B=4 T=32768, 30 % reuse: Q and O are 2^31 bytes each (byte offsets up to 2^31 - 1, element
        offsets past 2^30); rows 0 and 15 (the first and the highest addresses) whole, a
        2048-token range of every other row.
  cfg3  T=65536, d_qk=192, d_v=128, rule 3: KV head 0 whole, first and last 4096 tokens of the others.
  cfg4  the 16-sequence log-uniform varlen batch (G = 4): every row.
"""
import numpy as np
import pytest
import torch

import oracle
from nsa_hopper_b200 import capi, workload
from tests.helpers import compare

pytestmark = pytest.mark.gpu

WIN = 8192  # token rows per oracle call


def _run(name, seed=0):
    w = workload.CONFIGS[name]
    dev = torch.device("cuda")
    cu = None
    if w.n_seqs:
        _, cu = workload.varlen_setup(w, seed)
        T = int(cu[-1])
    else:
        T = w.T
    g = torch.Generator(device=dev).manual_seed(seed + 1000)
    q = torch.randn(w.B, w.Hq, T, w.d_qk, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(w.B, w.Hkv, T, w.d_qk, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(w.B, w.Hkv, T, w.d_v, device=dev, generator=g).to(torch.bfloat16)
    sel = workload.make_indices(w, seed=seed)
    assert sel.shape == (w.B, w.Hkv, T, w.n)
    sel_d = torch.from_numpy(sel).to(dev)
    cu_d = None if cu is None else torch.from_numpy(cu).to(dev)
    o = torch.full((w.B, w.Hq, T, w.d_v), float("nan"), device=dev, dtype=torch.bfloat16)
    lse = torch.full((w.B, w.Hq, T), float("nan"), device=dev, dtype=torch.float32)
    err = torch.zeros(1, device=dev, dtype=torch.int32)
    d = capi.make_desc(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), sel=sel_d.data_ptr(),
                       cu_seqlens=None if cu_d is None else cu_d.data_ptr(), n_seqs=0 if cu is None else len(cu) - 1,
                       o=o.data_ptr(), lse=lse.data_ptr(), err=err.data_ptr(), batch=w.B, heads_q=w.Hq,
                       heads_kv=w.Hkv, seq_len=T, d_qk=w.d_qk, d_v=w.d_v, n_qblocks=T, n_sel=w.n, block_size=w.block,
                       q_block=1, o_dtype=capi.DTYPE_BF16)
    capi.run(d, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return w, T, q, k, v, sel, cu, o, lse


def _check(w, T, q, k, v, sel, cu, o, lse, rows):
    """rows: list of (bkv, t0, t1); each range is compared in windows of WIN tokens."""
    G = w.G
    worst = {"o_max_abs": 0.0, "lse_max_rel": 0.0, "rows": 0}
    kv_host = {}
    for bkv, t0, t1 in rows:
        b, kvh = divmod(bkv, w.Hkv)
        if bkv not in kv_host:
            kv_host = {bkv: (k[b:b + 1, kvh:kvh + 1].contiguous().cpu(), v[b:b + 1, kvh:kvh + 1].contiguous().cpu(),
                             np.ascontiguousarray(sel[b:b + 1, kvh:kvh + 1]))}
        kh, vh, sh = kv_host[bkv]
        for a in range(t0, t1, WIN):
            e = min(t1, a + WIN)
            qh = q[b:b + 1, kvh * G:(kvh + 1) * G, a:e].contiguous().cpu()
            o_ref, l_ref = oracle.forward_window(qh, kh, vh, sh, w.block, 1, (a, e), cu_seqlens=cu)
            r = compare(o[b:b + 1, kvh * G:(kvh + 1) * G, a:e], lse[b:b + 1, kvh * G:(kvh + 1) * G, a:e],
                        o_ref.astype(np.float64), l_ref.astype(np.float64))
            worst["o_max_abs"] = max(worst["o_max_abs"], r["o_max_abs"])
            worst["lse_max_rel"] = max(worst["lse_max_rel"], r.get("lse_max_rel", 0.0))
            worst["rows"] += (e - a) * G
    print(f"{w.name}: {worst}")
    return worst


def test_north_star_every_row():
    w, T, *rest = _run("ns")
    r = _check(w, T, *rest, rows=[(bkv, 0, T) for bkv in range(w.B * w.Hkv)])
    assert r["rows"] == w.B * w.Hq * T


def test_config1_every_row():
    w, T, *rest = _run("cfg1", seed=1)
    _check(w, T, *rest, rows=[(bkv, 0, T) for bkv in range(w.B * w.Hkv)])


def test_config2_beyond_2gb_offsets():
    w, T, q, *rest = _run("cfg2", seed=2)
    assert q.numel() * q.element_size() >= (1 << 31)
    rng = np.random.default_rng(2)
    rows = [(0, 0, T), (w.B * w.Hkv - 1, 0, T)]
    for bkv in range(1, w.B * w.Hkv - 1):
        a = int(rng.integers(0, T - 2048))
        rows.append((bkv, a, a + 2048))
    _check(w, T, q, *rest, rows=rows)


def test_config3_dk192_full_length():
    w, T, *rest = _run("cfg3", seed=3)
    rows = [(0, 0, T)] + [(bkv, 0, 4096) for bkv in range(1, w.Hkv)] + [(bkv, T - 4096, T) for bkv in range(1, w.Hkv)]
    _check(w, T, *rest, rows=rows)


def test_config4_varlen_sixteen_sequences_every_row():
    w, T, q, k, v, sel, cu, o, lse = _run("cfg4", seed=4)
    assert len(cu) == 17 and T == int(cu[-1])
    _check(w, T, q, k, v, sel, cu, o, lse, rows=[(bkv, 0, T) for bkv in range(w.B * w.Hkv)])
