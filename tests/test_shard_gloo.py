"""The multi-GPU partition exercised on CPU: two gloo ranks each compute their shard of the
selected-branch forward (with the oracle standing in for the kernel), gather, and must reproduce
the single-process result exactly.  Also checks that a rank that fails is reported to the others
through the process group instead of hanging them."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from nsa_hopper_b200 import indices, shard


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs():
    g = torch.Generator().manual_seed(0)
    B, Hq, Hkv, T, D = 1, 8, 4, 700, 64
    q = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    sel = indices.rule0(B, Hkv, T, 8, 64, seed=0)
    return q, k, v, sel


def _worker(rank, world, port, out_q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        q, k, v, sel = _inputs()
        B, Hkv, T = q.shape[0], k.shape[1], q.shape[2]
        rects = shard.plan(B, Hkv, T, world)[rank]
        if rank == fail_rank:
            raise RuntimeError("injected failure on the host before the collective")
        o = np.zeros((q.shape[0], q.shape[1], T, v.shape[3]))
        l = np.zeros((q.shape[0], q.shape[1], T))
        mask = np.zeros((q.shape[0], q.shape[1], T), np.float64)
        G = q.shape[1] // Hkv
        for b0, b1, t0, t1 in rects:
            oracle.forward(q, k, v, sel, 64, 1, bkv_range=(b0, b1), t_range=(t0, t1), out=o, lse_out=l, threads=1)
            for bkv in range(b0, b1):
                b, kvh = divmod(bkv, Hkv)
                mask[b, kvh * G:(kvh + 1) * G, t0:t1] = 1
        to = torch.from_numpy(o * mask[..., None])
        tl = torch.from_numpy(np.where(mask > 0, l, 0.0))
        dist.all_reduce(to)  # shards are disjoint: a sum assembles them
        dist.all_reduce(tl)
        out_q.put((rank, "ok", to.numpy() if rank == 0 else None, tl.numpy() if rank == 0 else None))
    except Exception as e:  # report instead of hanging
        out_q.put((rank, f"error: {type(e).__name__}", None, None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q_.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return {r[0]: r for r in res}


def test_two_rank_shards_reassemble_exactly():
    res = _run(2)
    assert all(r[1] == "ok" for r in res.values())
    q, k, v, sel = _inputs()
    o, l = oracle.forward(q, k, v, sel, 64, 1, threads=1)
    np.testing.assert_array_equal(res[0][2], o)
    np.testing.assert_array_equal(res[0][3], l)


def test_failed_rank_is_reported_not_hung():
    res = _run(2, fail_rank=1)
    assert res[1][1].startswith("error")
    assert res[0][1].startswith("error")  # rank 0's collective ends with an error (peer gone / timeout)
