"""Benchmark of the NSA selected-branch forward on B200 (one JSON line on rank 0).

Default: the north-star workload (B=1, T=65536, Hq=64, Hkv=4, D=128, block 64, top-n=16,
BASELINE rule 0 indices).  A "step" is one forward over the whole job.  Under torchrun the job is
split over the ranks by (batch*KV head, query-token range) rectangles (nsa_hopper_b200.shard:
``--scaling strong``, the default), with no collective on the data path; ``--scaling weak`` runs
one independent copy of the job per rank instead.  ``--config`` picks another BASELINE
configuration (cfg1, cfg2, cfg3, cfg4 varlen).

Timing: W untimed warm-up steps, then K steps, each timed with CUDA events on the launching
stream; between timed steps a 256 MiB buffer is written to flush L2 (outside the events).  The
timed loop is bracketed by a barrier and torch.cuda.synchronize(); the step time reported is the
max over ranks of each rank's mean.  ``e2e`` repeats the K steps through the C ABI's host-buffer
entry point (pinned host inputs in, O/LSE out, copies inside the timed region).

After timing, a seeded sample of output rows of every rank is compared with the CPU oracle
(checker use only: ``parity`` in the line), and the on-chip ceilings of the kernel's dataflow
are measured with the committed microbenchmarks (libnsa_peaks.so) for the roofline.

``--impl reference`` times the CPU implementation of the same path (the oracle restatement of
the reference's PyTorch code, fp32, all host threads) on the whole job, every step.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "selected-attn fwd TFLOP/s & tokens/s at T=64K, 1/2/4/8 B200; % of roofline"
FLUSH_BYTES = 256 << 20
O_TOL, LSE_TOL = 2e-2, 1e-3  # bf16 O max-abs, LSE relative (floor |LSE| >= 1)


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            j = json.load(f)
        return {"hbm_gbs": float(j["hbm_gbs"]), "bf16_tflops": float(j["bf16_tflops"]),
                "bf16_tflops_sustained": float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), "kind": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "kind": "fallback"}


def committed_traffic(workload: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture),
    read from the committed summary profiles/nsa_sel_fwd_<workload>_dram.md, or None."""
    path = os.path.join(REPO, "profiles", f"nsa_sel_fwd_{workload}_dram.md")
    try:
        with open(path) as f:
            m = re.search(r"dram_bytes_per_launch\s*=\s*([0-9.eE+]+)", f.read())
        return (float(m.group(1)), os.path.relpath(path, REPO)) if m else (None, None)
    except OSError:
        return None, None


class ClockSampler:
    """SM clock and throttle-reason sampling while the timed region runs.  NVML is read every
    10 ms from a thread that has taken its first sample before the region starts, so even a
    100 ms region gets about ten samples; where NVML cannot be loaded, nvidia-smi is polled
    every 200 ms instead.  Only reads: no clock or other GPU setting is touched."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h nvmlClocksEventReason*)
    REASON_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                   ("sw_power_cap", 0x4))

    def __init__(self, gpu_index: int, period_s: float = 0.01):
        self.gpu = gpu_index
        self.period = period_s
        self.proc = None
        self.out = ""
        self.samples = []  # (sm MHz, max sm MHz, reason names)
        self.source = None
        self._thread = None
        self._stop = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(self.gpu)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def _poll(self, nv, h, first):
        while True:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            except Exception:
                first.set()
                return
            self.samples.append((float(sm), float(mx), [n for n, b in self.REASON_BITS if bits & b]))
            first.set()
            if self._stop.wait(self.period):
                return

    def __enter__(self):
        import threading

        try:
            nv, h = self._nvml_handle()
            self._stop, first = threading.Event(), threading.Event()
            self._thread = threading.Thread(target=self._poll, args=(nv, h, first), daemon=True)
            self._thread.start()
            first.wait(2.0)
            if self.samples:
                self.source = f"nvml every {int(self.period * 1000)} ms"
                return self
            self._stop.set()
            self._thread.join(timeout=2.0)
            self._thread = None
        except Exception:
            self._thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi every 200 ms"
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2.0)
            try:
                import pynvml

                pynvml.nvmlShutdown()
            except Exception:
                pass
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                self.out = ""

    def summary(self):
        sm, mx, reasons = [], [], set()
        for a, b, r in self.samples:
            sm.append(a)
            mx.append(b)
            reasons.update(r)
        names = [n for n, _ in self.REASON_BITS]
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": self.source}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "source": self.source}


def reduce_op(x: float, world: int, op: str = "max") -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------------------- job
class Job:
    """The workload's shapes, indices and (for varlen) sequence table, identical on every rank."""

    def __init__(self, name: str, seed: int):
        from nsa_hopper_b200 import workload

        self.w = w = workload.CONFIGS[name]
        self.name, self.seed = name, seed
        self.cu = None
        if w.n_seqs:
            _, self.cu = workload.varlen_setup(w, seed)
            self.T = int(self.cu[-1])
        else:
            self.T = w.T
        self.sel = workload.make_indices(w, seed=seed)
        self.G = w.G

    def config(self, args, world):
        w = self.w
        par = (f"strong: one job split over {world} GPU(s) by (batch*KV head, token range) shards, no collective"
               if args.scaling == "strong" else f"weak: {world} independent copies of the job, one per GPU")
        c = {"workload": self.name, "B": w.B, "T": self.T, "Hq": w.Hq, "Hkv": w.Hkv, "d_qk": w.d_qk, "d_v": w.d_v,
             "block": w.block, "top_n": w.n, "rule": w.rule, "parallelism": par,
             "l2": "256 MiB buffer written between timed steps (L2 flushed)"}
        if self.cu is not None:
            c["n_seqs"] = len(self.cu) - 1
        return c


def rank_rects(job: Job, args, rank: int, world: int):
    from nsa_hopper_b200 import shard

    rows = job.w.B * job.w.Hkv
    if args.scaling == "weak" or world == 1:
        return [(0, rows, 0, job.T)]
    return shard.plan(job.w.B, job.w.Hkv, job.T, world, top_n=job.w.n, block=job.w.block)[rank]


def device_inputs(job: Job, seed: int, dev):
    """Q/K/V N(0,1) from a seeded device generator rounded to bf16 (the same values on every rank
    for the same seed); indices and the varlen table from the host generator."""
    import torch

    w = job.w
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(w.B, w.Hq, job.T, w.d_qk, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(w.B, w.Hkv, job.T, w.d_qk, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(w.B, w.Hkv, job.T, w.d_v, device=dev, generator=g).to(torch.bfloat16)
    sel = torch.from_numpy(job.sel).to(dev)
    cu = None if job.cu is None else torch.from_numpy(job.cu).to(dev)
    return q, k, v, sel, cu


def make_desc(job: Job, q, k, v, sel, cu, o, lse, err, rect):
    from nsa_hopper_b200 import capi

    w = job.w
    d = capi.make_desc(q=q, k=k, v=v, sel=sel, cu_seqlens=cu, n_seqs=0 if job.cu is None else len(job.cu) - 1,
                       o=o, lse=lse, err=err, batch=w.B, heads_q=w.Hq, heads_kv=w.Hkv, seq_len=job.T, d_qk=w.d_qk,
                       d_v=w.d_v, n_qblocks=job.T, n_sel=w.n, block_size=w.block, q_block=1,
                       o_dtype=capi.DTYPE_BF16)
    d.bkv_begin, d.bkv_end, d.qb_begin, d.qb_end = rect
    return d


def parity_sample(job: Job, q, k, v, o, lse, rects, seed: int, ntok: int = 128):
    """Compare a seeded sample of this rank's output rows with the CPU oracle (fp32): for every
    rectangle, its first and last (batch*KV head) row, each on its last `ntok` tokens and on one
    seeded window of `ntok` tokens.  Checker use only, after timing."""
    import oracle

    rng = np.random.default_rng(seed + 77)
    G, w = job.G, job.w
    worst_o, worst_l, nrows = 0.0, 0.0, 0
    for b0, b1, t0, t1 in rects:
        for bkv in sorted({b0, b1 - 1}):
            b, kvh = divmod(bkv, w.Hkv)
            kh = k[b:b + 1, kvh:kvh + 1].contiguous().cpu()
            vh = v[b:b + 1, kvh:kvh + 1].contiguous().cpu()
            sh = np.ascontiguousarray(job.sel[b:b + 1, kvh:kvh + 1])
            n = min(ntok, t1 - t0)
            starts = {t1 - n, int(rng.integers(t0, t1 - n + 1))}
            for a in sorted(starts):
                e = a + n
                qh = q[b:b + 1, kvh * G:(kvh + 1) * G, a:e].contiguous().cpu()
                o_ref, l_ref = oracle.forward_window(qh, kh, vh, sh, w.block, 1, (a, e), cu_seqlens=job.cu)
                og = o[b:b + 1, kvh * G:(kvh + 1) * G, a:e].float().cpu().numpy().astype(np.float64)
                lg = lse[b:b + 1, kvh * G:(kvh + 1) * G, a:e].cpu().numpy().astype(np.float64)
                worst_o = max(worst_o, float(np.abs(og - o_ref).max()))
                inf_ref = np.isneginf(l_ref)
                if not np.array_equal(np.isneginf(lg), inf_ref):
                    worst_l = float("inf")
                fin = ~inf_ref
                if fin.any():
                    worst_l = max(worst_l, float((np.abs(lg[fin] - l_ref[fin]) / np.maximum(np.abs(l_ref[fin]), 1.0)).max()))
                nrows += n * G
    return worst_o, worst_l, nrows


PEAKS_LIB = os.path.join(REPO, "nsa_hopper_b200", "libnsa_peaks.so")


def run_peaks_kernels(dev, modes=(0, 1, 2), n_chunks=4000, reps=3):
    """The committed on-chip ceiling microbenchmarks (nsa_hopper_b200/csrc/nsa_peaks.cu) on this
    GPU: per mode the best of `reps` launches of 148 CTAs x n_chunks 128-key chunks.  Returns
    {mode: {"ms", "gbs" (gathered bytes per second), "cycles_per_chunk" at the sampled clock}}."""
    import torch

    lib = ctypes.CDLL(PEAKS_LIB)
    lib.nsa_peaks_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 5 + [ctypes.c_void_p] * 2
    lib.nsa_peaks_run.restype = ctypes.c_int
    H, T = 4, 65536
    g = torch.Generator(device=dev).manual_seed(5)
    kk = torch.randn(H, T, 128, device=dev, generator=g).to(torch.bfloat16)
    vv = torch.randn(H, T, 128, device=dev, generator=g).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    st = torch.cuda.current_stream(dev)
    out = {}
    for mode in modes:
        best = None
        for _ in range(reps + 1):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            rc = lib.nsa_peaks_run(kk.data_ptr(), vv.data_ptr(), H, T, n_chunks, mode, sms, err.data_ptr(),
                                   ctypes.c_void_p(st.cuda_stream))
            e1.record(st)
            torch.cuda.synchronize()
            if rc != 0 or int(err.item()) != 0:
                raise RuntimeError(f"peaks microbenchmark mode {mode} failed (rc {rc}, err {int(err.item())})")
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        # the first launch is a warm-up; `best` includes it only if it was the fastest
        out[mode] = {"ms": best, "gbs": sms * n_chunks * 65536 / (best * 1e-3) / 1e9, "n_chunks": n_chunks, "ctas": sms}
    del kk, vv
    return out


def run_ours(args, rank, world, local_rank):
    import torch

    from nsa_hopper_b200 import capi, workload

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    job = Job(args.config, args.seed)
    w, T = job.w, job.T
    seed = args.seed + (rank if args.scaling == "weak" else 0)
    if args.scaling == "weak" and seed != args.seed:
        job = Job(args.config, seed)
    rects = rank_rects(job, args, rank, world)
    q, k, v, sel, cu = device_inputs(job, seed, dev)
    o = torch.empty(w.B, w.Hq, T, w.d_v, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(w.B, w.Hq, T, device=dev, dtype=torch.float32)
    err = torch.zeros(1, device=dev, dtype=torch.int32)
    flush = torch.empty(FLUSH_BYTES // 4, device=dev, dtype=torch.float32)
    work = workload.rect_work(w, job.sel, rects, T=T, cu_seqlens=job.cu)
    cu_ptr = None if cu is None else cu.data_ptr()
    descs = [make_desc(job, q.data_ptr(), k.data_ptr(), v.data_ptr(), sel.data_ptr(), cu_ptr, o.data_ptr(),
                       lse.data_ptr(), err.data_ptr(), r) for r in rects]
    stream = torch.cuda.current_stream(dev)
    sh_ = stream.cuda_stream

    def step():
        for d in descs:
            capi.run(d, sh_)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise RuntimeError(f"kernel reported device error {int(err.item())}")

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world)
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        barrier(world)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    mean_ms = statistics.mean(step_ms)
    max_ms = reduce_op(mean_ms, world)
    if int(err.item()) != 0:
        raise RuntimeError(f"kernel reported device error {int(err.item())}")

    # ---- parity of the timed launches' output (checker only, outside the timed region)
    p_o, p_l, p_rows = parity_sample(job, q, k, v, o, lse, rects, seed)
    p_o, p_l = reduce_op(p_o, world), reduce_op(p_l, world)
    p_rows = int(reduce_op(float(p_rows), world, "sum"))
    parity = {"o_max_abs": p_o, "lse_max_rel": p_l, "rows": p_rows, "tol_o_max_abs": O_TOL, "tol_lse_rel": LSE_TOL,
              "ok": bool(p_o <= O_TOL and p_l <= LSE_TOL),
              "sample": "per shard rectangle: its first and last (batch*KV head) row, last 128 tokens + one seeded "
                        "128-token window, against the fp32 CPU oracle"}

    # ---- end to end through the C ABI with host buffers, the same K steps
    e2e = None
    if not args.no_e2e:
        o_dev = o.clone()
        hq = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
        hk = torch.empty(k.shape, dtype=k.dtype, pin_memory=True)
        hv = torch.empty(v.shape, dtype=v.dtype, pin_memory=True)
        hs = torch.empty(sel.shape, dtype=sel.dtype, pin_memory=True)
        ho = torch.zeros(o.shape, dtype=o.dtype, pin_memory=True)
        hl = torch.empty(lse.shape, dtype=lse.dtype, pin_memory=True)
        hq.copy_(q)
        hk.copy_(k)
        hv.copy_(v)
        hs.copy_(sel)
        dq, dk, dv_, ds = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(sel)
        d_e2e = [make_desc(job, dq.data_ptr(), dk.data_ptr(), dv_.data_ptr(), ds.data_ptr(), cu_ptr, o.data_ptr(),
                           lse.data_ptr(), err.data_ptr(), r) for r in rects]
        G = job.G
        h2d = d2h = 0
        for b0, b1, t0, t1 in rects:  # bytes the host pipeline moves for this rank's rectangles
            rows = (b1 - b0) * (t1 - t0)
            h2d += (b1 - b0) * T * (w.d_qk + w.d_v) * 2 + rows * G * w.d_qk * 2 + rows * w.n * 4
            d2h += rows * G * (w.d_v * 2 + 4)
        io = capi.make_host_io(q=hq.data_ptr(), k=hk.data_ptr(), v=hv.data_ptr(), sel=hs.data_ptr(),
                               o=ho.data_ptr(), lse=hl.data_ptr())

        def e2e_step():
            # nsa_sel_run_host: H2D of slice i+1, the kernel on slice i and D2H of slice i-1 overlap
            for d in d_e2e:
                capi.run_host(d, io, sh_)

        e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        ev1.record(stream)
        barrier(world)
        e2e_ms = reduce_op(ev0.elapsed_time(ev1) / args.steps, world)
        same = True
        for b0, b1, t0, t1 in rects:  # host result of the e2e path == the device-timed launches' result
            for bkv in range(b0, b1):
                b, kvh = divmod(bkv, w.Hkv)
                sl = (b, slice(kvh * G, (kvh + 1) * G), slice(t0, t1))
                same &= bool(torch.equal(ho[sl].to(dev).view(torch.int16), o_dev[sl].view(torch.int16)))
        same = reduce_op(0.0 if same else 1.0, world) == 0.0
        ceil_ms = reduce_op(copy_ceiling(job, rects, (hq, hk, hv, hs), (dq, dk, dv_, ds), (ho, hl), (o, lse),
                                         args.steps, world), world)
        tok = (w.B * T) if args.scaling == "strong" else (w.B * T * world)
        e2e = {"value": tok / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(reduce_op(float(h2d), world, "sum")),
               "d2h_bytes_per_step": int(reduce_op(float(d2h), world, "sum")), "steps": args.steps,
               "host_result_equals_device": same,
               "copy_ceiling_ms": ceil_ms, "frac_of_copy_ceiling": ceil_ms / e2e_ms,
               "copy_ceiling_what": "the same H2D and D2H bytes of every rank, H2D and D2H on two streams at once, "
                                    "no kernel, max over ranks: the host-link floor of the e2e step",
               "path": "C ABI nsa_sel_run_host: pinned host Q/K/V/sel in, O/LSE out, copies pipelined with the kernel"}
        del hq, hk, hv, hs, ho, hl, dq, dk, dv_, ds, o_dev

    gather = None
    if world > 1 and not args.no_gather:
        gather = time_gather(o, lse, rects, job, world, stream)

    # ---- roofline: the committed on-chip ceiling microbenchmarks, measured now on this GPU
    peaks = measured_peaks()
    ceil = run_peaks_kernels(dev)
    kernel_s = mean_ms * 1e-3
    kv_gbs = work["kv_bytes"] / kernel_s / 1e9
    tf = work["flops"] / kernel_s / 1e12
    traffic, traffic_src = committed_traffic(args.config) if (world == 1 and args.config == "ns") else (None, None)
    clocks = clk.summary()
    n_launch = int(reduce_op(float(args.steps * len(descs)), world, "sum"))
    tokens_job = (w.B * T) if args.scaling == "strong" else (w.B * T * world)
    flops_job = reduce_op(work["flops"], world, "sum")
    if rank != 0:
        return None
    return {
        "metric": METRIC,
        "value": tokens_job / (max_ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": max_ms,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: N(0,1) Q/K/V rounded to bf16, seeded BASELINE index rule",
        "config": job.config(args, world),
        "tflops": flops_job / (max_ms * 1e-3) / 1e12,
        "parity": parity,
        "roofline": {
            "bound": "l2_to_smem_gather",
            "achieved": kv_gbs, "peak": ceil[0]["gbs"], "unit": "GB/s", "frac": kv_gbs / ceil[0]["gbs"],
            "peak_kind": "measured in this run: TMA gather of the kernel's own K/V boxes and rings, no compute "
                         "(libnsa_peaks.so mode 0)",
            "algorithmic_bytes_per_launch": work["kv_bytes"],
            "bytes_what": "gathered K/V bytes of rank 0's launches (every selected block with a visible key, once per "
                          "token, no cross-token reuse): the bytes TMA moves from L2 into shared memory",
            "kernel_ms": mean_ms,
            "traffic": traffic,
            "traffic_source": (f"committed one-pass ncu capture {traffic_src}" if traffic_src else None),
            "dataflow_peak": ceil[1]["gbs"], "dataflow_frac": kv_gbs / ceil[1]["gbs"],
            "dataflow_what": "the same gather feeding the kernel's 16 UMMAs per chunk (N = 16) from its three issuers, "
                             "no softmax (libnsa_peaks.so mode 1)",
            "umma_only_gbs": ceil[2]["gbs"],
            "tensor": {"achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": tf / peaks["bf16_tflops"],
                       "peak_kind": f"{peaks['kind']} (MEASURED_PEAKS.json bf16_tflops, burst)"},
            "hbm": {"achieved": work["bytes"] / kernel_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": work["bytes"] / kernel_s / 1e9 / peaks["hbm_gbs"],
                    "algorithmic_bytes_per_launch": work["bytes"],
                    "note": "all gathered bytes counted as if from HBM; they are L2 hits (DRAM carries the "
                            "compulsory traffic), so this is not a binding bound"},
        },
        "e2e": e2e,
        "gather": gather,
        "clocks": clocks,
        "gpu_launches": n_launch,
        "step_ms": step_ms,
    }


def copy_ceiling(job, rects, host_in, dev_in, host_out, dev_out, steps, world):
    """ms per step of the e2e step's host<->device copies alone: for every (batch*KV head) row of
    this rank's rectangles, its K and V rows and its heads' Q and index rows host->device on one
    stream while its heads' O and LSE rows go device->host on another (the same bytes the host
    pipeline moves), with no kernel.  Barrier-bracketed; the caller takes the max over ranks."""
    import torch

    w, G = job.w, job.G
    hq, hk, hv, hs = host_in
    dq, dk, dv, ds = dev_in
    ho, hl = host_out
    o, lse = dev_out
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def one():
        with torch.cuda.stream(s_in):
            for b0, b1, t0, t1 in rects:
                for bkv in range(b0, b1):
                    b, kvh = divmod(bkv, w.Hkv)
                    dk[b, kvh].copy_(hk[b, kvh], non_blocking=True)
                    dv[b, kvh].copy_(hv[b, kvh], non_blocking=True)
                    ds[b, kvh, t0:t1].copy_(hs[b, kvh, t0:t1], non_blocking=True)
                    for h in range(kvh * G, (kvh + 1) * G):
                        dq[b, h, t0:t1].copy_(hq[b, h, t0:t1], non_blocking=True)
        with torch.cuda.stream(s_out):
            for b0, b1, t0, t1 in rects:
                for bkv in range(b0, b1):
                    b, kvh = divmod(bkv, w.Hkv)
                    for h in range(kvh * G, (kvh + 1) * G):
                        ho[b, h, t0:t1].copy_(o[b, h, t0:t1], non_blocking=True)
                        hl[b, h, t0:t1].copy_(lse[b, h, t0:t1], non_blocking=True)

    one()
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    torch.cuda.synchronize()
    return (time.perf_counter() - t0) * 1e3 / steps


def time_gather(o, lse, rects, job, world, stream, reps: int = 3):
    """Optional NCCL all-gather of each rank's O (bf16) and LSE rows over NVLink, timed on its
    own after the forward's timed region (the forward itself needs no collective).  Each rank
    packs its shard's rows once, untimed; shards of unequal size are padded to the largest."""
    import torch
    import torch.distributed as dist

    G, Hkv = job.G, job.w.Hkv
    parts = []
    for b0, b1, q0, q1 in rects:
        for bkv in range(b0, b1):
            b, kvh = divmod(bkv, Hkv)
            parts.append(o[b, kvh * G:(kvh + 1) * G, q0:q1].reshape(-1).view(torch.uint8))
            parts.append(lse[b, kvh * G:(kvh + 1) * G, q0:q1].reshape(-1).view(torch.uint8))
    n = sum(p.numel() for p in parts)
    nmax = int(reduce_op(float(n), world))
    send = torch.zeros(nmax, dtype=torch.uint8, device=o.device)
    torch.cat(parts, out=send[:n])
    recv = torch.empty(nmax * world, dtype=torch.uint8, device=o.device)
    dist.all_gather_into_tensor(recv, send)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        dist.all_gather_into_tensor(recv, send)
    e1.record(stream)
    barrier(world)
    ms = reduce_op(e0.elapsed_time(e1) / reps, world)
    del recv, send
    return {"ms": ms, "bytes_per_rank": nmax, "busbw_gbs": nmax * (world - 1) / (ms * 1e-3) / 1e9,
            "what": "NCCL all_gather_into_tensor of each rank's O (bf16) + LSE rows, timed separately"}


# ------------------------------------------------------------------------------- CPU arms
def host_inputs(job: Job, seed: int):
    """The job's inputs generated on the host (seeded CPU generator, N(0,1) rounded to bf16)."""
    import torch

    w = job.w
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(w.B, w.Hkv, job.T, w.d_qk, generator=g).to(torch.bfloat16)
    v = torch.randn(w.B, w.Hkv, job.T, w.d_v, generator=g).to(torch.bfloat16)
    q = torch.randn(w.B, w.Hq, job.T, w.d_qk, generator=g).to(torch.bfloat16)
    return q, k, v


def cpu_forward_job(job: Job, q, k, v, threads: int, token_limit: int = 0, win: int = 8192) -> float:
    """The CPU oracle (fp32, `threads` host threads) over the job in (batch*KV head, token window)
    pieces; returns the seconds spent in the oracle.  token_limit > 0 runs only the last
    token_limit tokens of every row (the warm-up sample)."""
    import oracle

    w, G = job.w, job.G
    secs = 0.0
    for bkv in range(w.B * w.Hkv):
        b, kvh = divmod(bkv, w.Hkv)
        kh = k[b:b + 1, kvh:kvh + 1].contiguous()
        vh = v[b:b + 1, kvh:kvh + 1].contiguous()
        sh = np.ascontiguousarray(job.sel[b:b + 1, kvh:kvh + 1])
        t_start = max(0, job.T - token_limit) if token_limit > 0 else 0
        for a in range(t_start, job.T, win):
            e = min(job.T, a + win)
            qh = q[b:b + 1, kvh * G:(kvh + 1) * G, a:e].contiguous()
            t0 = time.perf_counter()
            oracle.forward_window(qh, kh, vh, sh, w.block, 1, (a, e), cu_seqlens=job.cu, threads=threads)
            secs += time.perf_counter() - t0
    return secs


def cpu_baseline(args):
    """The oracle (fp32, all host threads) on the whole job once: tokens/s."""
    import oracle

    job = Job(args.config, args.seed)
    q, k, v = host_inputs(job, args.seed)
    threads = oracle.default_threads()
    secs = cpu_forward_job(job, q, k, v, threads)
    return {"value": job.w.B * job.T / secs, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"the whole '{args.config}' job ({job.w.B * job.T} tokens x {job.w.Hq} heads), fp32 C oracle, "
                      f"{secs:.2f} s"}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU algorithm (its PyTorch code cannot travel to the GPU
    box, so the C restatement that is pinned to its golden vectors stands in), fp32, all host
    threads, the whole job on every timed step.  Warm-up steps run a small sample (the last 1024
    tokens of every row): a CPU path has nothing to warm beyond pages and threads."""
    if rank != 0:
        return None
    import oracle

    job = Job(args.config, args.seed)
    q, k, v = host_inputs(job, args.seed)
    threads = oracle.default_threads()
    for _ in range(args.warmup):
        cpu_forward_job(job, q, k, v, threads, token_limit=1024)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_forward_job(job, q, k, v, threads)
        times.append(time.perf_counter() - t0)
    sec = statistics.mean(times)
    val = job.w.B * job.T / sec
    return {
        "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic: N(0,1) Q/K/V rounded to bf16, seeded BASELINE index rule",
        "impl": "reference", "config": job.config(args, world),
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"the whole '{args.config}' job every step ({job.w.B * job.T} tokens x {job.w.Hq} "
                                   f"heads), fp32 C restatement of ref_only.py / nsa_reference.py"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0, "step_s": times,
    }


# ------------------------------------------------------------------------------- other stages
FP32_FMA_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # nominal: 148 SMs x 128 FP32 lanes x FMA at max clock


# The reference's own published sweep rows (per-query-block selection, fp32 O, its
# results/sweep2_unstaged.csv on an H200 at 1980 MHz): (G, BQ, D, LP, S, KSEL, v2 median ms).
REF_SWEEP_ROWS = [
    (16, 4, 128, 64, 32768, 16, 5.009), (16, 4, 128, 64, 32768, 32, 7.1844),
    (4, 16, 128, 64, 32768, 16, 1.302), (16, 4, 128, 128, 16384, 32, 10.5025),
    (16, 4, 128, 256, 32768, 32, 64.1757),
]


def run_refsweep(args):
    """--stage refsweep: the reference harness's protocol (sweep2.py: Hkv = 2, Hq = G * Hkv, one
    random permutation prefix of the visible blocks per query block shared by all heads, fp32 O
    through the reference op's signature with a cycle-counter tensor, as sweep2.py:48-49 passes
    one, median of timed launches) on the rows for which the reference publishes a time, with the
    same FLOP count (whole selected blocks)."""
    import torch

    from nsa_hopper_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    rows = []
    with ClockSampler(0) as clk:
        for G, BQ, D, LP, S, KSEL, ref_ms in REF_SWEEP_ROWS:
            Hkv, B = 2, 1
            Hq, NQB, nblk = G * Hkv, (S + BQ - 1) // BQ, S // LP
            q = torch.randn(B, Hq, S, D, device=dev, generator=gen).to(torch.bfloat16)
            k = torch.randn(B, Hkv, S, D, device=dev, generator=gen).to(torch.bfloat16)
            v = torch.randn(B, Hkv, S, D, device=dev, generator=gen).to(torch.bfloat16)
            qb = torch.arange(NQB, device=dev)
            avail = torch.clamp((qb * BQ) // LP + 1, min=1)
            key = torch.rand(NQB, nblk, device=dev, generator=gen)
            key = torch.where(torch.arange(nblk, device=dev).view(1, -1) < avail.view(-1, 1), key,
                              torch.full_like(key, 2.0))
            perm = key.argsort(dim=1)[:, :KSEL].to(torch.int32)
            keep = torch.arange(KSEL, device=dev).view(1, -1) < torch.clamp(avail, max=KSEL).view(-1, 1)
            sel = torch.where(keep, perm, torch.full_like(perm, -1)).view(1, 1, NQB, KSEL).expand(
                B, Hkv, NQB, KSEL).contiguous()
            cyc = torch.zeros(NQB * B * Hkv * 2, dtype=torch.int64, device=dev)
            for _ in range(args.warmup):
                ops.forward(q, k, v, sel, LP, BQ, cyc)
            ts = []
            for _ in range(max(args.steps, 5)):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                ops.forward(q, k, v, sel, LP, BQ, cyc)
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1))
            ms = statistics.median(ts)
            nsel = float((sel[0, 0] >= 0).float().sum().item()) / NQB
            flops = 2 * 2 * B * Hq * NQB * BQ * nsel * LP * D
            wait = cyc[0::2].double().sum().item()
            busy = cyc[1::2].double().sum().item()
            rows.append({"G": G, "BQ": BQ, "D": D, "LP": LP, "S": S, "KSEL": KSEL, "ms": round(ms, 4),
                         "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "ref_h200_ms": ref_ms,
                         "speedup_vs_ref": round(ref_ms / ms, 2),
                         "wait_pct": round(100 * wait / max(wait + busy, 1.0), 2)})
            del q, k, v, sel, cyc
    geo = math.exp(sum(math.log(r["speedup_vs_ref"]) for r in rows) / len(rows))
    return {"metric": "reference sweep rows: ms per launch vs the reference's published H200 ms",
            "value": round(geo, 3), "unit": "geomean speed-up", "n_gpus": 1, "steps": max(args.steps, 5),
            "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16 (fp32 O)",
            "data": "synthetic: N(0,1) bf16 Q/K/V, sweep2.py selection rule", "config": {"workload": "refsweep"},
            "rows": rows, "clocks": clk.summary()}


def run_peaks(args):
    """--stage peaks: the on-chip ceiling microbenchmarks (libnsa_peaks.so) alone: the TMA gather of
    the kernel's K/V boxes (mode 0), the gather feeding the kernel's UMMAs (mode 1) and the UMMAs on
    resident tiles (mode 2), in GB/s of gathered bytes and cycles per 128-key chunk."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    with ClockSampler(0) as clk:
        res = run_peaks_kernels(dev, modes=(0, 1, 2, 3, 4), reps=max(args.steps, 3))
    c = clk.summary()
    mhz = c["sm_mhz"] or 1965.0
    for m in res.values():
        m["cycles_per_chunk"] = m["ms"] * 1e-3 * mhz * 1e6 / m["n_chunks"]
    return {"metric": "on-chip ceilings of the selected-branch dataflow", "value": res[0]["gbs"], "unit": "GB/s",
            "n_gpus": 1, "steps": max(args.steps, 3), "warmup": 1, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic N(0,1) K/V, pseudo-random 64-key blocks", "config": {"workload": "peaks"},
            "modes": {"0_gather": res[0], "1_gather_umma": res[1], "2_umma_only": res[2],
                      "3_gather_cp_umma": res[3], "4_cp_umma_only": res[4]}, "clocks": c}


def run_select(args):
    """--stage select: the block-selection kernel (nsa_sel_select) on the workload's shapes.
    Algorithmic work per (b, kvh, token t): the group sum of G query rows (G*d adds) and one
    d-long dot product per visible block (t // l_prime + 1 of them); bytes: Q (bf16) in, k int32
    indices out.  For d = 64 and 128 the scores run on the tensor cores as three bf16 products
    (hi*hi + hi*lo + lo*hi), so the roofline counts 3 * 2 * d flops per visible (token, block)
    against the measured bf16 peak; other d run on the fp32 CUDA cores against the nominal fp32
    FMA peak (no measured figure exists for it on this pool)."""
    import torch

    from nsa_hopper_b200 import capi, workload

    w = workload.CONFIGS[args.config]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    B, T, Hq, Hkv, D, lp, n = w.B, w.T, w.Hq, w.Hkv, w.d_qk, w.block, w.n
    G = Hq // Hkv
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    q = torch.randn(B, Hq, T, D, device=dev, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device=dev, generator=gen).to(torch.bfloat16)
    n_blk = (T + lp - 1) // lp
    kk = min(n, n_blk)
    ws = torch.empty(capi.select_workspace_bytes(B, Hkv, T, D, lp) // 4, device=dev, dtype=torch.float32)
    sel = torch.empty(B, Hkv, T, kk, device=dev, dtype=torch.int32)
    flush = torch.empty(FLUSH_BYTES // 4, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)

    def step():
        capi.select(q.data_ptr(), k.data_ptr(), ws.data_ptr(), sel.data_ptr(), B, Hq, Hkv, T, D, lp, n, 32, 16,
                    stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(0) as clk:
        for i in range(args.steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = np.arange(T, dtype=np.float64)
    pairs = B * Hkv * float((t // lp + 1).sum())
    tensor = D in (64, 128)
    if tensor:
        pk = measured_peaks()
        flops = pairs * 3 * 2 * D
        peak, bound = pk["bf16_tflops"], "tensor"
        peak_kind = f"{pk['kind']} (MEASURED_PEAKS.json bf16_tflops, burst)"
    else:
        flops = pairs * 2 * D + B * Hkv * float(T * G * D)
        peak, bound, peak_kind = FP32_FMA_PEAK_TFLOPS, "fp32", "nominal"
    byts = B * Hkv * T * (G * D * 2 + kk * 4)
    achieved = flops / (ms * 1e-3) / 1e12
    return {
        "metric": "block selection (scores + top-k) tokens/s", "value": B * T / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 hi/lo split, fp32 accumulate" if tensor else "fp32 (bf16 inputs)",
        "data": "synthetic N(0,1) bf16 Q/K",
        "config": {"workload": args.config, "stage": "select", "B": B, "T": T, "Hq": Hq, "Hkv": Hkv, "d": D,
                   "block": lp, "top_n": n, "l2": "256 MiB buffer written between timed steps (L2 flushed)"},
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": None, "peak_kind": peak_kind,
                     "algorithmic_flops_per_launch": flops, "algorithmic_bytes_per_launch": byts,
                     "hbm_gbs": byts / (ms * 1e-3) / 1e9},
        "e2e": None, "clocks": clk.summary(), "gpu_launches": 2 * args.steps, "cpu_baseline": None,
    }


def run_backward(args):
    """--stage backward: the selected branch's backward (nsa_sel_backward: row sums dO.O, the
    inverse selection index and the tcgen05 gradient kernel), with the fp32 gradient buffers
    zeroed inside the timed step, on the workload's shapes (d = 128, G = 8 or 16).  Algorithmic
    FLOPs: five products of 2*d per (query row, visible key) -- S and dP recomputed, dV, dK, dQ
    -- i.e. 2.5x the forward's, against the measured bf16 tensor peak.  After timing, dQ of a
    128-token window per KV head is compared with the CPU restatement (oracle/backward.py) and the
    exact sum identities (dV summed over keys = dO summed over rows; dK summed over keys = 0) are
    checked on the whole output."""
    import torch

    import oracle.backward as obwd
    from nsa_hopper_b200 import capi, workload

    w = workload.CONFIGS[args.config]
    if w.n_seqs or w.d_qk != 128 or w.d_v != 128 or w.G not in (8, 16):
        raise SystemExit(f"--stage backward: workload {args.config} is outside the backward kernel "
                         "(d = 128, G = 8 or 16, no varlen)")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    B, T, Hq, Hkv, D, lp, n = w.B, w.T, w.Hq, w.Hkv, w.d_qk, w.block, w.n
    sel_np = workload.make_indices(w, args.seed)
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    q = torch.randn(B, Hq, T, D, device=dev, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device=dev, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, device=dev, generator=gen).to(torch.bfloat16)
    d_o = torch.randn(B, Hq, T, D, device=dev, generator=gen).to(torch.bfloat16)
    sel = torch.from_numpy(sel_np).to(dev)
    o = torch.empty(B, Hq, T, D, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, T, device=dev, dtype=torch.float32)
    err = torch.zeros(1, device=dev, dtype=torch.int32)
    stream = torch.cuda.current_stream(dev)
    fwd = capi.make_desc(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), sel=sel.data_ptr(), o=o.data_ptr(),
                         lse=lse.data_ptr(), err=err.data_ptr(), batch=B, heads_q=Hq, heads_kv=Hkv, seq_len=T,
                         d_qk=D, d_v=D, n_qblocks=T, n_sel=n, block_size=lp, q_block=1, o_dtype=capi.DTYPE_BF16)
    capi.run(fwd, stream.cuda_stream)
    dq = torch.empty(B, Hq, T, D, device=dev, dtype=torch.float32)
    dk = torch.empty(B, Hkv, T, D, device=dev, dtype=torch.float32)
    dv = torch.empty_like(dk)
    desc = capi.make_bwd_desc(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), sel=sel.data_ptr(), o=o.data_ptr(),
                              lse=lse.data_ptr(), d_o=d_o.data_ptr(), dq=dq.data_ptr(), dk=dk.data_ptr(),
                              dv=dv.data_ptr(), err=err.data_ptr(), batch=B, heads_q=Hq, heads_kv=Hkv, seq_len=T,
                              d=D, n_sel=n, block_size=lp, o_dtype=capi.DTYPE_BF16)
    ws = torch.empty(capi.backward_workspace_bytes(desc), device=dev, dtype=torch.uint8)
    desc.workspace = ws.data_ptr()
    flush = torch.empty(FLUSH_BYTES // 4, device=dev, dtype=torch.float32)

    def step():
        dq.zero_()
        dk.zero_()
        dv.zero_()
        capi.backward(desc, stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise RuntimeError(f"backward kernel reported device error {int(err.item())}")
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(0) as clk:
        for i in range(args.steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    if int(err.item()) != 0:
        raise RuntimeError(f"backward kernel reported device error {int(err.item())}")
    work = workload.algorithmic_work(w, sel_np)
    flops = 2.5 * work["flops"]
    pk = measured_peaks()
    achieved = flops / (ms * 1e-3) / 1e12
    # parity: dQ windows against the restatement, sum identities on everything
    G = Hq // Hkv
    qc, kc, vc, doc = q.cpu(), k.cpu(), v.cpu(), d_o.cpu()
    worst = 0.0
    for kvh in range(min(Hkv, 4)):
        h, t0 = kvh * G + (kvh * 5) % G, max(0, T - 128 - 997 * kvh)
        r = obwd.dq_rows(qc, kc, vc, sel_np, lp, doc, 0, h, t0, t0 + 128)
        x = dq[0, h, t0:t0 + 128].double().cpu().numpy()
        worst = max(worst, float(np.abs(x - r).max() / max(np.abs(r).max(), 1e-30)))
    sum_do = d_o.double().view(B, Hkv, G, T, D).sum((2, 3))
    dv_gap = float(((dv.double().sum(2) - sum_do).abs() / d_o.double().abs().view(B, Hkv, G, T, D).sum((2, 3))).max())
    dk_gap = float((dk.double().sum(2).abs() / dk.double().abs().sum(2).clamp_min(1e-30)).max())
    return {
        "metric": "selected-branch backward tokens/s", "value": B * T / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 in, bf16 P/dS, fp32 accumulate and gradients",
        "data": "synthetic N(0,1) bf16 Q/K/V/dO, seeded BASELINE index rule",
        "config": {"workload": args.config, "stage": "backward", "B": B, "T": T, "Hq": Hq, "Hkv": Hkv, "d": D,
                   "block": lp, "top_n": n, "l2": "256 MiB buffer written between timed steps (L2 flushed)",
                   "timed": "zeroing dQ/dK/dV + nsa_sel_backward (row sums, index, gradient kernel)"},
        "tflops": achieved,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / pk["bf16_tflops"], "traffic": None,
                     "peak_kind": f"{pk['kind']} (MEASURED_PEAKS.json bf16_tflops, burst)",
                     "algorithmic_flops_per_launch": flops},
        "parity": {"dq_window_scaled_err": worst, "dv_sum_identity_rel": dv_gap, "dk_sum_identity_rel": dk_gap,
                   "tol_scaled": 2e-2, "ok": worst <= 2e-2,
                   "sample": "dQ of a 128-token window of one head per KV head vs oracle/backward.py (fp64)"},
        "e2e": None, "clocks": clk.summary(), "gpu_launches": 6 * args.steps, "cpu_baseline": None,
    }


def run_nsa(args):
    """--stage nsa: the full NSA forward (nsa_hopper_b200.nsa.nsa_forward: compression, the block
    selection kernel, the selected / sliding-window / compressed branches on the attention kernel
    and the gate) on the workload's shapes, window 512 and the reference's compression
    (32 keys every 16).  Reports tokens/s of the whole layer and each stage's time."""
    import torch

    from nsa_hopper_b200 import nsa, ops, workload

    w = workload.CONFIGS[args.config]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    B, T, Hq, Hkv, D, lp, n = w.B, w.T, w.Hq, w.Hkv, w.d_qk, w.block, w.n
    window = 512
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    q = torch.randn(B, Hq, T, D, device=dev, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device=dev, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, device=dev, generator=gen).to(torch.bfloat16)
    flush = torch.empty(FLUSH_BYTES // 4, device=dev, dtype=torch.float32)
    for _ in range(args.warmup):
        nsa.nsa_forward(q, k, v, n_sel=n, l_prime=lp, window=window)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    with ClockSampler(0) as clk:
        for i in range(args.steps):
            flush.fill_(float(i))
            ev[i][0].record()
            nsa.nsa_forward(q, k, v, n_sel=n, l_prime=lp, window=window)
            ev[i][1].record()
        torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b_) for a, b_ in ev)
    # stage breakdown (one untimed-loop pass each, CUDA events)
    stages = {}

    def timed(name, fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        flush.fill_(0.0)
        e0.record()
        r = fn()
        e1.record()
        torch.cuda.synchronize()
        stages[name] = round(e0.elapsed_time(e1), 3)
        return r

    Kc, Vc = timed("compress_kv", lambda: nsa.compress_kv(k, v, 32, 16))
    sel = timed("select_kernel", lambda: ops.select_blocks(q, k, n, lp))
    timed("selected_branch", lambda: ops.forward(q, k, v, sel, lp, 1))
    timed("window_branch", lambda: nsa.window_branch_kernel(q, k, v, window))
    timed("compressed_branch", lambda: nsa.compressed_branch_kernel(q, Kc, Vc))
    return {
        "metric": "NSA forward (3 branches + selection + gate) tokens/s", "value": B * T / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 branch outputs)",
        "data": "synthetic N(0,1) bf16 Q/K/V",
        "config": {"workload": args.config, "stage": "nsa", "B": B, "T": T, "Hq": Hq, "Hkv": Hkv, "d": D, "block": lp,
                   "top_n": n, "window": window, "cmp_block": 32, "cmp_stride": 16,
                   "l2": "256 MiB buffer written between timed steps (L2 flushed)"},
        "stages_ms": stages, "e2e": None, "clocks": clk.summary(), "cpu_baseline": None,
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="ns", choices=["ns", "cfg1", "cfg2", "cfg3", "cfg4"])
    ap.add_argument("--scaling", choices=["weak", "strong"], default="strong",
                    help="strong: one job split over the ranks (default); weak: one copy of the job per rank")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gather", action="store_true", help="skip the separately timed all-gather (N > 1)")
    ap.add_argument("--stage", choices=["selected", "select", "nsa", "refsweep", "peaks", "backward"],
                    default="selected",
                    help="selected: the selected-branch forward (the headline); select: the block-selection kernel; "
                         "nsa: the full NSA forward; refsweep: the reference's published sweep rows; peaks: the "
                         "on-chip ceiling microbenchmarks; backward: the selected branch's backward")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    local_rank = _env_int("LOCAL_RANK", 0)

    if args.stage != "selected":
        if rank == 0:
            fn = {"select": run_select, "nsa": run_nsa, "refsweep": run_refsweep, "peaks": run_peaks,
                  "backward": run_backward}[args.stage]
            print(json.dumps(fn(args)), flush=True)
        return

    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    if world > 1:
        import torch
        import torch.distributed as dist

        # NCCL_DEBUG=VERSION prints a banner on stdout, where rank 0's JSON line must stand alone.
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        res = run_ours(args, rank, world, local_rank)
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                cb = cpu_baseline(args)
                res["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
            else:
                res["cpu_baseline"] = None
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
