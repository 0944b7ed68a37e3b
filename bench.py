#!/usr/bin/env python
"""Throughput benchmark of the B200 FT.SEARCH KNN path.

Default workload: FLAT INT8 inner-product KNN over 1,000,000 x 1536 rows (1024-centre
L2-normalised Gaussian mixture, seed 1, per-row symmetric int8 with an fp32 scale),
1024-query batches, k = 10.  One step = one batch scored against the whole index and
reduced to the final top-k per query.  On N GPUs the rows are split into N contiguous
shards (strong scaling: the same total work), each rank scores its shard, an NCCL
all-gather exchanges the k candidates per query, and every rank merges them.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload flat_i8|flat_i8_b1|flat_f32|bq]

Rank 0 prints one JSON line.  `value` is whole-job queries/s timed on the device
(CUDA events on the launching stream, max over ranks, inputs resident in HBM);
`e2e` is the same metric through the C-ABI with host buffers (copies inside the
timed region).  `--impl reference` times the CPU oracle (the restatement of Pion's
open reference routines) on the host cores instead.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "KNN queries/sec (1536-d, k=10)"

WORKLOADS = {
    # name: rows, dim, centres, seed, batch, k, dtype
    "flat_i8": dict(rows=1_000_000, dim=1536, centres=1024, seed=1, batch=1024, k=10,
                    dtype="int8", desc="FLAT INT8 inner product, 1M x 1536, 1024-query batches"),
    "flat_i8_b1": dict(rows=1_000_000, dim=1536, centres=1024, seed=1, batch=1, k=10,
                       dtype="int8", desc="FLAT INT8 inner product, 1M x 1536, batch 1"),
    "flat_i8_10m": dict(rows=10_000_000, dim=1536, centres=4096, seed=4, batch=4096, k=10,
                        dtype="int8", desc="sharded FLAT INT8, 10M x 1536, 4096-query batches"),
}


def args_parse(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="flat_i8")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--rows", type=int, default=None,
                    help="override the index size (small cases for profiler captures)")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="target CPU work of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args(argv)


# ---------------------------------------------------------------- helpers --

def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profiled_traffic(key: str):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary
    (profiles/traffic.txt lines `workload kernel bytes_per_launch`), else None."""
    p = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        parts = line.split()
        if len(parts) >= 3 and parts[0] == key and not line.startswith("#"):
            try:
                return float(parts[2])
            except ValueError:
                return None
    return None


class ClockMonitor:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.dev), "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax.append(float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# --------------------------------------------------------------- reference arm --

def run_reference(a, wl):
    """CPU oracle timing (the restatement of Pion's open reference routines)."""
    world, rank, local = dist_env()
    if rank != 0:
        return 0
    import numpy as np
    import torch

    import oracle
    from pion_b200.workloads import mixture_torch

    oracle.build()
    batch = a.batch or wl["batch"]
    dev = f"cuda:{local}" if torch.cuda.is_available() else "cpu"
    _, qf = mixture_torch(wl["rows"], wl["dim"], wl["centres"], wl["seed"], batch, device=dev,
                          row_range=(0, 0))

    def q8(x):  # data preparation only: the reference's per-row quantiser in torch ops
        m = x.abs().amax(dim=1)
        scale = m / 127.0
        scale = torch.where(m == 0, torch.ones_like(scale), scale)
        inv = 1.0 / scale
        qv = x * inv[:, None]
        qi = torch.where(qv >= 0, torch.trunc(qv + 0.5), torch.trunc(qv - 0.5)).clamp(-127, 127)
        return qi.to(torch.int8).cpu().numpy(), scale.cpu().numpy()

    keys, ks = [], []
    for s in range(0, wl["rows"], 1 << 20):
        part, _ = mixture_torch(wl["rows"], wl["dim"], wl["centres"], wl["seed"], 0, device=dev,
                                row_range=(s, min(wl["rows"], s + (1 << 20))))
        a8, s8 = q8(part)
        keys.append(a8)
        ks.append(s8)
        del part
    keys, ks = np.concatenate(keys), np.concatenate(ks)
    q, qs = q8(qf)
    threads = os.cpu_count() or 1
    # size a step: throughput estimate on `threads` queries, then a sample per step so
    # that warmup + steps take about two minutes
    t0 = time.perf_counter()
    est_n = min(batch, threads)
    oracle.flat_i8_knn(keys, ks, q[:est_n], qs[:est_n], wl["k"], nthreads=threads)
    qps_est = est_n / (time.perf_counter() - t0)
    per_step = max(1, min(batch, int(120.0 * qps_est / max(1, a.steps + a.warmup))))
    for i in range(a.warmup):
        j = (i * per_step) % batch
        oracle.flat_i8_knn(keys, ks, q[j:j + per_step], qs[j:j + per_step], wl["k"],
                           nthreads=threads)
    t0 = time.perf_counter()
    done = 0
    for i in range(a.steps):
        j = (i * per_step) % max(1, batch - per_step + 1)
        oracle.flat_i8_knn(keys, ks, q[j:j + per_step], qs[j:j + per_step], wl["k"],
                           nthreads=threads)
        done += per_step
    dt = time.perf_counter() - t0
    qps = done / dt
    sample = (f"{per_step} queries of the {batch}-query batch per step against all "
              f"{wl['rows']:,} rows, {threads} threads (one query per thread)")
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s",
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": 1000.0 * dt / max(1, a.steps), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": wl["dtype"], "data": "synthetic",
        "config": {"workload": wl["desc"], "rows": wl["rows"], "dim": wl["dim"],
                   "batch": batch, "k": wl["k"], "seed": wl["seed"]},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------- our arm --

def run_ours(a, wl):
    import numpy as np
    import torch
    import torch.distributed as dist

    import pion_b200
    from pion_b200.workloads import mixture_torch

    world, rank, local = dist_env()
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # every kernel (torch's and ours) runs on one dedicated stream; the timing events
    # are recorded on it
    torch.cuda.set_stream(torch.cuda.Stream(device=dev))
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    batch = a.batch or wl["batch"]
    k = wl["k"]
    n, dim = wl["rows"], wl["dim"]
    lo, hi = n * rank // world, n * (rank + 1) // world
    ctx = pion_b200.Context(local)

    # ---- data: each rank draws only its shard (chunk-seeded, identical for any N)
    keys = torch.empty((hi - lo, dim), dtype=torch.int8, device=dev)
    ks = torch.empty(hi - lo, dtype=torch.float32, device=dev)
    piece = 1 << 20
    qf = None
    for s in range(lo, hi, piece):
        e = min(hi, s + piece)
        part, qq = mixture_torch(n, dim, wl["centres"], wl["seed"],
                                 batch if qf is None else 0, device=dev, row_range=(s, e))
        if qf is None:
            qf = qq
        kq, sq = pion_b200.quantize_rows_i8(ctx, part)
        keys[s - lo:e - lo] = kq
        ks[s - lo:e - lo] = sq
        del part, kq, sq
    if qf is None:
        _, qf = mixture_torch(n, dim, wl["centres"], wl["seed"], batch, device=dev,
                              row_range=(0, 0))
    q, qs = pion_b200.quantize_rows_i8(ctx, qf)
    torch.cuda.synchronize()
    ix = pion_b200.FlatI8Index(ctx, keys, ks, id_base=lo, borrow=True)
    ctx.use_torch_stream()
    stream = torch.cuda.current_stream()

    gathered_v = torch.empty((world, batch, k), dtype=torch.float32, device=dev)
    gathered_i = torch.empty((world, batch, k), dtype=torch.int32, device=dev)

    def step(qq, qqs):
        ids, sc = ix.search(qq, qqs, k)
        if world == 1:
            return ids, sc
        dist.all_gather_into_tensor(gathered_v, sc)
        dist.all_gather_into_tensor(gathered_i, ids)
        return pion_b200.merge_topk(ctx, gathered_v, gathered_i, k, descending=True,
                                    lists_major=True)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    for _ in range(max(3, a.warmup)):
        step(q, qs)
    barrier()

    clocks = ClockMonitor(local)
    clocks.start()
    ctx.timing(True)
    launches0 = ctx.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record(stream)
    for _ in range(a.steps):
        step(q, qs)
    ev1.record(stream)
    barrier()
    elapsed = ev0.elapsed_time(ev1)
    launches = ctx.launches - launches0
    kern_ms, kern_n = ctx.timing_read()
    ctx.timing(False)
    clk = clocks.stop()

    # ---- e2e: host (pinned) queries in, host results out, through the C ABI
    e2e_steps = a.e2e_steps or max(10, min(a.steps, 200))
    hq = torch.empty((batch, dim), dtype=torch.int8).pin_memory()
    hqs = torch.empty(batch, dtype=torch.float32).pin_memory()
    hq.copy_(q.cpu())
    hqs.copy_(qs.cpu())
    out_i = torch.empty((batch, k), dtype=torch.int32).pin_memory()
    out_v = torch.empty((batch, k), dtype=torch.float32).pin_memory()
    dq = torch.empty_like(q)
    dqs = torch.empty_like(qs)

    def e2e_step():
        if world == 1:  # the C-ABI host-buffer path (on the context's stream, set to the
            # dedicated stream above): copies, kernels, copies, sync
            ctx.check(ctx.lib.pion_v_b200_flat_i8_knn(ctx.h, ix.h, hq.data_ptr(), hqs.data_ptr(),
                                                      batch, k, out_i.data_ptr(),
                                                      out_v.data_ptr(), pion_b200._lib.MEM_HOST))
            return
        dq.copy_(hq, non_blocking=True)
        dqs.copy_(hqs, non_blocking=True)
        ids, sc = step(dq, dqs)
        out_i.copy_(ids, non_blocking=True)
        out_v.copy_(sc, non_blocking=True)
        stream.synchronize()

    for _ in range(3):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    h2d = batch * dim + batch * 4
    d2h = batch * k * 8

    # ---- max over ranks
    t = torch.tensor([elapsed, e2e_ms, kern_ms / max(1, kern_n)], device=dev, dtype=torch.float64)
    lt = torch.tensor([launches], device=dev, dtype=torch.int64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(lt, op=dist.ReduceOp.SUM)
    elapsed, e2e_ms, kern_avg_ms = t.tolist()
    launches = int(lt.item())

    line = None
    if rank == 0:
        qps = batch * a.steps / (elapsed / 1000.0)
        e2e_qps = batch * e2e_steps / (e2e_ms / 1000.0)
        peaks, peak_kind = measured_peaks()
        rows_local = hi - lo
        if batch > 1:
            ops = 2.0 * dim * rows_local * batch
            achieved = ops / (kern_avg_ms / 1000.0) / 1e12
            # the scoring kernel runs back to back for the whole timed region (hundreds of
            # ms under the 1 kW power cap), so the sustained figure is the denominator
            peak = 2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
            roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak,
                    "frac_of_burst": achieved / (2.0 * peaks["bf16_tflops"]),
                    "peak_source": f"2 x {peak_kind} dense bf16 sustained (int8 rate = 2 x bf16 "
                                   f"on B200); int8 tera-ops counted as TFLOP",
                    "algorithmic_per_launch": ops,
                    "kernel_ms": kern_avg_ms,
                    "traffic": profiled_traffic(f"{a.workload}_{world}")}
        else:
            byts = float(rows_local) * (dim + 4)
            achieved = byts / (kern_avg_ms / 1000.0) / 1e9
            peak = peaks["hbm_gbs"]
            roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                    "algorithmic_per_launch": byts, "kernel_ms": kern_avg_ms,
                    "traffic": profiled_traffic(f"{a.workload}_{world}")}
        line = {
            "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": elapsed / a.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": wl["dtype"],
            "data": "synthetic (seeded Gaussian mixture on the device)",
            "config": {"workload": wl["desc"], "rows": n, "dim": dim, "centres": wl["centres"],
                       "batch": batch, "k": k, "seed": wl["seed"],
                       "parallelism": f"row shards x{world}" + (" + NCCL all-gather"
                                                                if world > 1 else ""),
                       "l2": "index larger than L2 (no flush needed)"},
            "e2e": {"value": e2e_qps, "unit": "queries/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps},
            "gpu_launches": launches,
            "roofline": roof,
            "clocks": clk,
        }
    # ---- CPU baseline on rank 0 at N=1 (bounded sample of the same workload)
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_baseline(keys, ks, q, qs, k, batch, a.cpu_seconds)
        except Exception as e:  # pragma: no cover
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ix.free()
    ctx.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def cpu_baseline(keys, ks, q, qs, k, batch, seconds):
    import oracle
    oracle.build()
    hk, hks = keys.cpu().numpy(), ks.cpu().numpy()
    hq, hqs = q.cpu().numpy(), qs.cpu().numpy()
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    est = min(batch, threads)
    oracle.flat_i8_knn(hk, hks, hq[:est], hqs[:est], k, nthreads=threads)
    qps_est = est / (time.perf_counter() - t0)
    m = int(max(est, min(batch, qps_est * seconds)))
    t0 = time.perf_counter()
    oracle.flat_i8_knn(hk, hks, hq[:m], hqs[:m], k, nthreads=threads)
    dt = time.perf_counter() - t0
    return {"value": m / dt, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{m} of the {batch} queries against all {hk.shape[0]:,} rows "
                      f"({dt:.1f} s, one query per thread)"}


def main(argv=None):
    a = args_parse(argv)
    wl = dict(WORKLOADS[a.workload])
    if a.rows:
        wl["rows"] = a.rows
        wl["desc"] += f" (rows overridden: {a.rows:,})"
    if a.impl == "reference":
        return run_reference(a, wl)
    return run_ours(a, wl)


if __name__ == "__main__":
    sys.exit(main())
