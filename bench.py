#!/usr/bin/env python
"""Throughput benchmark of the B200 FT.SEARCH KNN path.

Default workload (`--workload flat_i8`): FLAT INT8 inner-product KNN over 1,000,000 x
1536 rows (1024-centre L2-normalised Gaussian mixture, seed 1, per-row symmetric int8
with an fp32 scale), 1024-query batches, k = 10.  One step = one batch scored against
the whole index and reduced to the final top-k per query.  On N GPUs the rows are split
into N contiguous shards (strong scaling: the same total work), each rank scores its
shard, an NCCL all-gather exchanges the k candidates per query, and every rank merges.

Other workloads: `flat_i8_b1` (the same index, one query per step), `flat_i8_10m`
(10M rows, 4096-query batches), `flat_f32` (FLAT FP32 cosine, 100,000 x 1536,
256 centres, 1000-query batches), `bq` (binary-quantised FLAT, 1M x 1536, Hamming
top-100 then fp32 cosine rerank to 10, 1024-query batches), `hnsw` (HNSW INT8 over 1M x
1536 rows of a 1024-centre mixture, seed 3, graph built on the host CPU with M = 16,
efConstruction = 200, GPU beam search at --ef (default 128), k = 10, 4096-query
batches; the line carries recall@10 against exact FLAT results).  HNSW does not shard
the graph: on N GPUs every rank holds the whole graph (built once on rank 0 and
broadcast) and serves its own 4096-query batch (weak scaling, N x 4096 queries per
step).  Like the reference's server (one query stream per worker thread), the HNSW bench
runs --workers contexts (default 3), each on its own CUDA stream, taking the batches in
turn, so the long tail of one batch (its slowest query does ~2.8x the mean work) overlaps
the start of the next; every batch is still one 4096-query call.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]

Rank 0 prints one JSON line.  `value` is whole-job queries/s timed on the device
(CUDA events on the launching stream, max over ranks, inputs resident in HBM);
`e2e` is the same metric through the C ABI with host buffers (copies inside the
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
    "flat_i8": dict(kind="i8", rows=1_000_000, dim=1536, centres=1024, seed=1, batch=1024, k=10,
                    desc="FLAT INT8 inner product, 1M x 1536, 1024-query batches"),
    "flat_i8_b1": dict(kind="i8", rows=1_000_000, dim=1536, centres=1024, seed=1, batch=1, k=10,
                       desc="FLAT INT8 inner product, 1M x 1536, batch 1"),
    "flat_i8_10m": dict(kind="i8", rows=10_000_000, dim=1536, centres=4096, seed=4, batch=4096,
                        k=10, desc="sharded FLAT INT8, 10M x 1536, 4096-query batches"),
    "flat_f32": dict(kind="f32", rows=100_000, dim=1536, centres=256, seed=0, batch=1000, k=10,
                     desc="FLAT FP32 cosine, 100K x 1536, 1000-query batches"),
    "flat_f32_b1": dict(kind="f32", rows=100_000, dim=1536, centres=256, seed=0, batch=1, k=10,
                        desc="FLAT FP32 cosine, 100K x 1536, batch 1 (exact HBM stream)"),
    "bq_b1": dict(kind="bq", rows=1_000_000, dim=1536, centres=1024, seed=2, batch=1, k=10,
                  desc="binary-quantised FLAT, 1M x 1536, batch 1 (popcount stream over the "
                       "192-byte codes, Hamming top-100, fp32 cosine rerank to 10)"),
    "bq": dict(kind="bq", rows=1_000_000, dim=1536, centres=1024, seed=2, batch=1024, k=10,
               desc="binary-quantised FLAT, 1M x 1536 (192-byte codes), Hamming top-100, "
                    "fp32 cosine rerank to 10, 1024-query batches"),
    "hnsw": dict(kind="hnsw", rows=1_000_000, dim=1536, centres=1024, seed=3, batch=4096, k=10,
                 M=16, ef_construction=200,
                 desc="HNSW INT8, 1M x 1536, M=16, efConstruction=200, 4096-query batches"),
    **{f"hnsw_{q}": dict(kind="quant", quant=q, rows=1_000_000, dim=1536, centres=1024, seed=3,
                          batch=4096, k=10, M=16, ef_construction=200,
                          desc=f"HNSW {name}, 1M x 1536, M=16, efConstruction=200, FP32 rerank, "
                               f"4096-query batches")
       for q, name in (("polar", "PolarQuant INT4"), ("nano", "NanoQuant INT2"),
                       ("turbo", "TurboQuant INT3 + QJL"))},
    "hnsw_brute": dict(kind="slot", rows=1_000_000, dim=1536, centres=1024, seed=3, batch=1024,
                       k=10, M=16, ef_construction=200,
                       desc="GPU brute-force scan of the HNSW slot buffer (INT8 L2 of every "
                            "slot, worst-replace top-20, FP32 rerank to 10), 1M x 1536, "
                            "1024-query batches"),
}


def args_parse(argv=None):
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="flat_i8")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--batch-sweep", default=None,
                    help="FLAT INT8: comma-separated batch sizes measured one after another on "
                         "the same index, one JSON line each (e.g. 1,64,4096)")
    ap.add_argument("--rows", type=int, default=None,
                    help="override the index size (small cases for profiler captures)")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="target CPU work of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ef", type=int, default=128, help="HNSW efSearch")
    ap.add_argument("--graph-cache", default=None,
                    help="HNSW workloads: load the graph from this index file (pion.hnsw.0 "
                         "format) when it exists, else build it and save it there")
    ap.add_argument("--build", choices=["lanes", "batched", "gpu"], default="lanes",
                    help="HNSW workloads: graph build -- the reference's parallel link lanes "
                         "(host), batched insertion on the host, or batched insertion with "
                         "the batches' searches on the GPU (the same graph as 'batched')")
    ap.add_argument("--build-batch", type=int, default=4096)
    ap.add_argument("--exchange", choices=["nccl", "peer", "peer-local"], default="nccl",
                    help="FLAT INT8 on N > 1 GPUs: the shards' lists cross NVLink through an "
                         "NCCL all-gather (each rank's own threshold sample), or through the "
                         "library's peer-memory exchange (with the threshold sample shared by "
                         "the ranks, or each rank's own sample share: peer-local)")
    ap.add_argument("--workers", type=int, default=None,
                    help="worker contexts (each its own CUDA stream) taking batches in turn; "
                         "default 3 for hnsw, 1 otherwise")
    return ap.parse_args(argv)


# ---------------------------------------------------------------- helpers --

def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
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
    """SM clocks, power and throttle reasons sampled DURING the timed region.

    A host thread reads them through NVML every `period_s` (read-only queries: clock,
    max clock, power, clocks-event reasons), so a timed region of a few tens of ms still
    gets several samples; nvidia-smi is the fallback when NVML is unavailable."""

    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40), ("sw_power_cap", 0x4))

    def __init__(self, device_index: int, period_s: float = 0.001):
        self.dev = device_index
        self.period = period_s
        self.samples = []
        self.thread = None
        self.proc = None
        self.path = None
        self.source = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid)
        except Exception:
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.dev]) if vis else self.dev
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(idx)

    def start(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.stop_flag = threading.Event()

            def run():
                while not self.stop_flag.is_set():
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                             float(smax), int(get_reasons(h)),
                                             nv.nvmlDeviceGetPowerUsage(h) / 1000.0))
                    except Exception:
                        pass
                    self.stop_flag.wait(self.period)
            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            self.source = f"NVML every {self.period * 1000:.0f} ms"
            return
        except Exception:
            self.thread = None
        try:  # fallback: nvidia-smi at its shortest loop period
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,"
                 "clocks_event_reasons.active,power.draw", "--format=csv,noheader,nounits",
                 "-i", str(self.dev), "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
            self.source = "nvidia-smi every 100 ms"
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
        elif self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()
            for line in open(self.path):
                p = [x.strip() for x in line.split(",")]
                try:
                    self.samples.append((float(p[0]), float(p[1]), int(p[2], 16),
                                         float(p[3])))
                except (ValueError, IndexError):
                    continue
            os.unlink(self.path)
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"],
                    "samples": 0}
        sm = [x[0] for x in self.samples]
        reasons = sorted({n for x in self.samples for n, bit in self.REASONS if x[2] & bit})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_min_mhz": min(sm) if sm else None,
                "sm_max_mhz": max(x[1] for x in self.samples) if sm else None,
                "power_w_max": max(x[3] for x in self.samples) if sm else None,
                "reasons": reasons, "samples": len(sm), "source": self.source}


def choose_regime(region_s: float, clk: dict) -> tuple:
    """Which measured peak fits the timed region: the burst figure (a kernel timed alone,
    clocks at max) when the region is shorter than 2 s or the median SM clock under load
    stayed within 5 % of max; the sustained figure (seconds under the 1 kW power cap)
    otherwise.  Returns (regime, reason)."""
    med, mx = clk.get("sm_mhz"), clk.get("sm_max_mhz")
    if region_s < 2.0:
        return "burst", f"timed region {region_s:.3f} s < 2 s"
    if med and mx and med >= 0.95 * mx:
        return "burst", f"median SM clock {med:.0f} MHz within 5 % of max {mx:.0f}"
    return "sustained", (f"timed region {region_s:.1f} s at median SM clock {med} MHz "
                         f"(max {mx})")


def tensor_peak(peaks, regime: str, factor: float):
    """(peak TFLOP/s, both candidates) for a tensor-bound kernel: `factor` x the measured
    dense bf16 figure of the regime (2 for int8, 1/3 for the 3 x bf16 split)."""
    burst = factor * peaks["bf16_tflops"]
    sus = factor * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    return (burst if regime == "burst" else sus), burst, sus


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def config_of(wl, batch, world, a=None):
    c = {"workload": wl["desc"], "rows": wl["rows"], "dim": wl["dim"],
         "centres": wl["centres"], "batch": batch, "k": wl["k"], "seed": wl["seed"],
         "parallelism": f"row shards x{world}" + (
             ((" + NVLink peer exchange" + (" (local bounds)" if a is not None and
                                              a.exchange == "peer-local" else ""))
              if (a is not None and a.exchange.startswith("peer")) and
              wl["kind"] == "i8" else " + NCCL all-gather") if world > 1 else ""),
         "l2": "index larger than L2 (no flush needed)"}
    if wl["kind"] == "hnsw":
        c.update({"M": wl["M"], "ef_construction": wl["ef_construction"],
                  "ef": a.ef if a is not None else None,
                  "parallelism": f"graph replicas x{world}, one batch per replica"})
    if wl["kind"] == "quant":
        c.update({"M": wl["M"], "ef_construction": wl["ef_construction"],
                  "ef": a.ef if a is not None else None, "quant": wl["quant"],
                  "parallelism": f"graph replicas x{world}, one batch per replica"})
    if wl["kind"] == "slot":
        c.update({"M": wl["M"], "ef_construction": wl["ef_construction"],
                  "oversample": 2 * wl["k"], "rerank": "fp32 rows by slot",
                  "parallelism": f"graph replicas x{world}, one batch per replica"})
    return c


# ------------------------------------------------------------ workloads --

class I8Workload:
    """FLAT INT8 inner product: rows quantised per row on the GPU (pkm_quantize_rows_i8)."""

    dtype = "int8"
    descending = True

    def __init__(self, wl, batch, dev, ctx, lo, hi):
        import torch

        import pion_b200
        from pion_b200.workloads import mixture_torch

        self.wl, self.batch, self.k, self.ctx = wl, batch, wl["k"], ctx
        n, dim = wl["rows"], wl["dim"]
        self.dim = dim
        keys = torch.empty((hi - lo, dim), dtype=torch.int8, device=dev)
        ks = torch.empty(hi - lo, dtype=torch.float32, device=dev)
        for s in range(lo, hi, 1 << 20):
            e = min(hi, s + (1 << 20))
            part, _ = mixture_torch(n, dim, wl["centres"], wl["seed"], 0, device=dev,
                                    row_range=(s, e))
            kq, sq = pion_b200.quantize_rows_i8(ctx, part)
            keys[s - lo:e - lo] = kq
            ks[s - lo:e - lo] = sq
            del part, kq, sq
        _, qf = mixture_torch(n, dim, wl["centres"], wl["seed"], batch, device=dev,
                              row_range=(0, 0))
        self.q, self.qs = pion_b200.quantize_rows_i8(ctx, qf)
        torch.cuda.synchronize()
        self.keys, self.ks = keys, ks
        self.ix = pion_b200.FlatI8Index(ctx, keys, ks, id_base=lo, borrow=True)

    def inputs(self):
        return [self.q, self.qs]

    def search(self, inp):
        return self.ix.search(inp[0], inp[1], self.k)

    def search_pairs(self, inp):
        return self.ix.search_pairs(inp[0], inp[1], self.k)

    def host_call(self, hin, out_i, out_v):
        import pion_b200
        c = self.ctx
        c.check(c.lib.pion_v_b200_flat_i8_knn(c.h, self.ix.h, hin[0].data_ptr(), hin[1].data_ptr(),
                                              self.batch, self.k, out_i.data_ptr(),
                                              out_v.data_ptr(), pion_b200._lib.MEM_HOST))

    def roofline(self, rows_local, kern_ms, peaks, peak_kind, regime="burst", phases=None):
        ops = 2.0 * self.dim * rows_local * self.batch
        byts = float(rows_local) * (self.dim + 4)
        t_ops = ops / (tensor_peak(peaks, regime, 2.0)[0] * 1e12)
        t_hbm = byts / (peaks["hbm_gbs"] * 1e9)
        if self.batch > 1 and t_ops >= t_hbm:  # enough queries per row for the tensor cores
            ops = 2.0 * self.dim * rows_local * self.batch
            achieved = ops / (kern_ms / 1000.0) / 1e12
            peak, burst, sus = tensor_peak(peaks, regime, 2.0)
            r = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                 "frac": achieved / peak, "regime": regime,
                 "frac_of_burst": achieved / burst, "frac_of_sustained": achieved / sus,
                 "peak_source": f"2 x {peak_kind} dense bf16 {regime} (int8 rate = 2 x bf16 "
                                f"on B200); int8 tera-ops counted as TFLOP",
                 "algorithmic_per_launch": ops, "kernel_ms": kern_ms,
                 "kernel_ms_covers": "threshold pass + its merge + main pass, per search"
                                    + (" + the shard exchanges" if phases and
                                       phases.get("exchange_ms") else "")}
            if phases and phases.get("main_ms"):
                r["main_pass_ms"] = phases["main_ms"]
                r["threshold_pass_ms"] = phases.get("threshold_ms")
                r["frac_main_pass"] = ops / (phases["main_ms"] / 1000.0) / 1e12 / peak
            if phases and phases.get("exchange_ms"):
                r["exchange_ms"] = phases["exchange_ms"]  # both exchanges, per search
                r["exchange_wait_ms"] = phases.get("exchange_wait_ms")
            return r
        # one query (the scan) or too few for the rows' bytes to be hidden: every row
        # streams from HBM once per batch
        achieved = byts / (kern_ms / 1000.0) / 1e9
        peak = peaks["hbm_gbs"]
        return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs (a copy: read "
                                                         f"+ write bytes)",
                "algorithmic_per_launch": byts, "kernel_ms": kern_ms,
                "tensor_frac": ops / (kern_ms / 1000.0) / 1e12 / tensor_peak(peaks, regime,
                                                                              2.0)[0]}

    def host_data(self):
        return (self.keys.cpu().numpy(), self.ks.cpu().numpy(), self.q.cpu().numpy(),
                self.qs.cpu().numpy())

    @staticmethod
    def cpu_run(data, lo, hi, k, threads):
        import oracle
        keys, ks, q, qs = data
        oracle.flat_i8_knn(keys, ks, q[lo:hi], qs[lo:hi], k, nthreads=threads)


class F32Workload:
    """FLAT FP32 cosine: rows normalised at registration (COSINE ingest)."""

    dtype = "fp32 (3 x bf16 split shortlist on tensor cores + exact fp32 rescore)"
    descending = False

    def __init__(self, wl, batch, dev, ctx, lo, hi):
        import torch

        import pion_b200
        from pion_b200.workloads import mixture_torch

        self.wl, self.batch, self.k, self.ctx = wl, batch, wl["k"], ctx
        n, dim = wl["rows"], wl["dim"]
        self.dim = dim
        rows, self.q = mixture_torch(n, dim, wl["centres"], wl["seed"], batch, device=dev,
                                     row_range=(lo, hi))
        torch.cuda.synchronize()
        self.ix = pion_b200.FlatF32Index(ctx, rows, id_base=lo)
        self.rows_raw = rows
        if batch == 1:
            self.dtype = "fp32 (exact 4-chain stream, no tensor cores)"

    def inputs(self):
        return [self.q]

    def search(self, inp):
        return self.ix.search(inp[0], self.k)

    def host_call(self, hin, out_i, out_v):
        import pion_b200
        c = self.ctx
        c.check(c.lib.pion_v_b200_flat_f32_knn(c.h, self.ix.h, hin[0].data_ptr(), self.batch,
                                               self.k, out_i.data_ptr(), out_v.data_ptr(),
                                               pion_b200._lib.MEM_HOST))

    def roofline(self, rows_local, kern_ms, peaks, peak_kind, regime="burst", phases=None):
        if self.batch == 1:  # the exact stream: every fp32 row once
            byts = float(rows_local) * self.dim * 4
            achieved = byts / (kern_ms / 1000.0) / 1e9
            return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                    "peak_source": f"{peak_kind} hbm_gbs",
                    "algorithmic_per_launch": byts, "kernel_ms": kern_ms,
                    "kernel_ms_covers": "query normalisation + the exact stream"}
        flops = 2.0 * self.dim * rows_local * self.batch
        achieved = flops / (kern_ms / 1000.0) / 1e12
        # three bf16 tensor passes per fp32 product (hi.hi + hi.lo + lo.hi)
        peak, burst, sus = tensor_peak(peaks, regime, 1.0 / 3.0)
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "regime": regime,
                "frac_of_burst": achieved / burst, "frac_of_sustained": achieved / sus,
                "peak_source": f"{peak_kind} dense bf16 {regime} / 3 (fp32 products as three "
                               f"bf16 passes); timed: query normalisation + bf16 split + "
                               f"tensor-core shortlist",
                "algorithmic_per_launch": flops, "kernel_ms": kern_ms}

    def host_data(self):
        import oracle
        return (oracle.l2_normalize_rows(self.rows_raw.cpu().numpy()), self.q.cpu().numpy())

    @staticmethod
    def cpu_run(data, lo, hi, k, threads):
        import oracle
        rows, q = data
        oracle.exact_knn(rows, q[lo:hi], k, cosine=True, nthreads=threads)


class BQWorkload:
    """Binary-quantised FLAT: sign codes + Hamming shortlist of 100, exact fp32 rerank."""

    dtype = "1-bit codes (int8 tensor-core Hamming) + fp32 rerank"
    descending = False
    shortlist = 100

    def __init__(self, wl, batch, dev, ctx, lo, hi):
        import torch

        import pion_b200
        from pion_b200.workloads import mixture_torch

        self.wl, self.batch, self.k, self.ctx = wl, batch, wl["k"], ctx
        n, dim = wl["rows"], wl["dim"]
        self.dim = dim
        rows, self.q = mixture_torch(n, dim, wl["centres"], wl["seed"], batch, device=dev,
                                     row_range=(lo, hi))
        torch.cuda.synchronize()
        self.ix = pion_b200.BQIndex(ctx, rows, id_base=lo)
        self.rows_raw = rows
        if batch == 1:
            self.dtype = "1-bit codes (popcount stream) + fp32 rerank"

    def inputs(self):
        return [self.q]

    def search(self, inp):
        return self.ix.search(inp[0], self.k, shortlist=self.shortlist)

    def host_call(self, hin, out_i, out_v):
        import pion_b200
        c = self.ctx
        c.check(c.lib.pion_v_b200_bq_rerank_knn(c.h, self.ix.h, hin[0].data_ptr(), self.batch,
                                                self.shortlist, self.k, out_i.data_ptr(),
                                                out_v.data_ptr(), pion_b200._lib.MEM_HOST))

    def roofline(self, rows_local, kern_ms, peaks, peak_kind, regime="burst", phases=None):
        if self.batch == 1:  # the popcount stream: every packed code once, 2-byte distances
            byts = float(rows_local) * (self.dim // 8 + 4)
            achieved = byts / (kern_ms / 1000.0) / 1e9
            return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                    "peak_source": f"{peak_kind} hbm_gbs",
                    "algorithmic_per_launch": byts, "kernel_ms": kern_ms,
                    "kernel_ms_covers": "query normalisation + signs + popcount stream + "
                                        "threshold + shortlist (rerank excluded)"}
        # Hamming of every (query, row) pair as +-1 int8 dot products on the tensor cores
        ops = 2.0 * self.dim * rows_local * self.batch
        achieved = ops / (kern_ms / 1000.0) / 1e12
        peak, burst, sus = tensor_peak(peaks, regime, 2.0)
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "regime": regime,
                "frac_of_burst": achieved / burst, "frac_of_sustained": achieved / sus,
                "peak_source": f"2 x {peak_kind} dense bf16 {regime} (int8 rate); timed: query "
                               f"normalisation + signs + staged Hamming shortlist",
                "algorithmic_per_launch": ops, "kernel_ms": kern_ms}

    def host_data(self):
        import oracle
        rn = oracle.l2_normalize_rows(self.rows_raw.cpu().numpy())
        return (oracle.bq_pack_signs(rn), rn, self.q.cpu().numpy())

    @staticmethod
    def cpu_run(data, lo, hi, k, threads):
        import oracle
        codes, rows, q = data
        oracle.bq_knn(codes, rows, q[lo:hi], BQWorkload.shortlist, k, nthreads=threads)


class HNSWWorkload:
    """HNSW INT8: the graph is built on the host CPU (pion_v_b200_hnsw_build, the
    reference's FT.OPTIMIZE build) on rank 0, broadcast to the other ranks, registered on
    every GPU; each rank searches its own batch (replicas, no merge, weak scaling)."""

    dtype = "int8 codes (exact int32 L2), fp32 pool distances"
    descending = False
    replicas = True

    def __init__(self, wl, batch, dev, ctx, lo, hi, ef=128):
        import numpy as np
        import torch
        import torch.distributed as dist

        import pion_b200
        from pion_b200.workloads import mixture_torch

        self.wl, self.k, self.ctx, self.ef = wl, wl["k"], ctx, ef
        n, dim = wl["rows"], wl["dim"]
        self.dim = dim
        world = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
        _, qall = mixture_torch(n, dim, wl["centres"], wl["seed"], batch * world, device=dev,
                                row_range=(0, 0))
        self.q = qall[batch * rank:batch * (rank + 1)].contiguous()
        self.batch = batch
        self.queries_per_step = batch * world
        self.graph = None
        self.build_s = None
        if rank == 0:
            rows = torch.empty((n, dim), dtype=torch.float32)
            for s in range(0, n, 1 << 18):
                e = min(n, s + (1 << 18))
                part, _ = mixture_torch(n, dim, wl["centres"], wl["seed"], 0, device=dev,
                                        row_range=(s, e))
                rows[s:e] = part.cpu()
                del part
            cache = wl.get("graph_cache")
            if cache and os.path.exists(cache):
                self.graph = pion_b200.HNSWGraph.load(cache)
                if self.graph.layout.num_nodes != n:
                    raise SystemExit(f"{cache} holds {self.graph.layout.num_nodes} nodes, not {n}")
            else:
                t0 = time.perf_counter()
                how = wl.get("build", "lanes")
                self.graph = pion_b200.HNSWGraph(
                    rows.numpy(), M=wl["M"], ef_construction=wl["ef_construction"],
                    batch=wl.get("build_batch", 4096) if how != "lanes" else 0,
                    gpu=ctx if how == "gpu" else None)
                self.build_s = time.perf_counter() - t0
                self.build_how = how
                if cache:
                    self.graph.save(cache)
            self.rows_host = rows
            arrays = self.graph.arrays()
        else:
            arrays = None
        if world > 1:
            arrays = self._broadcast(arrays, dev, rank)
        self.arrays = arrays
        self.ix = pion_b200.HNSWIndex(ctx, self.graph if rank == 0 else arrays)
        torch.cuda.synchronize()

    @staticmethod
    def _broadcast(arrays, dev, rank):
        """Rank 0's layout to every rank (NCCL broadcast of each buffer)."""
        import numpy as np
        import torch
        import torch.distributed as dist
        names = ["compact_buffer", "l0_compact", "l0_slots", "node_slot", "node_ids",
                 "node_level", "upper_offset", "upper_links"]
        scal = ["num_nodes", "dim", "M", "entry_point", "max_level", "compact_stride",
                "compact_hdr", "upper_rows", "metric"]
        meta = torch.zeros(len(scal) + 2, dtype=torch.float64, device=dev)
        if rank == 0:
            meta[:len(scal)] = torch.tensor([float(arrays[x]) for x in scal], dtype=torch.float64)
            meta[len(scal)] = float(arrays["global_min"])
            meta[len(scal) + 1] = float(arrays["global_max"])
        dist.broadcast(meta, 0)
        m = meta.tolist()
        out = {x: int(m[i]) for i, x in enumerate(scal)}
        out["global_min"], out["global_max"] = m[len(scal)], m[len(scal) + 1]
        out["global_min"] = float(np.float32(out["global_min"]))
        out["global_max"] = float(np.float32(out["global_max"]))
        for nm in names:
            if rank == 0:
                a = np.ascontiguousarray(arrays[nm])
                t = torch.from_numpy(a.view(np.uint8).reshape(-1)).to(dev)
                shp = torch.tensor(list(a.shape) + [0] * (2 - a.ndim), device=dev)
            else:
                shp = torch.zeros(2, dtype=torch.int64, device=dev)
            dist.broadcast(shp, 0)
            dt = {"compact_buffer": np.int8, "node_ids": np.int32, "node_level": np.int8,
                  "upper_offset": np.int64}.get(nm, np.uint32)
            shape = [int(x) for x in shp.tolist() if x > 0] if nm not in (
                "node_slot", "node_ids", "node_level", "upper_offset") else [int(shp[0])]
            nbytes = int(np.prod(shape)) * np.dtype(dt).itemsize
            if rank != 0:
                t = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            dist.broadcast(t, 0)
            out[nm] = t.cpu().numpy().view(dt).reshape(shape)
        out["deleted"] = None
        return out

    def inputs(self):
        return [self.q]

    def search(self, inp, ctx=None):
        return self.ix.search(inp[0], self.k, self.ef, ctx=ctx)

    def host_call(self, hin, out_i, out_v, ctx=None):
        import pion_b200
        c = ctx or self.ctx
        c.check(c.lib.pion_v_b200_hnsw_search(c.h, self.ix.h, hin[0].data_ptr(), self.batch,
                                              self.k, self.ef, out_i.data_ptr(),
                                              out_v.data_ptr(), pion_b200._lib.MEM_HOST))

    def roofline(self, rows_local, kern_ms, peaks, peak_kind, regime="burst", phases=None):
        st = self.ix.last_stats()
        byts = float(st["evals"] + st["upper_evals"]) * 1544.0 + st["expansions"] * 264.0
        # with several workers the batches overlap: kern_ms is then the time per batch
        # of the whole run (elapsed / steps), not a single launch's duration
        achieved = byts / (kern_ms / 1000.0) / 1e9
        peak = peaks["hbm_gbs"]
        return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                "algorithmic_per_launch": byts, "kernel_ms": kern_ms,
                "work_per_query": {k: v / max(1, self.batch) for k, v in st.items()},
                "note": "random 1.5 KB gathers, latency-bound: bytes = (level-0 + upper-level "
                        "distance evaluations) x 1544 + expansions x 264"}

    def extra(self, dev):
        """recall@10 of this rank's results against exact FLAT FP32 cosine (rank 0)."""
        import numpy as np
        import torch

        import pion_b200
        if self.graph is None:
            return {}
        rows = self.rows_host.to(dev)
        flat = pion_b200.FlatF32Index(self.ctx, rows)
        truth, _ = flat.search(self.q, self.k)
        ids, _ = self.ix.search(self.q, self.k, self.ef)
        t, r = truth.cpu().numpy(), ids.cpu().numpy()
        recall = float(np.mean([len(set(r[i]) & set(t[i])) / self.k for i in range(len(t))]))
        flat.free()
        del rows
        torch.cuda.empty_cache()
        return {"recall_at_10": recall, "ef": self.ef, "build_s": self.build_s,
                "build": getattr(self, "build_how", "cache"),
                "build_threads": os.cpu_count()}

    def host_data(self):
        return (self.graph.arrays(), self.q.cpu().numpy(), self.ef)

    @staticmethod
    def cpu_run(data, lo, hi, k, threads):
        import oracle
        arrays, q, ef = data
        oracle.hnsw_search(arrays, q[lo:hi], k, ef, nthreads=threads)


class SlotWorkload(HNSWWorkload):
    """search_gpu_brute_force over the HNSW slot buffer: every slot's INT8 L2 on the
    tensor cores, the worst-replace top-(2k) loop, FP32 rerank rows by slot, top k.
    The graph comes from the same host build as the hnsw workload (it fixes the slot
    order); replicas across GPUs, weak scaling."""

    dtype = "int8 codes (exact int32 dot products), fp32 rerank"

    def __init__(self, wl, batch, dev, ctx, lo, hi, ef=128):
        import numpy as np
        import torch

        from pion_b200.workloads import mixture_torch
        super().__init__(wl, batch, dev, ctx, lo, hi, ef)
        n, dim = wl["rows"], wl["dim"]
        slot = torch.from_numpy(np.ascontiguousarray(self.arrays["node_slot"]
                                                     if self.graph is None
                                                     else self.graph.arrays()["node_slot"])
                                .astype(np.int64)).to(dev)
        rr = torch.empty((n, dim), dtype=torch.float32, device=dev)
        for s in range(0, n, 1 << 18):
            e = min(n, s + (1 << 18))
            part, _ = mixture_torch(n, dim, wl["centres"], wl["seed"], 0, device=dev,
                                    row_range=(s, e))
            rr[slot[s:e]] = part
            del part
        self.ix.set_rerank_rows(rr)
        del rr
        torch.cuda.synchronize()

    def search(self, inp, ctx=None):
        return self.ix.brute_force(inp[0], self.k, ctx=ctx)

    def host_call(self, hin, out_i, out_v, ctx=None):
        import torch

        import pion_b200
        c = ctx or self.ctx
        found = getattr(self, "_found", None)
        if found is None or found.numel() != self.batch:
            found = self._found = torch.empty(self.batch, dtype=torch.int32).pin_memory()
        c.check(c.lib.pion_v_b200_hnsw_brute_force(c.h, self.ix.h, hin[0].data_ptr(), self.batch,
                                                   self.k, out_i.data_ptr(), out_v.data_ptr(),
                                                   found.data_ptr(), pion_b200._lib.MEM_HOST))

    def roofline(self, rows_local, kern_ms, peaks, peak_kind, regime="burst", phases=None):
        st = self.ix.slot_stats()
        ops = 2.0 * self.dim * self.wl["rows"] * self.batch
        achieved = ops / (kern_ms / 1000.0) / 1e12
        peak, burst, sus = tensor_peak(peaks, regime, 2.0)
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "regime": regime,
                "frac_of_burst": achieved / burst, "frac_of_sustained": achieved / sus,
                "peak_source": f"2 x {peak_kind} dense bf16 {regime} (int8 rate); timed: the "
                               f"staged tensor-core scan and the top-k replay",
                "algorithmic_per_launch": ops, "kernel_ms": kern_ms,
                "replayed_per_query": st["replayed"] / max(1, self.batch),
                "exact_scan_queries": st["exact_queries"]}

    def extra(self, dev):
        """recall@10 against exact FLAT FP32 cosine (rank 0)."""
        import numpy as np
        import torch

        import pion_b200
        if self.graph is None:
            return {}
        rows = self.rows_host.to(dev)
        flat = pion_b200.FlatF32Index(self.ctx, rows)
        truth, _ = flat.search(self.q, self.k)
        ids, _, _ = self.ix.brute_force(self.q, self.k)
        t, r = truth.cpu().numpy(), ids.cpu().numpy()
        recall = float(np.mean([len(set(r[i]) & set(t[i])) / self.k for i in range(len(t))]))
        flat.free()
        del rows
        torch.cuda.empty_cache()
        return {"recall_at_10": recall, "build_s": self.build_s}

    def host_data(self):
        import numpy as np
        A = self.graph.arrays()
        rr = np.empty_like(self.rows_host.numpy())
        rr[A["node_slot"]] = self.rows_host.numpy()
        return (A, self.q.cpu().numpy(), rr)

    @staticmethod
    def cpu_run(data, lo, hi, k, threads):
        from concurrent.futures import ThreadPoolExecutor

        import oracle
        A, q, rr = data
        chunks = [(s, min(hi, s + 1)) for s in range(lo, hi)]
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(lambda c: oracle.hnsw_brute_force(A, q[c[0]:c[1]], k, rr), chunks))


class QuantWorkload(HNSWWorkload):
    """The block-quantised HNSW search (PolarQuant / NanoQuant / TurboQuant): the graph of
    the hnsw workload, its slots quantised on the host (pion_v_b200_hnsw_quantize) with the
    FP32 rows kept for the rerank; replicas across GPUs, weak scaling."""

    dtype = "int4 / int2 / int3 + QJL block codes (exact int32 block dots), fp32 rerank"

    def __init__(self, wl, batch, dev, ctx, lo, hi, ef=128):
        import numpy as np
        import torch
        import torch.distributed as dist

        import pion_b200
        super().__init__(wl, batch, dev, ctx, lo, hi, ef)
        self.ix.free()  # the INT8 registration is not used
        kind = wl["quant"]
        self.dtype = {"polar": "int4", "nano": "int2", "turbo": "int3 + 1-bit QJL"}[kind] + \
            " block codes (exact int32 block dots), fp32 block sums and rerank"
        world = dist.get_world_size() if dist.is_initialized() else 1
        self.quant_s = None
        if self.graph is not None:
            t0 = time.perf_counter()
            self.quant = pion_b200.HNSWQuant(self.graph, self.rows_host.numpy(), kind)
            self.quant_s = time.perf_counter() - t0
            qa = self.quant.arrays()
        else:
            self.quant, qa = None, None
        if world > 1:
            qa = self._broadcast_quant(qa, kind, dev)
        self.qarrays = qa
        self.ix = pion_b200.HNSWQuantIndex(ctx, self.graph if self.graph is not None
                                           else self.arrays, self.quant or qa)
        self._found = {}
        torch.cuda.synchronize()

    @staticmethod
    def _broadcast_quant(qa, kind, dev):
        import numpy as np
        import torch
        import torch.distributed as dist
        rank = dist.get_rank()
        names = ["compact", "rerank"] + (["qjl", "qjl_res_norms", "qjl_random_signs"]
                                         if kind == "turbo" else [])
        dts = {"compact": np.int8, "rerank": np.float32, "qjl": np.uint64,
               "qjl_res_norms": np.float32, "qjl_random_signs": np.uint64}
        out = {"kind": kind, "qjl_lambda": 1.0}
        meta = torch.zeros(1, dtype=torch.int64, device=dev)
        if rank == 0:
            meta[0] = int(qa["stride"])
        dist.broadcast(meta, 0)
        out["stride"] = int(meta[0])
        for nm in names:
            if rank == 0:
                a = np.ascontiguousarray(qa[nm])
                shp = torch.tensor(list(a.shape) + [0] * (2 - a.ndim), device=dev)
                t = torch.from_numpy(a.view(np.uint8).reshape(-1)).to(dev)
            else:
                shp = torch.zeros(2, dtype=torch.int64, device=dev)
            dist.broadcast(shp, 0)
            shape = [int(x) for x in shp.tolist() if x > 0]
            nbytes = int(np.prod(shape)) * np.dtype(dts[nm]).itemsize
            if rank != 0:
                t = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            dist.broadcast(t, 0)
            out[nm] = t.cpu().numpy().view(dts[nm]).reshape(shape)
            del t
        return out

    def search(self, inp, ctx=None):
        ids, sc, _ = self.ix.search(inp[0], self.k, self.ef, ctx=ctx)
        return ids, sc

    def host_call(self, hin, out_i, out_v, ctx=None):
        import torch

        import pion_b200
        c = ctx or self.ctx
        found = self._found.get(id(c))
        if found is None:  # one pinned buffer per worker context
            found = self._found[id(c)] = torch.empty(self.batch, dtype=torch.int32).pin_memory()
        c.check(c.lib.pion_v_b200_hnsw_quant_search(c.h, self.ix.h, hin[0].data_ptr(),
                                                    self.batch, self.k, self.ef,
                                                    out_i.data_ptr(), out_v.data_ptr(),
                                                    found.data_ptr(), pion_b200._lib.MEM_HOST))

    def roofline(self, rows_local, kern_ms, peaks, peak_kind, regime="burst", phases=None):
        st = self.ix.last_stats()
        kind = self.wl["quant"]
        slot = 4 + 96 + {"polar": 768, "nano": 384, "turbo": 576}[kind] + \
            (196 if kind == "turbo" else 0)
        byts = float(st["evals"]) * slot + st["expansions"] * 264.0 + \
            self.batch * self.ef * 1536 * 4.0
        achieved = byts / (kern_ms / 1000.0) / 1e9
        peak = peaks["hbm_gbs"]
        return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                "algorithmic_per_launch": byts, "kernel_ms": kern_ms,
                "work_per_query": {k: v / max(1, self.batch) for k, v in st.items()},
                "note": f"random gathers, latency-bound: bytes = distance evaluations x {slot} "
                        f"(|v|^2, f16 scales, codes" + (", QJL row" if kind == "turbo" else "") +
                        ") + expansions x 264 + ef x 6144 (the FP32 rerank rows)"}

    def extra(self, dev):
        import numpy as np
        import torch

        import pion_b200
        if self.graph is None:
            return {}
        rows = self.rows_host.to(dev)
        flat = pion_b200.FlatF32Index(self.ctx, rows)
        truth, _ = flat.search(self.q, self.k)
        ids, _, _ = self.ix.search(self.q, self.k, self.ef)
        t, r = truth.cpu().numpy(), ids.cpu().numpy()
        recall = float(np.mean([len(set(r[i]) & set(t[i])) / self.k for i in range(len(t))]))
        flat.free()
        del rows
        torch.cuda.empty_cache()
        return {"recall_at_10": recall, "ef": self.ef, "quant": self.wl["quant"],
                "build_s": self.build_s, "quantize_s": self.quant_s,
                "rerank": "fp32 rows by node"}

    def host_data(self):
        return (self.graph.arrays(), self.quant.arrays(), self.q.cpu().numpy(), self.ef)

    @staticmethod
    def cpu_run(data, lo, hi, k, threads):
        import oracle
        A, Q, q, ef = data
        oracle.quant_search(A, Q, q[lo:hi], k, ef, nthreads=threads)


ADAPTERS = {"i8": I8Workload, "f32": F32Workload, "bq": BQWorkload, "hnsw": HNSWWorkload,
            "slot": SlotWorkload, "quant": QuantWorkload}


# --------------------------------------------------------------- reference arm --

def reference_data(wl, batch, dev):
    """The same workload on the host, prepared with plain torch/numpy and the oracle."""
    import numpy as np
    import torch

    import oracle
    from pion_b200.workloads import mixture_torch

    n, dim = wl["rows"], wl["dim"]
    _, qf = mixture_torch(n, dim, wl["centres"], wl["seed"], batch, device=dev, row_range=(0, 0))
    if wl["kind"] in ("hnsw", "slot", "quant"):  # the host build (restating the reference's)
        import pion_b200
        rows, _ = mixture_torch(n, dim, wl["centres"], wl["seed"], 0, device=dev)
        rows = rows.cpu().numpy()
        cache = wl.get("graph_cache")
        if cache and os.path.exists(cache):
            g = pion_b200.HNSWGraph.load(cache)
        else:
            g = pion_b200.HNSWGraph(rows, M=wl["M"], ef_construction=wl["ef_construction"])
        if wl["kind"] == "quant":
            qz = pion_b200.HNSWQuant(g, rows, wl["quant"])
            return (g.arrays(), qz.arrays(), qf.cpu().numpy(), wl["ef"]), (g, qz)
        if wl["kind"] == "slot":
            A = g.arrays()
            rr = np.empty_like(rows)
            rr[A["node_slot"]] = rows
            return (A, qf.cpu().numpy(), rr), g
        return (g.arrays(), qf.cpu().numpy(), wl["ef"]), g
    if wl["kind"] in ("f32", "bq"):
        rows, _ = mixture_torch(n, dim, wl["centres"], wl["seed"], 0, device=dev)
        rn = oracle.l2_normalize_rows(rows.cpu().numpy())
        if wl["kind"] == "bq":
            return oracle.bq_pack_signs(rn), rn, qf.cpu().numpy()
        return rn, qf.cpu().numpy()

    def q8(x):  # the reference's per-row quantiser in torch ops (data preparation only)
        m = x.abs().amax(dim=1)
        scale = m / 127.0
        scale = torch.where(m == 0, torch.ones_like(scale), scale)
        inv = 1.0 / scale
        qv = x * inv[:, None]
        qi = torch.where(qv >= 0, torch.trunc(qv + 0.5), torch.trunc(qv - 0.5)).clamp(-127, 127)
        return qi.to(torch.int8).cpu().numpy(), scale.cpu().numpy()

    keys, ks = [], []
    for s in range(0, n, 1 << 20):
        part, _ = mixture_torch(n, dim, wl["centres"], wl["seed"], 0, device=dev,
                                row_range=(s, min(n, s + (1 << 20))))
        a8, s8 = q8(part)
        keys.append(a8)
        ks.append(s8)
        del part
    q, qs = q8(qf)
    return np.concatenate(keys), np.concatenate(ks), q, qs


def run_reference(a, wl):
    """CPU oracle timing (the restatement of Pion's open reference routines)."""
    world, rank, local = dist_env()
    if rank != 0:
        return 0
    import torch

    import oracle

    oracle.build()
    batch = a.batch or wl["batch"]
    dev = f"cuda:{local}" if torch.cuda.is_available() else "cpu"
    data = reference_data(wl, batch, dev)
    keep = None
    if wl["kind"] in ("hnsw", "slot", "quant"):
        data, keep = data
    run = ADAPTERS[wl["kind"]].cpu_run
    threads = os.cpu_count() or 1
    # size a step: throughput estimate on `threads` queries, then a sample per step so
    # that warmup + steps take about two minutes
    t0 = time.perf_counter()
    est_n = min(batch, threads)
    run(data, 0, est_n, wl["k"], threads)
    qps_est = est_n / (time.perf_counter() - t0)
    per_step = max(1, min(batch, int(120.0 * qps_est / max(1, a.steps + a.warmup))))
    for i in range(a.warmup):
        j = (i * per_step) % max(1, batch - per_step + 1)
        run(data, j, j + per_step, wl["k"], threads)
    t0 = time.perf_counter()
    done = 0
    for i in range(a.steps):
        j = (i * per_step) % max(1, batch - per_step + 1)
        run(data, j, j + per_step, wl["k"], threads)
        done += per_step
    dt = time.perf_counter() - t0
    qps = done / dt
    sample = (f"{per_step} queries of the {batch}-query batch per step against all "
              f"{wl['rows']:,} rows, {threads} threads (one query per thread)")
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s",
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": 1000.0 * dt / max(1, a.steps), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": ADAPTERS[wl["kind"]].dtype,
        "data": "synthetic", "config": config_of(wl, batch, 1, a),
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------- our arm --

def run_ours(a, wl):
    import torch
    import torch.distributed as dist

    import pion_b200
    from pion_b200.sharded import ShardedSearch, shard_bounds

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
    if a.batch_sweep:  # queries for the largest batch, sliced per batch size
        batch = max(int(x) for x in a.batch_sweep.split(","))
    k = wl["k"]
    n = wl["rows"]
    lo, hi = shard_bounds(n, world, rank)
    ctx = pion_b200.Context(local)
    if wl["kind"] in ("hnsw", "slot", "quant"):
        W = ADAPTERS[wl["kind"]](wl, batch, dev, ctx, lo, hi, ef=a.ef)
    else:
        W = ADAPTERS[wl["kind"]](wl, batch, dev, ctx, lo, hi)
    local_batch = W.batch
    ctx.use_torch_stream()
    stream = torch.cuda.current_stream()

    def merge(pairs):  # [world, batch, k, 2]: the all-gather of every shard's pairs
        return pion_b200.merge_topk_pairs(ctx, pairs, k, descending=W.descending,
                                          lists_major=True)

    if getattr(W, "replicas", False):
        step = W.search
    elif world > 1 and wl["kind"] == "i8" and a.exchange.startswith("peer"):
        # the library's NVLink peer exchange: shared threshold sample, one call per step
        from pion_b200.sharded import PeerExchange, PeerShardedSearch
        step = PeerShardedSearch(W.ix, PeerExchange(ctx, batch, k),
                                 local_bound=a.exchange == "peer-local")
    else:
        step = ShardedSearch(W.search, k, merge, local_pairs=getattr(W, "search_pairs", None))
    workers = a.workers or (3 if wl["kind"] in ("hnsw", "quant") else 1)
    if workers > 1 and wl["kind"] not in ("hnsw", "slot", "quant"):
        raise SystemExit("--workers > 1 is for the hnsw workloads")
    ctxs = [ctx] + [pion_b200.Context(local) for _ in range(workers - 1)]
    streams = [stream] + [torch.cuda.Stream(device=dev) for _ in range(workers - 1)]

    def run_steps(n, inp):
        """n batches, worker i % workers takes batch i on its own context and stream."""
        if workers == 1:
            for _ in range(n):
                step(inp)
            return
        for st_ in streams[1:]:
            st_.wait_stream(stream)
        for i in range(n):
            w = i % workers
            with torch.cuda.stream(streams[w]):
                W.search(inp, ctx=ctxs[w])
        for st_ in streams[1:]:
            stream.wait_stream(st_)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def measure(batch, local_batch):
        """Warm-up, the timed region, the e2e region and rank 0's JSON line for one batch
        size (W's queries already set to it)."""
        inp = W.inputs()
        barrier()
        run_steps(max(3, a.warmup), inp)
        barrier()

        clocks = ClockMonitor(local)
        clocks.start()
        for c_ in ctxs:
            c_.timing(True)
        launches0 = sum(c_.launches for c_ in ctxs)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        ev0.record(stream)
        run_steps(a.steps, inp)
        ev1.record(stream)
        barrier()
        elapsed = ev0.elapsed_time(ev1)
        launches = sum(c_.launches for c_ in ctxs) - launches0
        kern_ms, kern_n = 0.0, 0
        phase_ms = {"threshold_ms": 0.0, "main_ms": 0.0, "exchange_ms": 0.0,
                    "exchange_wait_ms": 0.0}
        for c_ in ctxs:
            km, kn = c_.timing_read()
            for tag, key in ((1, "threshold_ms"), (2, "main_ms"), (3, "exchange_ms"),
                             (4, "exchange_wait_ms")):
                pm, pn = c_.timing_read(tag)
                phase_ms[key] += pm / max(1, kn)
            c_.timing(False)
            kern_ms, kern_n = kern_ms + km, kern_n + kn
        if workers > 1:  # overlapping batches: the time per batch of the whole run
            kern_ms, kern_n = elapsed, a.steps
        clk = clocks.stop()
        # per-phase device time of a few more steps: local scoring, all-gather, merge
        breakdown = None
        if isinstance(step, ShardedSearch):
            breakdown = step.breakdown(inp, max(3, min(a.steps, 20)))

        # ---- e2e: host (pinned) queries in, host results out, through the C ABI
        e2e_steps = a.e2e_steps or max(10, min(a.steps, 200))
        hin = [t.cpu().pin_memory() for t in inp]
        dbuf = [torch.empty_like(t) for t in inp]
        out_i = torch.empty((local_batch, k), dtype=torch.int32).pin_memory()
        out_v = torch.empty((local_batch, k), dtype=torch.float32).pin_memory()

        def e2e_step():
            if world == 1 or getattr(W, "replicas", False):
                # the C-ABI host-buffer path: copies, kernels, copies, sync
                W.host_call(hin, out_i, out_v)
                return
            for d, h in zip(dbuf, hin):
                d.copy_(h, non_blocking=True)
            ids, sc = step(dbuf)
            out_i.copy_(ids, non_blocking=True)
            out_v.copy_(sc, non_blocking=True)
            stream.synchronize()

        def e2e_threads(n):
            """n batches through the C ABI with host buffers, one host thread per worker
            context (each call copies in, searches and copies out, synchronously)."""
            import threading
            bufs = [([t.clone().pin_memory() for t in hin],
                     torch.empty_like(out_i).pin_memory(), torch.empty_like(out_v).pin_memory())
                    for _ in range(workers)]
            errs = []

            def work(w):
                try:
                    for i in range(w, n, workers):
                        W.host_call(bufs[w][0], bufs[w][1], bufs[w][2], ctx=ctxs[w])
                except Exception as e:  # pragma: no cover
                    errs.append(e)
            ths = [threading.Thread(target=work, args=(w,)) for w in range(workers)]
            for t_ in ths:
                t_.start()
            for t_ in ths:
                t_.join()
            if errs:
                raise errs[0]

        run_e2e = (lambda n: [e2e_step() for _ in range(n)]) if workers == 1 else e2e_threads
        run_e2e(3)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run_e2e(e2e_steps)
        e1.record(stream)
        barrier()
        e2e_ms = e0.elapsed_time(e1)
        for c_ in ctxs:  # any device-side wait that gave up (e.g. a peer's flag) fails the run
            c_.sync()
        h2d = sum(t.numel() * t.element_size() for t in hin)
        d2h = local_batch * k * 8

        # ---- max over ranks
        bd = [breakdown[x] for x in ("local_ms", "allgather_ms", "merge_ms")] if breakdown else [0.0] * 3
        t = torch.tensor([elapsed, e2e_ms, kern_ms / max(1, kern_n), phase_ms["threshold_ms"],
                          phase_ms["main_ms"], phase_ms["exchange_ms"],
                          phase_ms["exchange_wait_ms"], *bd], device=dev, dtype=torch.float64)
        lt = torch.tensor([launches], device=dev, dtype=torch.int64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dist.all_reduce(lt, op=dist.ReduceOp.SUM)
        (elapsed, e2e_ms, kern_avg_ms, thr_ms, main_ms, ex_ms, exw_ms, bd_local, bd_ag,
         bd_merge) = t.tolist()
        launches = int(lt.item())

        line = None
        if rank == 0:
            per_step = getattr(W, "queries_per_step", batch)
            qps = per_step * a.steps / (elapsed / 1000.0)
            e2e_qps = per_step * e2e_steps / (e2e_ms / 1000.0)
            peaks, peak_kind = measured_peaks()
            regime, why = choose_regime(elapsed / 1000.0, clk)
            roof = W.roofline(hi - lo, kern_avg_ms, peaks, peak_kind, regime=regime,
                              phases={"threshold_ms": thr_ms, "main_ms": main_ms,
                                      "exchange_ms": ex_ms, "exchange_wait_ms": exw_ms})
            roof["regime_reason"] = why
            roof["traffic"] = profiled_traffic(f"{a.workload}_{world}")
            line = {
                "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": elapsed / a.steps,
                "higher_is_better": True,
                "scaling": "weak" if getattr(W, "replicas", False) else "strong",
                "vs_baseline": None,
                "dtype": W.dtype, "data": "synthetic (seeded Gaussian mixture on the device)",
                "config": config_of(wl, batch, world, a),
                "e2e": {"value": e2e_qps, "unit": "queries/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "steps": e2e_steps},
                "gpu_launches": launches,
                "workers": workers,
                "roofline": roof,
                "clocks": clk,
            }
            if breakdown is not None:
                line["step_breakdown_ms"] = {
                    "local_search": bd_local, "allgather": bd_ag, "merge": bd_merge,
                    "note": "max over ranks of the per-step device time of each phase, CUDA events "
                            "over extra steps after the timed region"}
        # ---- CPU baseline on rank 0 at N=1 (bounded sample of the same workload)
        if rank == 0 and hasattr(W, "extra"):
            line["config"].update(W.extra(dev))
        if rank == 0 and world == 1 and not a.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline(W, batch, k, a.cpu_seconds)
            except Exception as e:  # pragma: no cover
                line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        if rank == 0:
            print(json.dumps(line), flush=True)

    sweep = [int(x) for x in a.batch_sweep.split(",")] if a.batch_sweep else None
    if sweep:
        if wl["kind"] != "i8":
            raise SystemExit("--batch-sweep is for the FLAT INT8 workloads")
        q_all, qs_all = W.q, W.qs
        for b in sweep:
            W.q, W.qs, W.batch = q_all[:b].contiguous(), qs_all[:b].contiguous(), b
            measure(b, b)
    else:
        measure(batch, local_batch)
    torch.cuda.synchronize()
    if world > 1:  # no rank frees its exchange buffers while a peer may still write them
        dist.barrier(device_ids=[local])
    if getattr(step, "ex", None) is not None:
        step.ex.close()
    W.ix.free()
    for c_ in ctxs[1:]:
        c_.close()
    ctx.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def cpu_baseline(W, batch, k, seconds):
    import oracle
    oracle.build()
    data = W.host_data()
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    est = min(batch, threads)
    W.cpu_run(data, 0, est, k, threads)
    qps_est = est / (time.perf_counter() - t0)
    m = int(max(est, min(batch, qps_est * seconds)))
    t0 = time.perf_counter()
    W.cpu_run(data, 0, m, k, threads)
    dt = time.perf_counter() - t0
    return {"value": m / dt, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{m} of the {batch} queries against all {W.wl['rows']:,} rows "
                      f"({dt:.1f} s, one query per thread)"}


def main(argv=None):
    a = args_parse(argv)
    wl = dict(WORKLOADS[a.workload])
    wl["ef"] = a.ef
    wl["graph_cache"] = a.graph_cache
    wl["build"] = a.build
    wl["build_batch"] = a.build_batch
    if a.rows:
        wl["rows"] = a.rows
        wl["desc"] += f" (rows overridden: {a.rows:,})"
    if a.impl == "reference":
        return run_reference(a, wl)
    return run_ours(a, wl)


if __name__ == "__main__":
    sys.exit(main())
