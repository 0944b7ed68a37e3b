"""bench.py's reference arm (the CPU oracle timed on the host cores) prints its one JSON
line for the HNSW workloads on a CPU-only machine, on a reduced index."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload", ["hnsw", "hnsw_nano", "hnsw_turbo"])
def test_reference_arm_prints_its_line(workload):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--workload", workload, "--rows", "1500", "--batch", "8", "--steps", "1",
                        "--warmup", "1", "--ef", "24"],
                       capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "queries/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "queries/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["rows"] == 1500 and line["config"]["ef"] == 24
    if workload != "hnsw":
        assert line["config"]["quant"] == workload.split("_")[1]


def _bench():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_regime_follows_the_timed_region_and_clock():
    """The roofline denominator: burst for a short region or a median SM clock within 5 %
    of its maximum, sustained for a long region at a lower clock."""
    b = _bench()
    assert b.choose_regime(0.027, {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0})[0] == "burst"
    assert b.choose_regime(30.0, {"sm_mhz": 1900.0, "sm_max_mhz": 1965.0})[0] == "burst"
    assert b.choose_regime(30.0, {"sm_mhz": 1300.0, "sm_max_mhz": 1965.0})[0] == "sustained"
    peaks = {"hbm_gbs": 6551.4, "bf16_tflops": 1630.1, "bf16_tflops_sustained": 1369.2}
    assert b.tensor_peak(peaks, "burst", 2.0) == (3260.2, 3260.2, 2738.4)
    assert b.tensor_peak(peaks, "sustained", 2.0)[0] == 2738.4


def test_flat_i8_roofline_is_reproducible_from_the_line():
    """frac = 2 * dim * rows * batch / kernel_ms / peak, and the main pass's own fraction
    from its time; for one query the bound is HBM: rows * (dim + 4) bytes per search."""
    b = _bench()
    peaks = {"hbm_gbs": 6551.4, "bf16_tflops": 1630.1, "bf16_tflops_sustained": 1369.2}
    w = b.I8Workload.__new__(b.I8Workload)
    w.dim, w.batch = 1536, 1024
    r = w.roofline(1_000_000, 1.2, peaks, "measured", "burst",
                   phases={"threshold_ms": 0.06, "main_ms": 1.1})
    ops = 2.0 * 1536 * 1_000_000 * 1024
    assert r["bound"] == "tensor" and r["peak"] == 3260.2
    assert abs(r["achieved"] - ops / 1.2e-3 / 1e12) < 1e-6
    assert abs(r["frac"] - r["achieved"] / 3260.2) < 1e-9
    assert abs(r["frac_main_pass"] - ops / 1.1e-3 / 1e12 / 3260.2) < 1e-9
    w.batch = 1
    r1 = w.roofline(1_000_000, 0.25, peaks, "measured", "burst")
    assert r1["bound"] == "hbm"
    assert abs(r1["achieved"] - 1_000_000 * 1540 / 0.25e-3 / 1e9) < 1e-6
