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
