"""`bench.py --impl reference` on the host cores: the line it prints keeps the
contract of the reference arm (same metric, unit and config as the CUDA arm,
a cpu_baseline describing the run, an e2e block with no host<->device bytes)."""
import json
import os
import subprocess
import sys

from conftest import REPO


def test_reference_arm_line():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "3"],
                       cwd=REPO, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "median HBM GB/s" and line["unit"] == "GB/s"
    assert line["higher_is_better"] is True and line["n_gpus"] == 1
    assert line["steps"] == 1 and line["warmup"] >= 3
    assert line["value"] > 0 and line["ms_per_step"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "[8192, 2048]" in line["config"]["workload"]
