"""``bench.py --impl reference`` on the CPU (no GPU): the reference arm's one JSON line.

The arm times the CPU restatement of the reference algorithm (``oracle/``) on a bounded sample of
configuration 5 and prints the line the driver compares with the B200 arm: the same metric, unit,
direction and workload, ``impl: reference``, a ``cpu_baseline`` describing the run and an ``e2e``
equal to the value with no host-device bytes.
"""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    j = json.loads(lines[0])
    assert j["impl"] == "reference"
    assert j["metric"].startswith("points/sec") and "config 5" in j["metric"]
    assert j["unit"] == "points/s" and j["higher_is_better"] is True
    assert j["config"]["workload"].startswith("c5:")
    assert j["steps"] == 1 and j["warmup"] == 0 and j["value"] > 0
    cb = j["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == j["value"] and cb["sample"]
    e = j["e2e"]
    assert e["value"] == j["value"] and e["unit"] == j["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
