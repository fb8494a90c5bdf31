"""bench.py's reference arm on the CPU: one JSON line with the keys the
bench contract names, the reference's marker and a zero-copy e2e block."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
        "cpu_baseline", "e2e", "impl"}


def test_reference_arm_json_line():
    out = subprocess.run(
        [sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1",
         "--cpu-sample-slots", "2"],
        cwd=ROOT, capture_output=True, text=True, timeout=600, check=True).stdout
    lines = [ln for ln in out.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= d.keys()
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["warmup"] >= 3  # the contract's minimum, whatever was asked
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
