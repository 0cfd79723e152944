"""bench.py's one-line JSON contract, checked on the CPU through the reference
arm (`--impl reference`: the reference's own projection code on the host
cores; the GPU arm prints the same keys and is exercised on a B200)."""
from __future__ import annotations

import json
import os
import subprocess
import sys

from common import ROOT

KEYS = ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
        "cpu_baseline", "e2e")


def test_reference_arm_prints_one_contract_line():
    import oracle
    oracle.build()  # the reference (or its restatement) the arm times
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "2", "--warmup", "3", "--cpu-seconds", "2"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for k in KEYS:
        assert k in d, k
    with open(os.path.join(ROOT, "BASELINE.json"), encoding="utf-8") as f:
        assert d["metric"] == json.load(f)["metric"]
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] >= 3
    assert d["value"] > 0 and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
