"""The benchmark's reference arm (bench.py --impl reference) on the host: it
runs QuickLM's own compiled int8 path (oracle/_ref) on the same workload and
prints one JSON line with the keys the harness reads — the same metric,
unit and direction as the device arm, a cpu_baseline of kind "reference"
describing the run, and an e2e block with no host<->device bytes."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from tests.conftest import ROOT


def test_reference_arm_json_line():
    from oracle import oracle as o
    if not os.path.exists(o.REF_LIB):
        pytest.skip("oracle/_ref/libqlm_refcpu.so not built (needs the reference tree)")
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    j = json.loads(lines[0])
    assert j["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "config"):
        assert key in j, key
    assert j["unit"] == "GB/s" and j["higher_is_better"] is True and j["value"] > 0
    assert j["warmup"] >= 3
    cb = j["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == j["value"] and cb["cores"] >= 1 and cb["sample"]
    e2e = j["e2e"]
    assert e2e["value"] == j["value"] and e2e["unit"] == j["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
