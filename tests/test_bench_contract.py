"""The benchmark's reference arm keeps its JSON contract (CPU).

``bench.py --impl reference`` times the reference's own ``QuestOnlyBackend``
on the host cores and prints one JSON line on rank 0 with the same metric,
unit and direction as the GPU arm, a ``cpu_baseline`` describing the sample
and an ``e2e`` object with no host<->device bytes; other ranks print nothing
and exit 0.  It needs no GPU, so the contract is checked here with a small
sample (two of the 64 requests).
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(env_extra: dict) -> subprocess.CompletedProcess:
    env = dict(os.environ, **env_extra)
    return subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3",
         "--cpu-seconds", "0.5", "--cpu-requests", "2"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=600,
    )


def test_reference_arm_prints_one_contract_line():
    proc = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "Quest sparse-decode layer-steps/sec per GPU and box"
    assert d["unit"] == "layer-steps/s" and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 3
    assert d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and "QuestOnlyBackend" in cb["sample"]
    assert d["port"]["value"] > 0
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith("config1")


def test_reference_arm_other_ranks_exit_quietly():
    proc = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert proc.stdout.strip() == ""
