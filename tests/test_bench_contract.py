"""The benchmark's command-line contract, checked without a GPU: the
reference arm prints one JSON line and exits 0, and a multi-GPU request
outside torchrun is refused before any device is touched."""

import json
import os
import subprocess
import sys

from mp import ROOT

ENV = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "1", "--steps", "2",
                        "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=300, env=ENV)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    # this image cannot build the reference (no UCX, no setuptools_scm)
    assert "unavailable" in line and line["unavailable"]


def test_multi_gpu_request_needs_torchrun():
    r = subprocess.run([sys.executable, "bench.py", "--gpus", "2"], cwd=ROOT, capture_output=True, text=True,
                       timeout=300, env=ENV)
    assert r.returncode != 0
    assert "launch N>1 with torchrun" in r.stdout + r.stderr
