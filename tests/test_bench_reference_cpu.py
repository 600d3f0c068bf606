"""bench.py's reference arm on the CPU: it times the reference's own CPU build (oracle/_ref) on
a bounded sample of the GRPO workload and prints one JSON line with the same metric, unit,
direction and workload as the GPU arm, marked impl "reference", whose cpu_baseline describes
the run (kind, cores, sample; value = the line's) and whose e2e moves no bytes between host
and device. Skipped when the reference build is absent."""
import json
import os
import subprocess
import sys

import pytest

from oracle import ref
from tests.gpu_util import ROOT


def test_reference_arm_prints_the_contract_line():
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    # a small time budget keeps the per-step sample at its minimum (one group of 2 rollouts);
    # OMP_NUM_THREADS=1 as a launcher sets it must not leave the reference on one thread
    env["OMP_NUM_THREADS"] = "1"
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1",
                          "--reference-budget", "1"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert out.returncode == 0, out.stdout + out.stderr
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("GRPO rollout tok/s") and d["unit"] == "tok/s"
    assert d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["steps"] == 1 and d["warmup"] == 1
    assert d["config"]["workload"] == "grpo_step_mla36m"
    assert d["config"]["rollouts"] == 2048 and d["config"]["sequence"] == 384
    assert d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"] and cb["sample"]
    assert cb["cores"] == cb["host_threads"] == len(os.sched_getaffinity(0))
    assert "one group of 2 rollouts" in cb["sample"] and cb["cpu_model"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
