"""bench.py's reference arm on the CPU: the one JSON line the benchmark contract asks
for (keys, types, the reference-arm extras), and the multi-rank rule that rank 0 alone
runs and prints while the other ranks exit 0 without work. A small row sample keeps it
to seconds; the arm's arithmetic is the oracle port, tested elsewhere."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
             "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"}


def _run(env_extra: dict, *args: str) -> subprocess.CompletedProcess:
    env = dict(os.environ)
    env.update(env_extra)
    env.setdefault("CUDA_VISIBLE_DEVICES", "")
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                           "--ref-rows", "32", "--steps", "2", "--warmup", "1", *args],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    r = _run({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert BASE_KEYS <= set(d), BASE_KEYS - set(d)
    assert d["impl"] == "reference"
    assert d["n_gpus"] == 1 and d["steps"] == 2
    assert d["warmup"] >= 3  # the timing rules' minimum, whatever was asked
    assert d["value"] > 0 and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["config"]["workload"] == "flux_qkv"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "32 of 4608 token rows" in cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_do_no_work():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_reference_arm_rank0_of_two_reports_the_world():
    r = _run({"RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["n_gpus"] == 2 and "of 2" in d["cpu_baseline"]["sample"]
