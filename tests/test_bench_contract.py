"""The reference arm of bench.py on the host: the one JSON line the driver reads.

`bench.py --impl reference` times the reference's CPU path (the C++ restatement) on one C2 layer
per step; it runs without a GPU, so its record format is checked here. Under torchrun only rank 0
prints; the other ranks exit 0 without work.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(extra_env=None, *args):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    r = _run(None, "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    rec = json.loads(lines[0])
    baseline = json.loads((ROOT / "BASELINE.json").read_text())
    assert rec["metric"] == baseline["metric"]
    assert rec["impl"] == "reference"
    assert rec["unit"] == "GB/s" and rec["higher_is_better"] is True
    assert rec["n_gpus"] == 1 and rec["steps"] == 1 and rec["warmup"] == 0
    assert rec["value"] > 0 and rec["ms_per_step"] > 0
    assert rec["config"]["workload"].startswith("C2 ")
    cb = rec["cpu_baseline"]
    assert cb["value"] == rec["value"] and cb["unit"] == rec["unit"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert cb["cpu_model"] and cb["sample"]
    e2e = rec["e2e"]
    assert e2e["value"] == rec["value"] and e2e["unit"] == rec["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_is_silent_on_other_ranks():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"}, "--gpus", "2", "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
