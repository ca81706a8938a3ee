"""bench.py's JSON-line contract, checked on the CPU through its reference arm
(``--impl reference`` times the reference's CPU algorithm and needs no GPU)."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run_reference_arm(*extra):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "0", *extra],
                         cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line_keeps_the_contract():
    line = _run_reference_arm()
    baseline = json.loads((ROOT / "BASELINE.json").read_text())
    assert line["impl"] == "reference"
    assert line["metric"] == baseline["metric"]
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert line["n_gpus"] == 1 and line["steps"] == 2
    assert line["warmup"] >= 3  # the timing rules' minimum, whatever was asked
    assert line["scaling"] == "weak" and line["data"] == "synthetic" and line["dtype"] == "bf16"
    assert "workload" in line["config"] and "model" not in line["config"]
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == line["value"] and cb["unit"] == line["unit"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
