"""The bench's reference arm (`bench.py --impl reference`) runs on the host
cores alone, so its JSON line is checked here without a GPU: one line on
stdout carrying the metric, unit and direction of the B200 arm, the cfg5
workload, a cpu_baseline describing the run, and an e2e block with no host
copies (the CPU path reads host memory directly)."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, check=True, timeout=600,
                         cwd=str(ROOT)).stdout
    lines = [ln for ln in out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("per-op achieved HBM GB/s")
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert "cfg5" in d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["unit"] == "GB/s"
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
