"""bench.py's reference arm runs on the host alone (the CPU restatement of the
reference forward), so its JSON line contract can be checked without a GPU."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    proc = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", "smoke", "--steps", "1",
         "--warmup", "1"],
        capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "positions/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["warmup"] >= 3 and d["steps"] == 1
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    for key in ("metric", "n_gpus", "ms_per_step", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d
