"""bench.py's reference arm (`--impl reference`) on the CPU: one step of config 1 prints the
driver's JSON line (metric, value, the cpu_baseline and e2e objects the contract asks for) and
imports nothing from the GPU package, so the arm cannot load its library."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = r"""
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1", "--config", "conv1"]
try:
    runpy.run_path("bench.py", run_name="__main__")
except SystemExit as e:
    if e.code not in (None, 0):
        raise
print("PACKAGE_IMPORTED", any(m == "zenjpegai_b200" or m.startswith("zenjpegai_b200.")
                              for m in sys.modules))
"""


def test_reference_arm_line_and_isolation():
    r = subprocess.run([sys.executable, "-c", _CHILD], cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] and d["unit"] and d["value"] > 0 and d["steps"] == 1
    assert d["higher_is_better"] is True
    assert d["config"]["workload"].startswith("conv1")
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert "PACKAGE_IMPORTED False" in r.stdout
