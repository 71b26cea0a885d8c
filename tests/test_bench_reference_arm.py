"""`bench.py --impl reference` on the host cores (CPU only): the reference's own `tgc batch`
(built from its sources into oracle/_ref by the build step) times config 1 and prints one
JSON line carrying the keys the benchmark contract names for the reference arm."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "tgc")),
                    reason="oracle/_ref/tgc is built only where the reference sources are present")
def test_reference_arm_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "lr",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "latent_reasoner int8 batch rows/s (config 1)" and d["unit"] == "rows/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    base = d["cpu_baseline"]
    assert base["kind"] == "reference" and base["value"] == d["value"] and base["cores"] >= 1 and base["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith("config1")
