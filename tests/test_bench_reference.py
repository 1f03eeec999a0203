"""CPU: `bench.py --impl reference` (the reference arm) prints one JSON line
with the reference's CPU rate, its bounded sample and the fields the bench
contract asks of that arm, and its run stays bounded."""
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line():
    t0 = time.time()
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "2", "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "rows/s"
    assert d["higher_is_better"] is True and d["steps"] == 2
    cb = d["cpu_baseline"]
    assert cb["cores"] >= 1 and cb["kind"] in ("reference", "port") and cb["value"] == d["value"]
    assert "rows per step" in cb["sample"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert time.time() - t0 < 300
