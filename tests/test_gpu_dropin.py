"""GPU: the reference's own scoring drivers, unmodified, on the product library.

test_tria_gqa.c (the reference's GQA known-answer test, PASS below 1e-2
relative against the reference's Python exporter) and bench_tria.c (every
(layer, kv-head) for 256..4096 rows) are compiled against
include/triattention.h and libtriattention_b200.so; tria_score_kv_head runs on
the B200 through its cached context.
"""
import os
import subprocess

import pytest

import oracle_py
import workloads
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _need(path):
    if not os.path.exists(path):
        pytest.skip(f"{os.path.basename(path)} not built (oracle/Makefile dropin needs the reference sources)")
    return path


def test_reference_gqa_kat_passes_on_product(torch_dev):
    exe = _need(oracle_py.dropin_tool("test_tria_gqa"))
    r = subprocess.run([exe, os.path.join(GOLDEN, "synth_l2h8kv4.tria"),
                        os.path.join(GOLDEN, "kat_gqa_synth_L1KV2.bin"), "1", "2"],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout, r.stdout


def test_reference_bench_runs_on_product(torch_dev, tmp_path):
    exe = _need(oracle_py.dropin_tool("bench_tria"))
    stats = workloads.write_tria(str(tmp_path / "b.tria"), 4, 32, 8, 128, seed=3)
    r = subprocess.run([exe, stats], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    def timing_row(ln):                 # "seq_len time_ms us/head", three numbers
        t = ln.split()
        return len(t) == 3 and t[0].isdigit() and all(x.replace(".", "", 1).isdigit() for x in t[1:])
    rows = [ln.split() for ln in r.stdout.splitlines() if timing_row(ln)]
    assert [int(x[0]) for x in rows] == [256, 512, 1024, 2048, 4096], r.stdout
    assert "tria_score_kv_head:" not in r.stderr, r.stderr      # no failure message from the library
