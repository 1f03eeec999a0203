"""The reference's own C callers, unmodified, on the product library.

oracle/Makefile's `dropin` target compiles the reference's test_tria_lib.c,
test_tria_gqa.c and bench_tria.c against include/triattention.h and
libtriattention_b200.so (not triattention.c).  The loader driver needs no GPU:
its output must be the same text as the same driver built on the reference.
The scoring drivers run on the GPU (tests/test_gpu_dropin.py).
"""
import os
import subprocess

import pytest

import oracle_py
from conftest import GOLDEN


def _need(path):
    if not os.path.exists(path):
        pytest.skip(f"{os.path.basename(path)} not built (oracle/Makefile dropin needs the reference sources)")
    return path


def test_dropin_drivers_link_the_product():
    for name in ("test_tria_gqa", "test_tria_lib", "bench_tria"):
        exe = _need(oracle_py.dropin_tool(name))
        out = subprocess.run(["ldd", exe], capture_output=True, text=True, check=True).stdout
        assert "libtriattention_b200.so" in out and "not found" not in out, out
        assert "libtria_ref" not in out


@pytest.mark.parametrize("stats", ["synth_l2h8kv4.tria"])
def test_reference_loader_driver_same_output(stats):
    path = os.path.join(GOLDEN, stats)
    ours = subprocess.run([_need(oracle_py.dropin_tool("test_tria_lib")), path], capture_output=True, text=True)
    ref = subprocess.run([_need(oracle_py.ref_tool("test_tria_lib")), path], capture_output=True, text=True)
    assert ours.returncode == 0 and ref.returncode == 0
    assert ours.stdout == ref.stdout and ours.stdout.rstrip().endswith("OK")


def test_reference_loader_driver_rejects_bad_file(tmp_path):
    bad = tmp_path / "bad.tria"
    bad.write_bytes(b"NOPE" + b"\0" * 60)
    r = subprocess.run([_need(oracle_py.dropin_tool("test_tria_lib")), str(bad)], capture_output=True, text=True)
    assert r.returncode == 1
