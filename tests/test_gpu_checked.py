"""GPU: the checked build (libtriattention_b200_checked.so, `make checked`).

Its kernels test every index and extent that comes from device data or from
the call, report a failure as TRIA_ERR_BOUNDS and skip the access; this is
the stand-in for a memory checker, which is not available on the GPU pool.

- The GPU suites run again in a child process with TRIA_B200_LIB=checked:
  every parity, configuration, ramp, post-RoPE, z-norm and global-budget test
  must pass with no check failing.
- In that child, test_bounds_check_fires hands tria_compact kept indices and
  a kept count that lie past a unit's rows and must get TRIA_ERR_BOUNDS.  The
  planted values stay inside the buffers' allocations (rows past n_rows but
  below n_cells), so nothing outside the buffers is touched even if a check
  were missing.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import tria_b200
import workloads

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def test_gpu_suites_on_checked_build(torch_dev):
    if tria_b200.checked_build():
        pytest.skip("already running on the checked build")
    if not os.path.exists(tria_b200.CHECKED_LIB_PATH):
        tria_b200.build()
    env = dict(os.environ, TRIA_B200_LIB="checked")
    cmd = [sys.executable, "-m", "pytest", os.path.join(REPO, "tests"), "-m", "gpu", "-x", "-q", "-rs",
           "-p", "no:cacheprovider",
           "--deselect", "tests/test_gpu_checked.py::test_gpu_suites_on_checked_build",
           "--ignore", os.path.join(HERE, "test_gpu_dropin.py")]
    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=1500)
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0, tail
    assert "passed" in r.stdout and " failed" not in r.stdout, tail
    assert "runs on the checked build only" not in r.stdout, tail      # the planted-index test ran


@pytest.mark.parametrize("type_id", [workloads.TYPE_F16, workloads.TYPE_Q8_0])
def test_bounds_check_fires(torch_dev, tmp_path, type_id):
    if not tria_b200.checked_build():
        pytest.skip("runs on the checked build only (TRIA_B200_LIB=checked)")
    import torch
    import devcache
    L, H, KV, HD, CELLS, ROWS = 2, 32, 8, 128, 3000, 2000
    path = workloads.write_tria(str(tmp_path / "b.tria"), L, H, KV, HD, seed=3)
    st = tria_b200.load(path)
    try:
        ctx = tria_b200.Context(st, 0)
        src = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
        src.fill_synthetic(seed=4)
        dst = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
        units = L * KV
        n_rows = np.full(units, ROWS, np.int32)
        keep = 700
        kept = torch.zeros((units, CELLS), dtype=torch.int32, device=torch_dev)
        kept[:, :keep] = torch.arange(keep, dtype=torch.int32, device=torch_dev) * 2
        n_kept = torch.full((units,), keep, dtype=torch.int32, device=torch_dev)

        # a clean call: no check fails, rows copied as asked
        ctx.compact(src.view(), dst.view(), n_rows, kept, n_kept)
        ctx.check()
        rb = workloads.row_bytes(type_id, HD)
        assert torch.equal(dst.k[1, :keep, 3 * rb:4 * rb], src.k[1, 0:2 * keep:2, 3 * rb:4 * rb])

        # a kept index past the unit's rows (inside the allocation)
        bad = kept.clone()
        bad[3, 5] = ROWS + 3
        ctx.compact(src.view(), dst.view(), n_rows, bad, n_kept)
        with pytest.raises(tria_b200.TriaError) as ei:
            ctx.check()
        assert ei.value.status == tria_b200.ERR_BOUNDS
        ctx.check()                                      # cleared

        # a kept count above the unit's rows (inside the destination)
        nk = n_kept.clone()
        nk[4] = ROWS + 1
        ctx.compact(src.view(), dst.view(), n_rows, kept, nk)
        with pytest.raises(tria_b200.TriaError) as ei:
            ctx.check()
        assert ei.value.status == tria_b200.ERR_BOUNDS

        # the context stays usable: a full step afterwards is clean
        params = tria_b200.EvictParams(ROWS, 400, 100, 64, 4, 0)
        ctx.evict(src.view(shared_pos=True), dst.view(), n_rows, params)
        _, counts = ctx.get_n_kv(units)
        assert (counts > 0).all()
        ctx.close()
    finally:
        tria_b200.free(st)
