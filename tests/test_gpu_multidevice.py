"""GPU: one process driving two devices, as llama.cpp does when it splits
layers over GPUs.

Kernels whose shared memory is above the default 48 KB (the TMA scorer, the
whole-pass z-norm, the shared-memory select, the level-0 key histogram) need
their limit raised on each device's copy of the kernel.  A context on device 1
created after one on device 0 has run must give byte-identical results, and so
must the context-free key histogram called with device 1 current.  Skipped on a
box with one GPU.
"""
import numpy as np
import pytest

import tria_b200
import workloads

pytestmark = pytest.mark.gpu

L, H, KV, HD, CELLS = 2, 32, 8, 128, 20000


def _n_rows():
    n_rows = np.full(L * KV, CELLS, np.int32)
    n_rows[3] = 14000
    return n_rows


def _run(torch, path, dev, type_id, filled):
    """One eviction step and a level-0 key histogram on `dev` over a copy of
    the cache `filled`; results on the CPU."""
    import devcache
    st = tria_b200.load(path)
    try:
        ctx = tria_b200.Context(st, dev.index)
        src = devcache.DeviceCache(type_id, L, KV, HD, CELLS, dev)
        src.k.copy_(filled.k)
        src.v.copy_(filled.v)
        src.pos_shared = filled.pos_shared.to(dev)
        dst = devcache.DeviceCache(type_id, L, KV, HD, CELLS, dev)
        n_rows = _n_rows()
        params = tria_b200.EvictParams(CELLS, 3000, 100, 256, 4, 0)
        ctx.evict(src.view(shared_pos=True), dst.view(), n_rows, params)
        _, counts = ctx.get_n_kv(L * KV)
        with torch.cuda.device(dev):
            scores = torch.empty((L * KV, CELLS), dtype=torch.float32, device=dev)
            ctx.score(src.view(shared_pos=True), n_rows, CELLS, scores)
            hist = torch.zeros(65536, dtype=torch.int32, device=dev)
            tria_b200.key_histogram(scores, CELLS, n_rows, 0, 0, hist)
            torch.cuda.synchronize(dev)
        out = (counts, dst.k.cpu(), dst.v.cpu(), dst.pos.cpu(), hist.cpu())
        ctx.close()
        return out
    finally:
        tria_b200.free(st)


@pytest.mark.parametrize("type_id", [workloads.TYPE_F16, workloads.TYPE_Q8_0])
def test_second_device_matches_first(torch_dev, tmp_path, type_id):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs in one process")
    import devcache
    path = workloads.write_tria(str(tmp_path / "m.tria"), L, H, KV, HD, seed=13)
    filled = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch.device("cuda:0"))
    filled.fill_synthetic(seed=5)
    a = _run(torch, path, torch.device("cuda:0"), type_id, filled)
    b = _run(torch, path, torch.device("cuda:1"), type_id, filled)
    counts0, counts1 = a[0], b[0]
    assert np.array_equal(counts0, counts1)
    assert int(a[4].sum()) == int(_n_rows().sum()) and torch.equal(a[4], b[4])
    rb = workloads.row_bytes(type_id, HD)
    for l in range(L):
        for h in range(KV):
            m = int(counts0[l * KV + h])
            sl = slice(h * rb, (h + 1) * rb)
            assert torch.equal(a[1][l, :m, sl], b[1][l, :m, sl]), (l, h)
            assert torch.equal(a[2][l, :m, sl], b[2][l, :m, sl]), (l, h)
            assert torch.equal(a[3][l, h, :m], b[3][l, h, :m]), (l, h)
