"""tria_select_noalloc: selection for callers that cannot allocate device memory.

Some integrations may not call cudaMalloc when they evict (a runtime whose
pool owns the GPU memory, a memory-planned graph, a plugin host that forbids
allocation).  tria_select_noalloc serves them from a fixed static device
array instead of context scratch.  These tests drive it through the C ABI
and require its output to equal the existing tria_select's (exact equality:
this is integer index work) on two calls in a row, so a second call that
finds the first call's keys still in the shared array must not be affected.
"""
import numpy as np
import pytest

import tria_b200
import workloads

pytestmark = pytest.mark.gpu


def _case(rng, L, KV, n_cells, ties):
    scores = rng.standard_normal((L * KV, n_cells)).astype(np.float32)
    if ties:
        scores = (np.round(scores * 4) / 4).astype(np.float32)
        scores[0, :40] = np.nan
        scores[1, 10:90] = -0.0
    n_rows = rng.integers(1, n_cells + 1, L * KV).astype(np.int32)
    n_rows[0] = n_cells
    return scores, n_rows


def test_noalloc_matches_tria_select_twice(synth_stats_path):
    import torch
    import devcache
    assert torch.cuda.is_available(), "needs a CUDA device"
    if not __import__("os").path.exists(tria_b200.LIB_PATH):
        tria_b200.build()
    dev = torch.device("cuda:0")
    L, KV, hd, scales = 2, 4, 128, [0.9, 1.1]      # geometry of the synthetic stats file
    st = tria_b200.load(synth_stats_path)
    ctx = tria_b200.Context(st, 0)
    rng = np.random.default_rng(123)
    try:
        calls = [(5000, True, 64, 4, 700, 100), (3100, False, 0, 0, 300, 40)]
        for n_cells, ties, window, sink, budget, ramp in calls:
            scores, n_rows = _case(rng, L, KV, n_cells, ties)
            cur = n_cells + 7
            pos = np.stack([np.sort(rng.choice(cur, n_cells, replace=False))
                            for _ in range(L * KV)]).astype(np.int32)
            view_cache = devcache.DeviceCache(workloads.TYPE_F16, L, KV, hd, n_cells, dev, with_v=False)
            view_cache.fill_from_host(np.zeros((L, n_cells, KV * 2 * hd), np.uint8), None,
                                      pos.reshape(L, KV, n_cells))
            params = tria_b200.EvictParams(cur, budget, ramp, window, sink, 0)
            d_scores = torch.from_numpy(scores).to(dev)
            kept_ref = torch.full((L * KV, n_cells), -1, dtype=torch.int32, device=dev)
            nk_ref = torch.zeros(L * KV, dtype=torch.int32, device=dev)
            ctx.select(view_cache.view(), n_rows, d_scores, params, kept_ref, nk_ref)

            keep = np.array([workloads.layer_keep(int(n_rows[u]),
                                                  workloads.layer_budget(scales[u // KV], budget), ramp)
                             for u in range(L * KV)], np.int32)
            kept = torch.full((L * KV, n_cells), -1, dtype=torch.int32, device=dev)
            nk = torch.zeros(L * KV, dtype=torch.int32, device=dev)
            tria_b200.select_noalloc(d_scores, n_cells, n_rows, keep, kept, n_cells, nk,
                                     pos=view_cache.pos, pos_stride=n_cells, cur_pos=cur,
                                     window=window, sink=sink)
            torch.cuda.synchronize()
            nk_a, nk_b = nk.cpu().numpy(), nk_ref.cpu().numpy()
            assert np.array_equal(nk_a, nk_b)
            ka, kb = kept.cpu().numpy(), kept_ref.cpu().numpy()
            for u in range(L * KV):
                assert np.array_equal(ka[u, :nk_a[u]], kb[u, :nk_b[u]]), (n_cells, u)
        # one shared [rows] position array (pos_stride == 0), window and sink on,
        # against tria_select on a view whose positions are shared
        n_cells = 4000
        scores, n_rows = _case(rng, L, KV, n_cells, True)
        cur = n_cells + 3
        shared = np.sort(rng.choice(cur, n_cells, replace=False)).astype(np.int32)
        view_cache = devcache.DeviceCache(workloads.TYPE_F16, L, KV, hd, n_cells, dev, with_v=False)
        view_cache.fill_from_host(np.zeros((L, n_cells, KV * 2 * hd), np.uint8), None, None, shared)
        params = tria_b200.EvictParams(cur, 500, 100, 300, 8, 0)
        d_scores = torch.from_numpy(scores).to(dev)
        kept_ref = torch.full((L * KV, n_cells), -1, dtype=torch.int32, device=dev)
        nk_ref = torch.zeros(L * KV, dtype=torch.int32, device=dev)
        ctx.select(view_cache.view(shared_pos=True), n_rows, d_scores, params, kept_ref, nk_ref)
        keep = np.array([workloads.layer_keep(int(n_rows[u]), workloads.layer_budget(scales[u // KV], 500), 100)
                         for u in range(L * KV)], np.int32)
        kept = torch.full((L * KV, n_cells), -1, dtype=torch.int32, device=dev)
        nk = torch.zeros(L * KV, dtype=torch.int32, device=dev)
        tria_b200.select_noalloc(d_scores, n_cells, n_rows, keep, kept, n_cells, nk,
                                 pos=view_cache.pos_shared, pos_stride=0, cur_pos=cur, window=300, sink=8)
        torch.cuda.synchronize()
        nk_a, nk_b = nk.cpu().numpy(), nk_ref.cpu().numpy()
        assert np.array_equal(nk_a, nk_b)
        ka, kb = kept.cpu().numpy(), kept_ref.cpu().numpy()
        for u in range(L * KV):
            assert np.array_equal(ka[u, :nk_a[u]], kb[u, :nk_b[u]]), ("shared", u)
    finally:
        ctx.close()
        tria_b200.free(st)


def test_noalloc_rejects_oversize_without_launching():
    import torch
    dev = torch.device("cuda:0")
    units, n = 17, 65536                       # 17 x 65536 > 1 Mi keys
    scores = torch.zeros((units, n), device=dev)
    kept = torch.zeros((units, n), dtype=torch.int32, device=dev)
    nk = torch.zeros(units, dtype=torch.int32, device=dev)
    with pytest.raises(tria_b200.TriaError) as ei:
        tria_b200.select_noalloc(scores, n, np.full(units, n, np.int32), np.full(units, 10, np.int32),
                                 kept, n, nk)
    assert ei.value.status == tria_b200.ERR_UNSUPPORTED
    assert "scratch" in str(ei.value)
