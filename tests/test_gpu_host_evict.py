"""GPU: tria_evict_host (cache in page-locked host memory) gives the same kept
counts and the same compacted K, V and positions bytes as tria_evict on the
same cache in device memory; pageable buffers are refused before any launch."""
import numpy as np
import pytest

import tria_b200
import workloads

pytestmark = pytest.mark.gpu


def _host_view(type_id, k, v, pos, n_cells, KV, rb, shared):
    L = k.shape[0]
    return tria_b200.make_view(type_id, [k[l] for l in range(L)], [v[l] for l in range(L)] if v is not None else None,
                               pos, n_cells, KV * rb, rb, KV, 0, 0, pos_shared=shared)


@pytest.mark.parametrize("type_id,shared,window,sink", [
    (workloads.TYPE_F16, True, 0, 0),
    (workloads.TYPE_Q8_0, False, 0, 0),
    (workloads.TYPE_F16, False, 100, 4),
])
def test_evict_host_matches_device_path(torch_dev, tmp_path, type_id, shared, window, sink):
    import torch
    import devcache
    L, H, KV, hd, cells, cur, budget = 5, 32, 8, 128, 3000, 3000, 300
    path = workloads.write_tria(str(tmp_path / "h.tria"), L, H, KV, hd, seed=29)
    st = tria_b200.load(path)
    rng = np.random.default_rng(4)
    rb = workloads.row_bytes(type_id, hd)
    try:
        ctx = tria_b200.Context(st, 0)
        if type_id == workloads.TYPE_F16:
            K = workloads.f16_cache(L, cells, KV, hd, seed=1)
            V = workloads.f16_cache(L, cells, KV, hd, seed=2)
        else:
            K = workloads.q8_0_cache(L, cells, KV, hd, seed=1)
            V = workloads.q8_0_cache(L, cells, KV, hd, seed=2)
        if shared:
            pshared = np.arange(cells, dtype=np.int32)
            pos = np.broadcast_to(pshared, (L, KV, cells)).copy()
        else:
            pshared = None
            pos = np.stack([np.stack([np.sort(rng.choice(cur, cells, replace=False)) for _ in range(KV)])
                            for _ in range(L)]).astype(np.int32)
        n_rows = np.full(L * KV, cells, np.int32)
        n_rows[7] = 1234
        params = tria_b200.EvictParams(cur, budget, 100, window, sink, 0)
        # device path
        src = devcache.DeviceCache(type_id, L, KV, hd, cells, torch_dev)
        dst = devcache.DeviceCache(type_id, L, KV, hd, cells, torch_dev)
        src.fill_from_host(K, V, pos, pshared)
        ctx.evict(src.view(shared), dst.view(), n_rows, params)
        _, ref_counts = ctx.get_n_kv(L * KV)
        Kd, Vd, Pd = dst.k.cpu().numpy(), dst.v.cpu().numpy(), dst.pos.cpu().numpy()
        # host path: page-locked buffers, dst sized for the kept rows only
        cap = workloads.layer_keep(cells, budget, 100) + window + sink + 16    # the documented dst bound
        hk = torch.from_numpy(K).pin_memory()
        hv = torch.from_numpy(V).pin_memory()
        hp = torch.from_numpy(pshared if shared else pos).pin_memory()
        ok = torch.zeros((L, cap, KV * rb), dtype=torch.uint8).pin_memory()
        ov = torch.zeros_like(ok).pin_memory()
        opos = torch.full((L, KV, cap), -1, dtype=torch.int32).pin_memory()
        sv = _host_view(type_id, hk, hv, hp, cells, KV, rb, shared)
        dv = _host_view(type_id, ok, ov, opos, cap, KV, rb, False)
        ctx.evict_host(sv, dv, n_rows, params)
        _, counts = ctx.get_n_kv(L * KV)
        assert np.array_equal(counts, ref_counts)
        okn, ovn, opn = ok.numpy(), ov.numpy(), opos.numpy()
        for u in range(L * KV):
            l, h = divmod(u, KV)
            m = int(counts[u])
            assert np.array_equal(opn[l, h, :m], Pd[l, h, :m]), u
            assert np.array_equal(okn[l, :m, h * rb:(h + 1) * rb], Kd[l, :m, h * rb:(h + 1) * rb]), u
            assert np.array_equal(ovn[l, :m, h * rb:(h + 1) * rb], Vd[l, :m, h * rb:(h + 1) * rb]), u
        # a second call on the same context reuses its staging buffers
        ctx.evict_host(sv, dv, n_rows, params)
        _, counts2 = ctx.get_n_kv(L * KV)
        assert np.array_equal(counts2, ref_counts)
        ctx.close()
    finally:
        tria_b200.free(st)


def test_evict_host_refuses_pageable_memory(torch_dev, synth_stats_path):
    st = tria_b200.load(synth_stats_path)
    try:
        ctx = tria_b200.Context(st, 0)
        L, KV, cells, rb = 1, 4, 256, 256
        k = np.zeros((L, cells, KV * rb), np.uint8)
        v = np.zeros_like(k)
        pos = np.arange(cells, dtype=np.int32)
        ok = np.zeros_like(k)
        opos = np.zeros((L, KV, cells), np.int32)
        sv = tria_b200.make_view(workloads.TYPE_F16, [k[0].ctypes.data], [v[0].ctypes.data], pos.ctypes.data,
                                 cells, KV * rb, rb, KV, 0, 0, pos_shared=True)
        dv = tria_b200.make_view(workloads.TYPE_F16, [ok[0].ctypes.data], [ok[0].ctypes.data], opos.ctypes.data,
                                 cells, KV * rb, rb, KV, 0, 0)
        with pytest.raises(tria_b200.TriaError) as ei:
            ctx.evict_host(sv, dv, np.full(KV, cells, np.int32), tria_b200.EvictParams(cells, 64, 100, 0, 0, 0))
        assert ei.value.status == tria_b200.ERR_INVALID
        ctx.close()
    finally:
        tria_b200.free(st)
