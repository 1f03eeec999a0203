"""GPU: the ggml bridge on a llama.cpp-layout cache.

Each layer's K and V are one 2-D ggml tensor [head_dim * n_head_kv, kv_size]
(llama.cpp's unified cache with flash attention's V layout).  tria_ggml_evict
must give the same kept counts and byte-identical K, V and positions as
tria_evict on the equivalent view, for device buffers (CUDA backend) and for
page-locked host buffers (CPU backend through tria_evict_host), and refuse
pageable host memory.
"""
import numpy as np
import pytest

import tria_b200
import workloads

pytestmark = pytest.mark.gpu

L, H, KV, HD, CELLS = 3, 32, 8, 128, 3000


def _ggml_of(cache, pos, pos_shared):
    """ggml descriptors of a devcache.DeviceCache (or host tensors with its shapes)."""
    k, v = cache["k"], cache["v"]
    cell = k.shape[2]
    tk = [tria_b200.ggml_tensor(cache["type"], HD * KV, k.shape[1], cell, k[l]) for l in range(k.shape[0])]
    tv = [tria_b200.ggml_tensor(cache["type"], HD * KV, v.shape[1], cell, v[l]) for l in range(v.shape[0])]
    return tria_b200.ggml_cache(tk, tv, KV, HD, pos, pos_shared=pos_shared)


@pytest.mark.parametrize("type_id", [workloads.TYPE_F16, workloads.TYPE_Q8_0])
def test_ggml_evict_matches_tria_evict(torch_dev, tmp_path, type_id):
    import torch
    import devcache
    path = workloads.write_tria(str(tmp_path / "g.tria"), L, H, KV, HD, seed=31)
    st = tria_b200.load(path)
    try:
        ctx = tria_b200.Context(st, 0)
        src = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
        src.fill_synthetic(seed=8)
        n_rows = np.full(L * KV, CELLS, np.int32)
        n_rows[4] = 2100
        params = tria_b200.EvictParams(CELLS, 400, 100, 256, 4, 0)
        ref = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
        ctx.evict(src.view(shared_pos=True), ref.view(), n_rows, params)
        _, ref_counts = ctx.get_n_kv(L * KV)

        # device buffers: the CUDA backend
        dst = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
        sg = _ggml_of({"type": type_id, "k": src.k, "v": src.v}, src.pos_shared, True)
        dg = _ggml_of({"type": type_id, "k": dst.k, "v": dst.v}, dst.pos, False)
        ctx.ggml_evict(sg, dg, n_rows, params)
        _, counts = ctx.get_n_kv(L * KV)
        assert np.array_equal(counts, ref_counts)
        for l in range(L):
            for h in range(KV):
                m = int(counts[l * KV + h])
                sl = slice(h * src.rb, (h + 1) * src.rb)
                assert torch.equal(dst.k[l, :m, sl], ref.k[l, :m, sl]), (l, h)
                assert torch.equal(dst.v[l, :m, sl], ref.v[l, :m, sl]), (l, h)
                assert torch.equal(dst.pos[l, h, :m], ref.pos[l, h, :m]), (l, h)

        # page-locked host buffers: the CPU backend, through tria_evict_host
        hk = src.k.cpu().pin_memory()
        hv = src.v.cpu().pin_memory()
        hp = src.pos_shared.cpu().pin_memory()
        ok = torch.zeros_like(hk).pin_memory()
        ov = torch.zeros_like(hv).pin_memory()
        op = torch.zeros((L, KV, CELLS), dtype=torch.int32).pin_memory()
        hs = _ggml_of({"type": type_id, "k": hk, "v": hv}, hp, True)
        hd = _ggml_of({"type": type_id, "k": ok, "v": ov}, op, False)
        ctx.ggml_evict(hs, hd, n_rows, params)
        _, hcounts = ctx.get_n_kv(L * KV)
        assert np.array_equal(hcounts, ref_counts)
        rk, rv, rp = ref.k.cpu(), ref.v.cpu(), ref.pos.cpu()
        for l in range(L):
            for h in range(KV):
                m = int(hcounts[l * KV + h])
                sl = slice(h * src.rb, (h + 1) * src.rb)
                assert torch.equal(ok[l, :m, sl], rk[l, :m, sl]) and torch.equal(ov[l, :m, sl], rv[l, :m, sl])
                assert torch.equal(op[l, h, :m], rp[l, h, :m])

        # pageable host memory is refused before any work is queued
        pk = np.zeros(tuple(src.k.shape), np.uint8)
        pv = np.zeros(tuple(src.v.shape), np.uint8)
        bad = tria_b200.ggml_cache(
            [tria_b200.ggml_tensor(type_id, HD * KV, CELLS, src.k.shape[2], pk[l].ctypes.data) for l in range(L)],
            [tria_b200.ggml_tensor(type_id, HD * KV, CELLS, src.k.shape[2], pv[l].ctypes.data) for l in range(L)],
            KV, HD, hp, pos_shared=True)
        with pytest.raises(tria_b200.TriaError) as ei:
            ctx.ggml_evict(bad, dg, n_rows, params)
        assert ei.value.status == tria_b200.ERR_INVALID and "page-locked" in str(ei.value)
        ctx.close()
    finally:
        tria_b200.free(st)
