"""GPU: an eviction step captured in a CUDA graph.

A serving loop evicts between decode steps with the same shapes every time,
so it can capture tria_evict once (after one eager call has sized the
context's scratch and set the kernels' attributes) and replay the graph.  The
replay must give the eager call's kept counts (through tria_get_n_kv, whose
copy-back is part of the graph and which waits for the replayed step) and
byte-identical K, V and positions, for a
fresh cache (shared positions, 2-CTA cluster selection at these few units)
and for a compacted one (per-head positions, table rows read from L2).
"""
import numpy as np
import pytest

import tria_b200
import workloads

pytestmark = pytest.mark.gpu

L, H, KV, HD, CELLS = 2, 32, 8, 128, 6000


@pytest.mark.parametrize("type_id", [workloads.TYPE_F16, workloads.TYPE_Q8_0])
def test_evict_in_cuda_graph(torch_dev, tmp_path, type_id):
    import torch
    import devcache
    path = workloads.write_tria(str(tmp_path / "cg.tria"), L, H, KV, HD, seed=41)
    st = tria_b200.load(path)
    try:
        ctx = tria_b200.Context(st, 0)
        src = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
        src.fill_synthetic(seed=6)
        n_rows = np.full(L * KV, CELLS, np.int32)
        n_rows[3] = 4100
        params = tria_b200.EvictParams(CELLS, 900, 100, 128, 4, 0)
        s = torch.cuda.Stream(device=torch_dev)
        # compacted cache for the second case: per-head positions
        mid = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
        with torch.cuda.stream(s):
            ctx.evict(src.view(shared_pos=True), mid.view(), n_rows, params, stream=s)
        _, mid_counts = ctx.get_n_kv(L * KV)
        for view, rows in ((src.view(shared_pos=True), n_rows), (mid.view(), mid_counts.astype(np.int32))):
            p = tria_b200.EvictParams(CELLS, 400, 100, 64, 4, 0)
            eager = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
            graphed = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
            with torch.cuda.stream(s):
                ctx.evict(view, eager.view(), rows, p, stream=s)       # also sizes scratch, sets attributes
            _, ref_counts = ctx.get_n_kv(L * KV)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                ctx.evict(view, graphed.view(), rows, p, stream=s)
            other = devcache.DeviceCache(type_id, L, KV, HD, CELLS, torch_dev)
            p_other = tria_b200.EvictParams(CELLS, 800, 100, 64, 4, 0)
            for _ in range(2):                                          # replays are repeatable
                # an eager step with other counts first, then the replay queued
                # behind a bounded sleep: tria_get_n_kv must wait for the replay
                with torch.cuda.stream(s):
                    ctx.evict(view, other.view(), rows, p_other, stream=s)
                _, other_counts = ctx.get_n_kv(L * KV)
                assert not np.array_equal(other_counts, ref_counts)
                with torch.cuda.stream(s):
                    torch.cuda._sleep(int(5e7))
                    g.replay()
                _, counts = ctx.get_n_kv(L * KV)
                assert np.array_equal(counts, ref_counts)
                torch.cuda.synchronize()
                for l in range(L):
                    for h in range(KV):
                        m = int(counts[l * KV + h])
                        sl = slice(h * eager.rb, (h + 1) * eager.rb)
                        assert torch.equal(graphed.k[l, :m, sl], eager.k[l, :m, sl]), (l, h)
                        assert torch.equal(graphed.v[l, :m, sl], eager.v[l, :m, sl]), (l, h)
                        assert torch.equal(graphed.pos[l, h, :m], eager.pos[l, h, :m]), (l, h)
                graphed.k.zero_()
            del g
        ctx.close()
    finally:
        tria_b200.free(st)
