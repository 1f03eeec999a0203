"""GPU: global budget across units of each sequence (multi-sequence serving).

Three sequences with different lengths and decode positions in one q8_0
geometry are scored on the device; the three-pass histogram threshold
(tria_key_histogram / tria_key_count / tria_select_key), and the one-exchange
protocol over candidates (tria_key_gather), must keep exactly the oracle's
global top-k of the same scores, and the compacted rows must be the kept
rows byte for byte.  tria_key_gather itself must return the scores at or
above a key, and report the full count when they do not fit.
"""
import numpy as np
import pytest

import global_budget as gb
import oracle_py
import tria_b200
import workloads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("protocol", ["histograms", "candidates"])
def test_global_budget_vs_oracle(torch_dev, tmp_path, protocol):
    import torch
    import devcache
    L, H, KV, hd, cells = 3, 32, 8, 128, 3000
    path = workloads.write_tria(str(tmp_path / "g.tria"), L, H, KV, hd, seed=23)
    st = tria_b200.load(path)
    rng = np.random.default_rng(9)
    try:
        ctx = tria_b200.Context(st, 0)
        seqs, caches, ks = [], [], []
        for s, (n_kv, budget) in enumerate([(2999, 200), (1200, 64), (2048, 2048)]):
            c = devcache.DeviceCache(workloads.TYPE_Q8_0, L, KV, hd, cells, torch_dev)
            c.fill_synthetic(seed=100 + s, n_rows=n_kv)
            n_rows = np.full(L * KV, n_kv, np.int32)
            n_rows[5] = n_kv // 3                        # a ragged unit
            scores = torch.empty((L * KV, cells), dtype=torch.float32, device=torch_dev)
            ctx.score(c.view(shared_pos=True), n_rows, n_kv, scores)
            kept = torch.full((L * KV, cells), -1, dtype=torch.int32, device=torch_dev)
            nk = torch.zeros(L * KV, dtype=torch.int32, device=torch_dev)
            seqs.append({"scores": scores, "stride": cells, "n_rows": n_rows, "kept_idx": kept,
                         "kept_stride": cells, "n_kept": nk})
            caches.append(c)
            ks.append(budget * L * KV)
        select = gb.global_select if protocol == "histograms" else gb.global_select_candidates
        select(seqs, ks, lambda t: t[None], gb.DeviceBackend(torch_dev), 0)
        torch.cuda.synchronize()
        for s, sq in enumerate(seqs):
            sc = sq["scores"].cpu().numpy()
            keys = [oracle_py.score_keys(sc[u, :sq["n_rows"][u]]) for u in range(L * KV)]
            exp = oracle_py.global_select(keys, ks[s])
            nk, kept = sq["n_kept"].cpu().numpy(), sq["kept_idx"].cpu().numpy()
            assert int(nk.sum()) == min(ks[s], int(sq["n_rows"].sum()))
            for u in range(L * KV):
                assert nk[u] == exp[u].size, (s, u)
                assert np.array_equal(kept[u, :nk[u]], exp[u]), (s, u)
            # compaction of the globally selected rows
            dst = devcache.DeviceCache(workloads.TYPE_Q8_0, L, KV, hd, cells, torch_dev)
            ctx.compact(caches[s].view(shared_pos=True), dst.view(), sq["n_rows"], sq["kept_idx"], sq["n_kept"])
            torch.cuda.synchronize()
            Ks, Kd = caches[s].k.cpu().numpy(), dst.k.cpu().numpy()
            rb = dst.rb
            for u in (0, 5, L * KV - 1):
                l, h = divmod(u, KV)
                m = int(nk[u])
                assert np.array_equal(Kd[l, :m, h * rb:(h + 1) * rb], Ks[l, exp[u], h * rb:(h + 1) * rb])
        ctx.close()
    finally:
        tria_b200.free(st)


def test_key_gather(torch_dev):
    """The scores whose key is >= key_min, as a multiset, and the total count
    when more than cap of them exist."""
    import torch
    rng = np.random.default_rng(17)
    units, stride = 5, 4096
    sc = rng.standard_normal((units, stride)).astype(np.float32)
    sc[1, :40] = np.nan
    sc[2, 100:300] = 0.5
    n_rows = np.array([4096, 3000, 2500, 0, 1777], np.int32)
    d_sc = torch.from_numpy(sc).to(torch_dev)
    for key_min in (0, int(oracle_py.score_keys(np.array([0.5], np.float32))[0]), 0xFFFFFFFF):
        live = [sc[u, :n_rows[u]] for u in range(units)]
        allk = np.concatenate([oracle_py.score_keys(x) for x in live])
        exp = np.sort(allk[allk >= np.uint32(key_min)])
        for cap in (len(exp) + 8, max(1, len(exp) // 3)):
            out = torch.zeros(cap, dtype=torch.float32, device=torch_dev)
            cnt = torch.zeros(1, dtype=torch.int32, device=torch_dev)
            tria_b200.key_gather(d_sc, stride, n_rows, key_min, out, cap, cnt)
            torch.cuda.synchronize()
            assert int(cnt.item()) == len(exp), (key_min, cap)
            got = oracle_py.score_keys(out.cpu().numpy()[:min(cap, len(exp))])
            if cap >= len(exp):
                assert np.array_equal(np.sort(got), exp)
            else:                                    # a subset of the qualifying keys
                assert np.isin(got, exp).all() and (got >= np.uint32(key_min)).all()

