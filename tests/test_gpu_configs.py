"""GPU parity on the benched workloads and on every scoring-kernel variant.

The reference's per-(layer, kv-head) result (triattention.c:198-253) is what
every case must match:
  - every gqa the scoring kernels are built for (1, 2, 4, 5, 6), for fresh
    caches (one shared position row: table rows staged with the K tile) and
    compacted ones (per-head positions: table rows read from L2), f16 and
    q8_0, with stats of 64 layers read at the last layers;
  - the benched workloads at full size, with the oracle checking a sample of
    units spread over the layers (including the last ones):
      qwen3-8b-f16-32k   36 x 8 x 32768 f16, 12 % budget;
      qwen3-8b-q8_0-64k  36 x 8 x 65536 q8_0, budget 512, ramp 10 % and 100 %;
      27b-f16-64k        64 x 8 x 65536 f16, gqa 5, 12 % budget;
      multiseq-q8_0-global  8 sequences x 36 x 8 in one q8_0 cache, one
                         global budget per sequence;
  - the destination outside the kept rows is never written: every test here
    fills dst with a poison pattern first and checks it survives.
Bars: z-scores within 1e-4 relative or 1e-5 absolute of the oracle (itself
bit-identical to the compiled reference), kept sets identical, compacted K,
V and positions byte-identical.
"""
import numpy as np
import pytest

import oracle_py
import tria_b200
import workloads
from test_gpu_parity import _cache_case, assert_scores_close

pytestmark = pytest.mark.gpu

POISON = 0xA5                   # fill byte of every destination before a step
POISON_POS = -0x5A5A5A5B        # int32 with every byte 0xA5


def _stats(tmp_path, name, L, H, KV, hd=128, seed=0, scales=None):
    return workloads.write_tria(str(tmp_path / name), L, H, KV, hd, rope_theta=1e6, seed=seed, scales=scales)


def _poisoned_dst(torch_dev, type_id, L, KV, hd, cells, layer0=0):
    import devcache
    d = devcache.DeviceCache(type_id, L, KV, hd, cells, torch_dev, layer0=layer0)
    d.k.fill_(POISON)
    d.v.fill_(POISON)
    d.pos.fill_(POISON_POS)
    return d


def _check_unit(oracle, ost, type_id, hd, Ku, Vu, pos_u, n, cur, layer, head, keep, dst, l, h, count,
                got_scores=None, window=0, sink=0):
    """One unit against the oracle: z-scores (optional), kept set, compacted
    bytes, and poison beyond the kept rows of this head."""
    rb = workloads.row_bytes(type_id, hd)
    re, im = workloads.rows_to_split(type_id, Ku[:n], hd)
    sc = oracle.score_kv_head(ost, re, im, pos_u[:n], cur, layer, head)
    if got_scores is not None:
        assert_scores_close(got_scores[:n], sc, f"layer {layer} head {head}")
    exp = oracle.select(sc, keep, pos_u[:n], cur, window, sink)
    assert count == exp.size, (layer, head, count, exp.size)
    m = exp.size
    Pd = dst.pos[l, h].cpu().numpy()
    Kd = dst.k[l, :, h * rb:(h + 1) * rb].cpu().numpy()
    Vd = dst.v[l, :, h * rb:(h + 1) * rb].cpu().numpy()
    assert np.array_equal(Pd[:m], pos_u[exp]), f"kept set differs, layer {layer} head {head}"
    assert np.array_equal(Kd[:m], Ku[exp]), f"K bytes differ, layer {layer} head {head}"
    assert np.array_equal(Vd[:m], Vu[exp]), f"V bytes differ, layer {layer} head {head}"
    assert (Pd[m:] == POISON_POS).all(), f"positions written beyond kept rows, layer {layer} head {head}"
    assert (Kd[m:] == POISON).all(), f"K written beyond kept rows, layer {layer} head {head}"
    assert (Vd[m:] == POISON).all(), f"V written beyond kept rows, layer {layer} head {head}"


# ---------------- every scoring-kernel variant ----------------

@pytest.mark.parametrize("H,type_id,shared", [
    (8, workloads.TYPE_F16, True), (8, workloads.TYPE_F16, False),           # gqa 1: 32- / 16-cell tiles
    (16, workloads.TYPE_F16, True), (16, workloads.TYPE_Q8_0, False),        # gqa 2
    (40, workloads.TYPE_F16, True), (40, workloads.TYPE_F16, False),         # gqa 5 (27B-class layout)
    (40, workloads.TYPE_Q8_0, True), (40, workloads.TYPE_Q8_0, False),
    (48, workloads.TYPE_F16, True), (48, workloads.TYPE_F16, False),         # gqa 6
])
def test_evict_every_gqa_vs_oracle(torch_dev, oracle, tmp_path, H, type_id, shared):
    """Scores, kept sets and compacted bytes of the last two layers of a
    64-layer stats file (stats lookup at high layer indices), ragged units."""
    import torch
    L_stats, L, KV, hd, n_cells, cur = 64, 2, 8, 128, 1800, 2600
    layer0 = L_stats - L
    scales = np.linspace(0.7, 1.3, L_stats).astype(np.float32)
    path = _stats(tmp_path, "g.tria", L_stats, H, KV, seed=H, scales=scales)
    st, ost = tria_b200.load(path), oracle.load(path)
    try:
        src, K, V, pos = _cache_case(torch_dev, type_id, L, KV, hd, n_cells, None, cur, 40 + H, shared)
        src.layer0 = layer0
        n_rows = np.full(L * KV, n_cells, np.int32)
        n_rows[3] = 1001
        n_rows[12] = 7
        ctx = tria_b200.Context(st, 0)
        scores = torch.full((L * KV, n_cells), float("nan"), device=torch_dev)
        ctx.score(src.view(shared), n_rows, cur, scores)
        ctx.check()
        got = scores.cpu().numpy()
        dst = _poisoned_dst(torch_dev, type_id, L, KV, hd, n_cells, layer0)
        budget = 300
        params = tria_b200.EvictParams(cur, budget, 100, 0, 0, 0)
        ctx.evict(src.view(shared), dst.view(), n_rows, params)
        _, counts = ctx.get_n_kv(L * KV)
        rb = src.rb
        for u in range(L * KV):
            l, h = divmod(u, KV)
            n = int(n_rows[u])
            keep = workloads.layer_keep(n, workloads.layer_budget(scales[layer0 + l], budget), 100)
            _check_unit(oracle, ost, type_id, hd, np.ascontiguousarray(K[l, :, h * rb:(h + 1) * rb]),
                        np.ascontiguousarray(V[l, :, h * rb:(h + 1) * rb]), pos[l, h], n, cur, layer0 + l, h,
                        keep, dst, l, h, int(counts[u]), got_scores=got[u])
        ctx.close()
    finally:
        tria_b200.free(st)
        oracle.free(ost)


def test_evict_window_sink_ragged_poison(torch_dev, oracle, tmp_path):
    """Protected rows make the kept counts differ per head; rows past each
    head's count must keep the poison (per-head positions, f16)."""
    L, H, KV, hd, n_cells, cur = 2, 32, 8, 128, 2400, 5000
    path = _stats(tmp_path, "w.tria", L, H, KV, seed=77)
    st, ost = tria_b200.load(path), oracle.load(path)
    try:
        src, K, V, pos = _cache_case(torch_dev, workloads.TYPE_F16, L, KV, hd, n_cells, None, cur, 91, False)
        dst = _poisoned_dst(torch_dev, workloads.TYPE_F16, L, KV, hd, n_cells)
        n_rows = np.full(L * KV, n_cells, np.int32)
        n_rows[1] = 1500
        params = tria_b200.EvictParams(cur, 200, 100, 700, 30, 0)
        ctx = tria_b200.Context(st, 0)
        ctx.evict(src.view(False), dst.view(), n_rows, params)
        _, counts = ctx.get_n_kv(L * KV)
        assert len(set(counts.tolist())) > 1          # ragged counts
        rb = src.rb
        for u in range(L * KV):
            l, h = divmod(u, KV)
            keep = workloads.layer_keep(int(n_rows[u]), 200, 100)
            _check_unit(oracle, ost, workloads.TYPE_F16, hd, np.ascontiguousarray(K[l, :, h * rb:(h + 1) * rb]),
                        np.ascontiguousarray(V[l, :, h * rb:(h + 1) * rb]), pos[l, h], int(n_rows[u]), cur, l, h,
                        keep, dst, l, h, int(counts[u]), window=700, sink=30)
        ctx.close()
    finally:
        tria_b200.free(st)
        oracle.free(ost)


# ---------------- the benched workloads at full size ----------------

def _full_size(torch_dev, oracle, tmp_path, type_id, L, H, KV, n, budget, ramps, sample, seed):
    import torch
    import devcache
    hd = 128
    path = _stats(tmp_path, "full.tria", L, H, KV, seed=0)
    st, ost = tria_b200.load(path), oracle.load(path)
    try:
        ctx = tria_b200.Context(st, 0)
        src = devcache.DeviceCache(type_id, L, KV, hd, n, torch_dev)
        src.fill_synthetic(seed=seed)
        n_rows = np.full(L * KV, n, np.int32)
        pos = np.arange(n, dtype=np.int32)
        rb = src.rb
        scores = torch.empty((L * KV, n), dtype=torch.float32, device=torch_dev)
        ctx.score(src.view(True), n_rows, n, scores)
        ctx.check()
        dst = _poisoned_dst(torch_dev, type_id, L, KV, hd, n)
        host = {}
        for u in sample:
            l, h = divmod(u, KV)
            host[u] = (src.k[l, :, h * rb:(h + 1) * rb].cpu().numpy(), src.v[l, :, h * rb:(h + 1) * rb].cpu().numpy(),
                       scores[u].cpu().numpy())
        for t, ramp in enumerate(ramps):
            if t:
                dst.k.fill_(POISON)
                dst.v.fill_(POISON)
                dst.pos.fill_(POISON_POS)
            ctx.evict(src.view(True), dst.view(), n_rows, tria_b200.EvictParams(n, budget, ramp, 0, 0, 0))
            _, counts = ctx.get_n_kv(L * KV)
            keep = workloads.layer_keep(n, budget, ramp)
            assert (counts == keep).all(), (ramp, counts[:8], keep)
            for u in sample:
                l, h = divmod(u, KV)
                Ku, Vu, su = host[u]
                _check_unit(oracle, ost, type_id, hd, Ku, Vu, pos, n, n, l, h, keep, dst, l, h, int(counts[u]),
                            got_scores=su if t == 0 else None)
        ctx.close()
    finally:
        tria_b200.free(st)
        oracle.free(ost)


def test_qwen3_8b_f16_32k_full_size_sampled(torch_dev, oracle, tmp_path):
    """The default bench step: 36 x 8 x 32768 f16, gqa 4, budget 12 %."""
    sample = [0, 7, 8 * 9 + 3, 8 * 17 + 5, 8 * 18, 8 * 27 + 6, 8 * 34 + 2, 8 * 35, 8 * 35 + 7]
    _full_size(torch_dev, oracle, tmp_path, workloads.TYPE_F16, 36, 32, 8, 32768, int(32768 * 12 / 100),
               (100,), sample, seed=1000)


def test_qwen3_8b_q8_0_64k_full_size_sampled(torch_dev, oracle, tmp_path):
    """36 x 8 x 65536 q8_0, budget 512: the first ramp stage (10 %: 59034 rows
    kept) and the last (100 %: 512 kept) from the same cache."""
    sample = [0, 8 * 11 + 4, 8 * 23 + 1, 8 * 35 + 7]
    _full_size(torch_dev, oracle, tmp_path, workloads.TYPE_Q8_0, 36, 32, 8, 65536, 512, (10, 100), sample, seed=2000)


def test_27b_f16_64k_full_size_sampled(torch_dev, oracle, tmp_path):
    """64 x 8 x 65536 f16, gqa 5 (H = 40), budget 12 %."""
    sample = [0, 8 * 31 + 5, 8 * 63, 8 * 63 + 7]
    _full_size(torch_dev, oracle, tmp_path, workloads.TYPE_F16, 64, 40, 8, 65536, int(65536 * 12 / 100),
               (100,), sample, seed=3000)


def test_multiseq_global_budget_full_size(torch_dev, oracle, tmp_path):
    """Eight sequences of up to 16384 rows in one 36 x 8 q8_0 cache, n_kv ~
    U[8192, 16384], one global budget of 512 rows per unit per sequence: the
    kept sets must be each sequence's global top-K under the oracle's rule,
    the z-scores of sampled units must match the oracle, and the compacted
    rows must be the kept rows byte for byte."""
    import torch
    import devcache
    import global_budget as gb
    L, H, KV, hd, cells, n_seq = 36, 32, 8, 128, 16384, 8
    path = _stats(tmp_path, "ms.tria", L, H, KV, seed=0)
    st, ost = tria_b200.load(path), oracle.load(path)
    rng = np.random.default_rng(77)
    n_kv = rng.integers(cells // 2, cells + 1, n_seq).astype(np.int32)
    try:
        ctx = tria_b200.Context(st, 0)
        src = devcache.DeviceCache(workloads.TYPE_Q8_0, L, KV, hd, cells * n_seq, torch_dev)
        src.fill_synthetic(seed=900)
        src.pos_shared = torch.arange(cells, dtype=torch.int32, device=torch_dev).repeat(n_seq)
        rb = src.rb
        seqs, views, k_total = [], [], []
        for q in range(n_seq):
            sl = slice(q * cells, (q + 1) * cells)
            v = tria_b200.make_view(workloads.TYPE_Q8_0, [src.k[l][sl] for l in range(L)],
                                    [src.v[l][sl] for l in range(L)], src.pos_shared[sl], cells, KV * rb, rb, KV,
                                    pos_shared=True)
            views.append(v)
            nr = np.full(L * KV, n_kv[q], np.int32)
            sc = torch.empty((L * KV, cells), dtype=torch.float32, device=torch_dev)
            ctx.score(v, nr, int(n_kv[q]), sc)
            seqs.append({"scores": sc, "stride": cells, "n_rows": nr,
                         "kept_idx": torch.full((L * KV, cells), -1, dtype=torch.int32, device=torch_dev),
                         "kept_stride": cells, "n_kept": torch.zeros(L * KV, dtype=torch.int32, device=torch_dev)})
            k_total.append(512 * L * KV)
        ctx.check()
        gb.global_select(seqs, k_total, lambda t: t[None], gb.DeviceBackend(torch_dev), 0)
        pos = np.arange(cells, dtype=np.int32)
        for q in range(n_seq):
            sq = seqs[q]
            n = int(n_kv[q])
            sc = sq["scores"].cpu().numpy()
            exp = oracle_py.global_select([oracle_py.score_keys(sc[u, :n]) for u in range(L * KV)], k_total[q])
            nk, kept = sq["n_kept"].cpu().numpy(), sq["kept_idx"].cpu().numpy()
            assert int(nk.sum()) == k_total[q]
            for u in range(L * KV):
                assert nk[u] == exp[u].size, (q, u)
                assert np.array_equal(kept[u, :nk[u]], exp[u]), (q, u)
            dst = _poisoned_dst(torch_dev, workloads.TYPE_Q8_0, L, KV, hd, cells)
            ctx.compact(views[q], dst.view(), sq["n_rows"], sq["kept_idx"], sq["n_kept"])
            for u in (q * 37 % (L * KV), L * KV - 1 - q):
                l, h = divmod(u, KV)
                Ku = src.k[l, q * cells:(q + 1) * cells, h * rb:(h + 1) * rb].cpu().numpy()
                Vu = src.v[l, q * cells:(q + 1) * cells, h * rb:(h + 1) * rb].cpu().numpy()
                re, im = workloads.rows_to_split(workloads.TYPE_Q8_0, Ku[:n], hd)
                ref = oracle.score_kv_head(ost, re, im, pos[:n], n, l, h)
                assert_scores_close(sc[u, :n], ref, f"sequence {q} unit {u}")
                m = int(nk[u])
                Kd = dst.k[l, :, h * rb:(h + 1) * rb].cpu().numpy()
                Vd = dst.v[l, :, h * rb:(h + 1) * rb].cpu().numpy()
                Pd = dst.pos[l, h].cpu().numpy()
                assert np.array_equal(Kd[:m], Ku[exp[u]]) and np.array_equal(Vd[:m], Vu[exp[u]])
                assert np.array_equal(Pd[:m], exp[u])
                assert (Kd[m:] == POISON).all() and (Pd[m:] == POISON_POS).all()
            del dst
        ctx.close()
    finally:
        tria_b200.free(st)
        oracle.free(ost)
