"""GPU parity: the CUDA path through the C ABI vs the reference / oracle.

Bars (from the path's spec):
  scores       |gpu - ref| <= 1e-4 * |ref|  or  |gpu - ref| <= 1e-5, every row
  kept sets    identical index sets (ties -> lower row)
  compaction   byte-identical K, V and positions
The oracle is the CPU restatement pinned bit-exactly to the compiled
reference by the CPU tests; `reflib` is the compiled reference itself.
"""
import os

import numpy as np
import pytest

import oracle_py
import tria_b200
import workloads
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

REL_TOL, ABS_TOL = 1e-4, 1e-5


def assert_scores_close(got, ref, what=""):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    ok = (d <= REL_TOL * np.abs(ref)) | (d <= ABS_TOL)
    if not ok.all():
        i = int(np.argmax(np.where(ok, 0, d)))
        raise AssertionError(f"{what}: {int((~ok).sum())} rows out of tolerance; worst row {i}: "
                             f"gpu={got[i]!r} ref={ref[i]!r} |d|={d[i]:.3g}")


def _stats_file(tmp_path_factory, name, L, H, KV, hd, theta, seed, scales=None):
    p = str(tmp_path_factory.mktemp("stats") / name)
    workloads.write_tria(p, L, H, KV, hd, rope_theta=theta, seed=seed, scales=scales)
    return p


# ---------------- reference-signature entry point ----------------

@pytest.mark.parametrize("name", ["refc_synth_L1KV2_n300.bin", "refc_synth_L0KV1_n512.bin"])
def test_score_kv_head_vs_committed_reference_output(torch_dev, synth_stats_path, name):
    d = oracle_py.read_refc(os.path.join(GOLDEN, name))
    st = tria_b200.load(synth_stats_path)
    try:
        out = tria_b200.score_kv_head(st, d["k_re"], d["k_im"], d["key_pos"], d["cur_pos"],
                                      d["layer"], d["kv_head"])
    finally:
        tria_b200.free(st)
    assert_scores_close(out, d["expected"], name)


def test_score_kv_head_vs_reference_python_gqa_golden(torch_dev, synth_stats_path):
    """test_tria_gqa.c's own criterion against the Python exporter's vector."""
    d = oracle_py.read_kat_gqa(os.path.join(GOLDEN, "kat_gqa_synth_L1KV2.bin"))
    st = tria_b200.load(synth_stats_path)
    try:
        out = tria_b200.score_kv_head(st, d["k_re"], d["k_im"], d["key_pos"], d["cur_pos"], 1, 2)
    finally:
        tria_b200.free(st)
    denom = np.where(np.abs(d["expected"]) > 1e-6, np.abs(d["expected"]), 1.0)
    assert (np.abs(out - d["expected"]) / denom).max() < 1e-2


@pytest.mark.parametrize("geom", [
    # (L, H, KV, hd, theta, n, cur_pos, layer, heads)        config-0: Qwen3-1.7B geometry
    (1, 16, 8, 128, 1e6, 4096, 4096, 0, range(8)),
    (2, 24, 4, 64, 1e7, 3000, 70000, 1, range(4)),            # hd 64, gqa 6 (27B-class stats)
    (1, 40, 8, 128, 1e6, 8192, 8192, 0, [3]),                 # gqa 5 (27B/32B-class layout)
    (1, 32, 8, 128, 1e6, 32768, 32768, 0, [0, 5]),            # config-1 rows: z-norm over 32k rows
    (1, 8, 8, 128, 1e6, 1, 1, 0, [0]),                        # gqa 1, one row
])
def test_score_kv_head_vs_oracle(torch_dev, oracle, tmp_path_factory, geom):
    L, H, KV, hd, theta, n, cur, layer, heads = geom
    path = _stats_file(tmp_path_factory, "g.tria", L, H, KV, hd, theta, seed=n)
    st, ost = tria_b200.load(path), oracle.load(path)
    rng = np.random.default_rng(n)
    try:
        for h in heads:
            k = workloads.fp32_keys(n, hd, seed=1000 * layer + h)[0]
            re, im = workloads.split_halves(k)
            if cur == n:
                pos = np.arange(n, dtype=np.int32)
            else:
                pos = np.sort(rng.choice(cur, size=n, replace=False)).astype(np.int32)
            got = tria_b200.score_kv_head(st, re, im, pos, cur, layer, h)
            ref = oracle.score_kv_head(ost, re, im, pos, cur, layer, h)
            assert_scores_close(got, ref, f"geom={geom[:5]} head={h}")
    finally:
        tria_b200.free(st)
        oracle.free(ost)


def test_score_kv_head_vs_live_reference(torch_dev, reflib, tmp_path_factory):
    path = _stats_file(tmp_path_factory, "r.tria", 2, 32, 8, 128, 1e6, seed=5)
    st, rs = tria_b200.load(path), reflib.load(path)
    try:
        k = workloads.fp32_keys(5000, 128, seed=9)[0]
        re, im = workloads.split_halves(k)
        pos = np.arange(5000, dtype=np.int32) + 123
        got = tria_b200.score_kv_head(st, re, im, pos, 6000, 1, 7)
        ref = reflib.score_kv_head(rs, re, im, pos, 6000, 1, 7)
        assert_scores_close(got, ref, "live reference")
    finally:
        tria_b200.free(st)
        reflib.free(rs)


def test_score_kv_head_negative_deltas(torch_dev, oracle, synth_stats_path):
    """Keys after cur_pos (negative deltas) are valid input for the reference."""
    st, ost = tria_b200.load(synth_stats_path), oracle.load(synth_stats_path)
    try:
        k = workloads.fp32_keys(200, 128, seed=3)[0]
        re, im = workloads.split_halves(k)
        pos = np.arange(200, dtype=np.int32) * 7
        got = tria_b200.score_kv_head(st, re, im, pos, 500, 0, 3)
        ref = oracle.score_kv_head(ost, re, im, pos, 500, 0, 3)
        assert_scores_close(got, ref, "negative deltas")
    finally:
        tria_b200.free(st)
        oracle.free(ost)


# ---------------- device path on caches ----------------

def _cache_case(torch_dev, type_id, L, KV, hd, n_cells, n_rows, cur_pos, seed, shared):
    import devcache
    c = devcache.DeviceCache(type_id, L, KV, hd, n_cells, torch_dev)
    if type_id == workloads.TYPE_F16:
        K = workloads.f16_cache(L, n_cells, KV, hd, seed=seed)
        V = workloads.f16_cache(L, n_cells, KV, hd, seed=seed + 1)
    else:
        K = workloads.q8_0_cache(L, n_cells, KV, hd, seed=seed)
        V = workloads.q8_0_cache(L, n_cells, KV, hd, seed=seed + 1)
    rng = np.random.default_rng(seed)
    if shared:
        pos_shared = np.arange(n_cells, dtype=np.int32) + (cur_pos - n_cells)
        pos = np.broadcast_to(pos_shared, (L, KV, n_cells)).copy()
    else:
        pos = np.stack([np.stack([np.sort(rng.choice(cur_pos, n_cells, replace=False))
                                  for _ in range(KV)]) for _ in range(L)]).astype(np.int32)
        pos_shared = None
    c.fill_from_host(K, V, pos, pos_shared)
    return c, K, V, pos


def _oracle_unit_scores(oracle, ost, type_id, K, pos, l, h, n, hd, cur_pos, layer0=0, head0=0):
    rb = workloads.row_bytes(type_id, hd)
    re, im = workloads.rows_to_split(type_id, np.ascontiguousarray(K[l, :n, h * rb:(h + 1) * rb]), hd)
    return oracle.score_kv_head(ost, re, im, pos[l, h, :n], cur_pos, layer0 + l, head0 + h)


@pytest.mark.parametrize("type_id,shared,n_cells", [
    (workloads.TYPE_F16, True, 2600), (workloads.TYPE_F16, False, 2600),
    (workloads.TYPE_Q8_0, True, 2600), (workloads.TYPE_Q8_0, False, 2600),
    (workloads.TYPE_F16, False, 2601),          # n_cells % 4 != 0: the general scoring kernel
])
def test_tria_score_cache_vs_oracle(torch_dev, oracle, tmp_path_factory, type_id, shared, n_cells):
    import torch
    L, H, KV, hd, cur = 3, 32, 8, 128, 4000
    path = _stats_file(tmp_path_factory, "c.tria", L, H, KV, hd, 1e6, seed=11)
    st, ost = tria_b200.load(path), oracle.load(path)
    try:
        c, K, V, pos = _cache_case(torch_dev, type_id, L, KV, hd, n_cells, None, cur, 21, shared)
        n_rows = np.full(L * KV, n_cells, np.int32)
        n_rows[5] = 1777                                     # ragged units
        n_rows[9] = 0
        ctx = tria_b200.Context(st, 0)
        scores = torch.full((L * KV, n_cells), float("nan"), device=torch_dev)
        ctx.score(c.view(shared), n_rows, cur, scores)
        torch.cuda.synchronize()
        got = scores.cpu().numpy()
        for u in range(L * KV):
            l, h = divmod(u, KV)
            n = int(n_rows[u])
            if n == 0:
                continue
            ref = _oracle_unit_scores(oracle, ost, type_id, K, pos, l, h, n, hd, cur)
            assert_scores_close(got[u, :n], ref, f"type={type_id} unit={u}")
        ctx.close()
    finally:
        tria_b200.free(st)
        oracle.free(ost)


@pytest.mark.parametrize("split", [0, 1, 3])
@pytest.mark.parametrize("seed,n_cells", [(0, 5000), (1, 5000), (2, 5000), (3, 5000), (1, 40000), (2, 70000),
                                          (3, 131000)])
def test_tria_select_exact_on_oracle_scores(torch_dev, oracle, synth_stats_path, seed, n_cells, split):
    """Selection alone: the GPU radix select on the oracle's own scores must
    return the oracle's index sets exactly (ties, NaN, signed zeros, window,
    sink), up to units of 131000 rows (several 32-row chunks per warp).  With
    8 units the default (split 0) gives each unit a cluster of 8 CTAs, split 3
    a cluster of 3 (uneven shares), split 1 one block per unit."""
    import torch
    rng = np.random.default_rng(seed)
    L, KV, hd = 2, 4, 128
    st = tria_b200.load(synth_stats_path)
    try:
        ctx = tria_b200.Context(st, 0)
        ctx.set_select_split(split)
        scores = rng.standard_normal((L * KV, n_cells)).astype(np.float32)
        if seed % 2:
            scores = (np.round(scores * 4) / 4).astype(np.float32)     # heavy ties
            scores[0, :50] = np.nan
            scores[1, 100:200] = -0.0
        n_rows = rng.integers(0, n_cells + 1, L * KV).astype(np.int32)
        n_rows[0] = n_cells
        cur = n_cells + 10
        pos = np.stack([np.sort(rng.choice(cur, n_cells, replace=False)) for _ in range(L * KV)]).astype(np.int32)
        import devcache
        c = devcache.DeviceCache(workloads.TYPE_F16, L, KV, hd, n_cells, torch_dev, with_v=False)
        c.fill_from_host(np.zeros((L, n_cells, KV * 256), np.uint8), None, pos.reshape(L, KV, n_cells))
        window, sink = (64, 4) if seed >= 2 else (0, 0)
        params = tria_b200.EvictParams(cur, 700, [100, 40, 100, 10][seed], window, sink, 0)
        d_scores = torch.from_numpy(scores).to(torch_dev)
        kept = torch.full((L * KV, n_cells), -1, dtype=torch.int32, device=torch_dev)
        nk = torch.zeros(L * KV, dtype=torch.int32, device=torch_dev)
        ctx.select(c.view(), n_rows, d_scores, params, kept, nk)
        torch.cuda.synchronize()
        kept, nk = kept.cpu().numpy(), nk.cpu().numpy()
        scales = [0.9, 1.1]
        for u in range(L * KV):
            n = int(n_rows[u])
            keep = workloads.layer_keep(n, workloads.layer_budget(scales[u // KV], 700), params.ramp_pct)
            exp = oracle.select(scores[u, :n], keep, pos[u, :n], cur, window, sink)
            assert nk[u] == exp.size, u
            assert np.array_equal(kept[u, :nk[u]], exp), u
        ctx.close()
    finally:
        tria_b200.free(st)


@pytest.mark.parametrize("type_id", [workloads.TYPE_F16, workloads.TYPE_Q8_0])
def test_evict_end_to_end_vs_oracle(torch_dev, oracle, tmp_path_factory, type_id):
    """score -> select -> compact: kept sets identical to the oracle's, compacted
    K/V/positions byte-identical to the oracle's compaction."""
    import torch
    import devcache
    L, H, KV, hd, n_cells, cur = 2, 32, 8, 128, 3000, 3000
    path = _stats_file(tmp_path_factory, "e.tria", L, H, KV, hd, 1e6, seed=13,
                       scales=np.array([1.0, 0.8], np.float32))
    st, ost = tria_b200.load(path), oracle.load(path)
    try:
        src, K, V, pos = _cache_case(torch_dev, type_id, L, KV, hd, n_cells, None, cur, 31, True)
        dst = devcache.DeviceCache(type_id, L, KV, hd, n_cells, torch_dev)
        n_rows = np.full(L * KV, n_cells, np.int32)
        n_rows[3] = 2500
        params = tria_b200.EvictParams(cur, 360, 100, 0, 0, 0)
        ctx = tria_b200.Context(st, 0)
        ctx.evict(src.view(True), dst.view(), n_rows, params)
        mx, counts = ctx.get_n_kv(L * KV)
        rb = src.rb
        Kd, Vd, Pd = dst.k.cpu().numpy(), dst.v.cpu().numpy(), dst.pos.cpu().numpy()
        for u in range(L * KV):
            l, h = divmod(u, KV)
            n = int(n_rows[u])
            sc = _oracle_unit_scores(oracle, ost, type_id, K, pos, l, h, n, hd, cur)
            keep = workloads.layer_keep(n, workloads.layer_budget([1.0, 0.8][l], 360), 100)
            exp = oracle.select(sc, keep, pos[l, h, :n], cur)
            assert counts[u] == exp.size
            assert np.array_equal(Pd[l, h, :exp.size], pos[l, h, exp]), f"kept set differs in unit {u}"
            assert np.array_equal(Kd[l, :exp.size, h * rb:(h + 1) * rb], K[l, exp, h * rb:(h + 1) * rb])
            assert np.array_equal(Vd[l, :exp.size, h * rb:(h + 1) * rb], V[l, exp, h * rb:(h + 1) * rb])
        assert mx == counts.max()
        ctx.close()
    finally:
        tria_b200.free(st)
        oracle.free(ost)


def test_position_outside_range_is_reported(torch_dev, synth_stats_path):
    """A key position beyond cur_pos is refused by a bounds check in the kernel
    (no out-of-bounds table read) and surfaces as TRIA_ERR_POSITION."""
    import devcache
    st = tria_b200.load(synth_stats_path)
    try:
        ctx = tria_b200.Context(st, 0)
        src = devcache.DeviceCache(workloads.TYPE_F16, 1, 4, 128, 256, torch_dev, layer0=1)
        dst = devcache.DeviceCache(workloads.TYPE_F16, 1, 4, 128, 256, torch_dev, layer0=1)
        src.fill_synthetic(seed=1)
        src.pos[0, 2, 17] = 10_000                       # beyond cur_pos = 256
        ctx.evict(src.view(), dst.view(), np.full(4, 256, np.int32), tria_b200.EvictParams(256, 64, 100, 0, 0, 0))
        with pytest.raises(tria_b200.TriaError) as ei:
            ctx.get_n_kv(4)
        assert ei.value.status == tria_b200.ERR_POSITION
        ctx.close()
    finally:
        tria_b200.free(st)
