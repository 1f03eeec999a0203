"""GPU: the q8_0 ramp sequence (five consecutive evictions at 10/20/40/80/100 %
of the way to the budget, new rows appended between steps), checked against
the oracle after every step: kept sets, compacted K/V bytes and positions.

This is the eviction schedule of the q8_0 workload at a size the oracle runs
in seconds: the first step sees one shared position row (a fresh cache), every
later step per-head positions (each head kept different rows).
"""
import numpy as np
import pytest

import tria_b200
import workloads

pytestmark = pytest.mark.gpu

RAMPS = (10, 20, 40, 80, 100)


def _append_rows(rng, L, KV, hd, n_new, type_id):
    if type_id == workloads.TYPE_Q8_0:
        x = rng.standard_normal((L, n_new, KV, hd), dtype=np.float32)
        return workloads.quantize_q8_0(x).reshape(L, n_new, KV, -1)
    x = rng.standard_normal((L, n_new, KV, hd), dtype=np.float32).astype(np.float16)
    return x.view(np.uint8).reshape(L, n_new, KV, -1)


@pytest.mark.parametrize("type_id", [workloads.TYPE_Q8_0, workloads.TYPE_F16])
def test_ramp_sequence_vs_oracle(torch_dev, oracle, tmp_path, type_id):
    import torch
    import devcache
    L, H, KV, hd, n0, base, n_new = 2, 32, 8, 128, 2048, 128, 64
    scales = np.array([1.0, 0.8], np.float32)
    path = workloads.write_tria(str(tmp_path / "ramp.tria"), L, H, KV, hd, scales=scales, seed=17)
    st, ost = tria_b200.load(path), oracle.load(path)
    rng = np.random.default_rng(5)
    cap = n0 + len(RAMPS) * n_new
    rb = workloads.row_bytes(type_id, hd)
    try:
        ctx = tria_b200.Context(st, 0)
        bufs = [devcache.DeviceCache(type_id, L, KV, hd, cap, torch_dev) for _ in range(2)]
        # host mirror per unit: rows (bytes) and positions
        k0 = _append_rows(rng, L, KV, hd, n0, type_id)
        v0 = _append_rows(rng, L, KV, hd, n0, type_id)
        hk = [[k0[l, :, h].copy() for h in range(KV)] for l in range(L)]
        hv = [[v0[l, :, h].copy() for h in range(KV)] for l in range(L)]
        hp = [[np.arange(n0, dtype=np.int32) for _ in range(KV)] for _ in range(L)]
        src = bufs[0]
        kfill = np.zeros((L, cap, KV * rb), np.uint8)
        kfill[:, :n0] = k0.reshape(L, n0, -1)
        vfill = np.zeros_like(kfill)
        vfill[:, :n0] = v0.reshape(L, n0, -1)
        pfill = np.zeros((L, KV, cap), np.int32)
        pfill[:, :, :n0] = np.arange(n0, dtype=np.int32)
        shared = np.zeros(cap, np.int32)
        shared[:n0] = np.arange(n0, dtype=np.int32)
        src.fill_from_host(kfill, vfill, pfill, shared)
        n_rows = np.full(L * KV, n0, np.int32)
        cur = n0
        for step, ramp in enumerate(RAMPS):
            dst = bufs[1] if src is bufs[0] else bufs[0]
            params = tria_b200.EvictParams(cur, base, ramp, 0, 0, 0)
            ctx.evict(src.view(shared_pos=(step == 0)), dst.view(), n_rows, params)
            _, counts = ctx.get_n_kv(L * KV)
            Kd, Vd, Pd = dst.k.cpu().numpy(), dst.v.cpu().numpy(), dst.pos.cpu().numpy()
            for u in range(L * KV):
                l, h = divmod(u, KV)
                rows_k = np.ascontiguousarray(hk[l][h])
                re, im = workloads.rows_to_split(type_id, rows_k, hd)
                sc = oracle.score_kv_head(ost, re, im, hp[l][h], cur, l, h)
                keep = workloads.layer_keep(len(hp[l][h]), workloads.layer_budget(scales[l], base), ramp)
                exp = oracle.select(sc, keep, hp[l][h], cur)
                assert counts[u] == exp.size, (step, u)
                hk[l][h], hv[l][h], hp[l][h] = hk[l][h][exp], hv[l][h][exp], hp[l][h][exp]
                m = exp.size
                assert np.array_equal(Pd[l, h, :m], hp[l][h]), f"step {step} unit {u}: kept set"
                assert np.array_equal(Kd[l, :m, h * rb:(h + 1) * rb], hk[l][h]), f"step {step} unit {u}: K"
                assert np.array_equal(Vd[l, :m, h * rb:(h + 1) * rb], hv[l][h]), f"step {step} unit {u}: V"
            # decode n_new more tokens: rows appended after each unit's kept rows
            kn = _append_rows(rng, L, KV, hd, n_new, type_id)
            vn = _append_rows(rng, L, KV, hd, n_new, type_id)
            newpos = np.arange(cur, cur + n_new, dtype=np.int32)
            for u in range(L * KV):
                l, h = divmod(u, KV)
                m = int(counts[u])
                dst.k[l, m:m + n_new, h * rb:(h + 1) * rb] = torch.from_numpy(kn[l, :, h].copy()).to(torch_dev)
                dst.v[l, m:m + n_new, h * rb:(h + 1) * rb] = torch.from_numpy(vn[l, :, h].copy()).to(torch_dev)
                dst.pos[l, h, m:m + n_new] = torch.from_numpy(newpos).to(torch_dev)
                hk[l][h] = np.concatenate([hk[l][h], kn[l, :, h]])
                hv[l][h] = np.concatenate([hv[l][h], vn[l, :, h]])
                hp[l][h] = np.concatenate([hp[l][h], newpos])
                n_rows[u] = m + n_new
            cur += n_new
            src = dst
        ctx.close()
    finally:
        tria_b200.free(st)
        oracle.free(ost)
