"""GPU: scoring a cache of post-RoPE keys (TRIA_VIEW_POST_ROPE), as llama.cpp
stores them, against the oracle on the recovered pre-RoPE keys.

The cache holds k_post = s * e^{i*theta_p} * k_pre (NeoX pairs, theta_p =
fl(p * omega_f) in fp32, s = attn_scale of the stats), rounded to the cache
type.  The oracle undoes the rotation of the stored values in double
(triattention_validate_rope.py:17-28 does the same in torch), rounds the
pre-RoPE keys to fp32 and scores them with the reference arithmetic; the GPU
folds the inverse rotation into its table.  Scores must agree to 1e-4
relative or 1e-5 absolute, and a whole eviction must keep the same rows as
the oracle's selection on the oracle's scores.
"""
import numpy as np
import pytest

import tria_b200
import workloads
from test_gpu_parity import assert_scores_close

pytestmark = pytest.mark.gpu


def _rope(k_pre, pos, omega, s):
    """[n, hd] fp32 pre-RoPE keys at positions pos -> post-RoPE keys (fp32)."""
    fc = k_pre.shape[1] // 2
    ang = (pos.astype(np.float32)[:, None] * omega[None, :]).astype(np.float32).astype(np.float64)
    c, sn = np.cos(ang), np.sin(ang)
    re, im = k_pre[:, :fc].astype(np.float64), k_pre[:, fc:].astype(np.float64)
    return (s * np.concatenate([re * c - im * sn, re * sn + im * c], axis=1)).astype(np.float32)


def _unrope(k_post, pos, omega, s):
    fc = k_post.shape[1] // 2
    ang = (pos.astype(np.float32)[:, None] * omega[None, :]).astype(np.float32).astype(np.float64)
    c, sn = np.cos(ang), np.sin(ang)
    re, im = k_post[:, :fc].astype(np.float64) / s, k_post[:, fc:].astype(np.float64) / s
    return (re * c + im * sn).astype(np.float32), (im * c - re * sn).astype(np.float32)


@pytest.mark.parametrize("type_id,shared", [(workloads.TYPE_F16, True), (workloads.TYPE_Q8_0, False),
                                            (workloads.TYPE_F16, False)])
def test_post_rope_scores_vs_oracle(torch_dev, oracle, tmp_path, type_id, shared):
    import torch
    import devcache
    L, H, KV, hd, cells, cur, s = 2, 32, 8, 128, 2600, 3000, 1.25
    fc = hd // 2
    path = workloads.write_tria(str(tmp_path / "r.tria"), L, H, KV, hd, attn_scale=s, seed=31)
    st, ost = tria_b200.load(path), oracle.load(path)
    rng = np.random.default_rng(8)
    rb = workloads.row_bytes(type_id, hd)
    try:
        omega = np.ctypeslib.as_array(st.contents.omega, shape=(fc,)).astype(np.float32).copy()
        if shared:
            pos = np.broadcast_to(np.arange(cells, dtype=np.int32) + (cur - cells), (L, KV, cells)).copy()
        else:
            pos = np.stack([np.stack([np.sort(rng.choice(cur, cells, replace=False)) for _ in range(KV)])
                            for _ in range(L)]).astype(np.int32)
        k_pre = workloads.f16_values(L, cells, KV, hd, seed=3)                     # [L, n, KV, hd] fp32
        k_post = np.empty_like(k_pre)
        for l in range(L):
            for h in range(KV):
                k_post[l, :, h] = _rope(k_pre[l, :, h], pos[l, h], omega, s)
        if type_id == workloads.TYPE_F16:
            K = k_post.astype(np.float16).view(np.uint8).reshape(L, cells, -1)
        else:
            K = workloads.quantize_q8_0(k_post).reshape(L, cells, -1)
        c = devcache.DeviceCache(type_id, L, KV, hd, cells, torch_dev, with_v=False)
        c.fill_from_host(K, None, pos, pos[0, 0] if shared else None)
        view = tria_b200.make_view(type_id, [c.k[l] for l in range(L)], None, c.pos_shared if shared else c.pos,
                                   cells, KV * rb, rb, KV, 0, 0, pos_shared=shared, flags=tria_b200.VIEW_POST_ROPE)
        n_rows = np.full(L * KV, cells, np.int32)
        n_rows[3] = 1500
        ctx = tria_b200.Context(st, 0)
        scores = torch.full((L * KV, cells), float("nan"), device=torch_dev)
        ctx.score(view, n_rows, cur, scores)
        got = scores.cpu().numpy()
        for u in range(L * KV):
            l, h = divmod(u, KV)
            n = int(n_rows[u])
            rows = np.ascontiguousarray(K[l, :n, h * rb:(h + 1) * rb])
            re_q, im_q = workloads.rows_to_split(type_id, rows, hd)          # the stored (rounded) keys
            re, im = _unrope(np.concatenate([re_q, im_q], axis=1), pos[l, h, :n], omega, s)
            ref = oracle.score_kv_head(ost, np.ascontiguousarray(re), np.ascontiguousarray(im), pos[l, h, :n], cur, l, h)
            assert_scores_close(got[u, :n], ref, f"post-RoPE type={type_id} unit={u}")
        ctx.close()
    finally:
        tria_b200.free(st)
        oracle.free(ost)
